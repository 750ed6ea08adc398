// visibility.hpp -- export macros of libgicc.so (built with -fvisibility=hidden).
#pragma once
#define GICC_API extern "C" __attribute__((visibility("default")))
#define GICC_EXPORT __attribute__((visibility("default")))
