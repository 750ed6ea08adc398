// gicc_device.cuh -- the device API in one include, under the name the reference's kernels
// use (#include <gicc/gicc_device.cuh>): put / get / put_no_db / flush / quiet on a
// DeviceCtx or GiccContext, put_signal and bounded signal waits, the device barrier, and the
// active-message device calls.
#pragma once

#include "gicc/device/am.cuh"
#include "gicc/device/comm.cuh"
