/* gda_barrier_proxy.h -- the header name under which the reference's proxy-barrier programs
 * include the proxy barrier calls (gda_proxy_barrier_alloc / _get_dev / _get_stats / _free,
 * gda_proxy_start / _stop, device gda_gpu_proxy_barrier_wait); they are declared in gda.h. */
#pragma once

#include "gda.h"
