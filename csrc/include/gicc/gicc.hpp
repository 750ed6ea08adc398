// gicc.hpp -- the host API in one include, under the name the reference's programs use
// (#include <gicc/gicc.hpp>): Runtime (symmetric memory, exchange, device contexts, host-queued
// puts), Barrier, Bootstrap, the host collectives, active messages, the command ring, the
// NVSHMEM-style API, configuration and the fused operations.
#pragma once

#include "gicc/am.hpp"
#include "gicc/api.hpp"
#include "gicc/barrier.hpp"
#include "gicc/bootstrap.hpp"
#include "gicc/cmdring.hpp"
#include "gicc/coll.hpp"
#include "gicc/config.hpp"
#include "gicc/error.hpp"
#include "gicc/ops.hpp"
#include "gicc/runtime.hpp"
#include "gicc/types.hpp"
