// gicc_types.hpp -- the reference's name for the shared host/device types (Buffer,
// RemoteBufferInfo, DeviceCtx, GiccContext, BarrierCtx, limits); they live in gicc/types.hpp.
#pragma once

#include "gicc/types.hpp"
