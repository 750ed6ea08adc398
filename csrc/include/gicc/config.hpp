// config.hpp -- every GICC_* environment knob in one validated struct, a rank-prefixed
// logger and NVTX ranges for the host API.
//
// The reference reads its environment ad hoc (GICC_IB_DEV, GICC_MTU, GICC_GID_INDEX,
// GICC_DEBUG, GICC_DISABLE_IPC: ibv_context.hpp:139-361, comm.hpp:182-389) and prints
// with printf.  Here the variables that exist on an NVLink node are parsed once, range
// checked (a bad value is an error naming the variable, not a silent default), and the
// summary is printed by rank 0 at runtime start when GICC_LOG_LEVEL >= info.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

#include "gicc/visibility.hpp"

namespace gicc {

enum LogLevel : int { LOG_ERROR = 0, LOG_WARN = 1, LOG_INFO = 2, LOG_DEBUG = 3 };

struct GICC_EXPORT Config {
  uint64_t timeout_ms = 5000;            // GICC_TIMEOUT_MS: bound of every device wait [1, 3600000]
  uint64_t bootstrap_timeout_ms = 0;     // GICC_BOOTSTRAP_TIMEOUT_MS: 0 = 120 s [100, 86400000]
  int log_level = LOG_WARN;              // GICC_LOG_LEVEL: error | warn | info | debug | 0..3
  bool checks = false;                   // GICC_CHECKS: bounds-check every device put
  bool disable_nvls = false;             // GICC_DISABLE_NVLS: never bind multicast objects
  bool debug_puts = false;               // GICC_DEBUG: log every host-initiated transfer
  size_t signal_heap_bytes = 0;          // GICC_SIGNAL_HEAP_BYTES: 0 = the RuntimeOptions value [64 KiB, 1 GiB]
  int gemm_group_m = 16;                 // GICC_GEMM_GROUP_M: m-blocks per raster group of gemm_bf16 [1, 1024]
  int gemm_l2_hint = 0;                  // GICC_GEMM_L2_HINT: 0 none, 1 keep A / stream B, 2 the reverse
  int gemm_pair_group_m = 16;            // GICC_GEMM_PAIR_GROUP_M: the CTA-pair kernel's raster group [1, 1024]
  int gemm_pair_l2_hint = 0;             // GICC_GEMM_PAIR_L2_HINT: as GICC_GEMM_L2_HINT, for the CTA-pair kernel
  int gemm_pair_prefetch = 0;            // GICC_GEMM_PAIR_PREFETCH: L2 prefetch distance in k-steps [0, 64], 0 off
  int gemm_pair_tma_store = 1;           // GICC_GEMM_PAIR_TMA_STORE: 1 = bf16 C through shared memory and TMA, 0 = per thread

  // Parses the environment now; throws std::invalid_argument naming the bad variable.
  static Config from_env();
  std::string summary() const;
};

// The configuration as the environment says now (parsed on every call: it is read at
// runtime start and by the rare paths that depend on it, so changes before a Runtime is
// built take effect).
GICC_EXPORT Config config();

// "[gicc r<rank>] <message>" on stderr when level <= GICC_LOG_LEVEL.
GICC_EXPORT void set_log_rank(int rank);
GICC_EXPORT void log(int level, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Scoped NVTX range (domain "gicc") around a host API call; free when no tool is attached.
class GICC_EXPORT NvtxRange {
 public:
  explicit NvtxRange(const char* name);
  ~NvtxRange();
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace gicc
