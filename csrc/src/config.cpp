// config.cpp -- environment parsing, logger, NVTX ranges (see gicc/config.hpp).
#include "gicc/config.hpp"

#include <nvtx3/nvToolsExt.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>

namespace gicc {
namespace {

bool parse_u64(const char* name, uint64_t lo, uint64_t hi, uint64_t* out) {
  const char* s = std::getenv(name);
  if (!s || !*s) return false;
  char* end = nullptr;
  const unsigned long long v = std::strtoull(s, &end, 0);
  if (end == s || *end != '\0' || s[0] == '-')
    throw std::invalid_argument(std::string(name) + "=" + s + ": not a non-negative integer");
  if (v < lo || v > hi)
    throw std::invalid_argument(std::string(name) + "=" + s + ": outside [" + std::to_string(lo) + ", " +
                                std::to_string(hi) + "]");
  *out = v;
  return true;
}

bool parse_bool(const char* name, bool* out) {
  const char* s = std::getenv(name);
  if (!s) return false;
  if (!*s || !std::strcmp(s, "1") || !strcasecmp(s, "true") || !strcasecmp(s, "yes") || !strcasecmp(s, "on")) {
    *out = true;  // set but empty counts as on, like the reference's presence checks
  } else if (!std::strcmp(s, "0") || !strcasecmp(s, "false") || !strcasecmp(s, "no") || !strcasecmp(s, "off")) {
    *out = false;
  } else {
    throw std::invalid_argument(std::string(name) + "=" + s + ": expected 0/1/true/false");
  }
  return true;
}

const char* level_name(int l) {
  switch (l) {
    case LOG_ERROR: return "error";
    case LOG_WARN: return "warn";
    case LOG_INFO: return "info";
    default: return "debug";
  }
}

int g_rank = -1;
nvtxDomainHandle_t g_domain = nullptr;
std::once_flag g_domain_once;

}  // namespace

Config Config::from_env() {
  Config c;
  parse_u64("GICC_TIMEOUT_MS", 1, 3600000ull, &c.timeout_ms);
  parse_u64("GICC_BOOTSTRAP_TIMEOUT_MS", 100, 86400000ull, &c.bootstrap_timeout_ms);
  if (const char* s = std::getenv("GICC_LOG_LEVEL")) {
    if (!strcasecmp(s, "error") || !std::strcmp(s, "0")) c.log_level = LOG_ERROR;
    else if (!strcasecmp(s, "warn") || !strcasecmp(s, "warning") || !std::strcmp(s, "1")) c.log_level = LOG_WARN;
    else if (!strcasecmp(s, "info") || !std::strcmp(s, "2")) c.log_level = LOG_INFO;
    else if (!strcasecmp(s, "debug") || !std::strcmp(s, "3")) c.log_level = LOG_DEBUG;
    else throw std::invalid_argument(std::string("GICC_LOG_LEVEL=") + s + ": expected error|warn|info|debug|0..3");
  }
  parse_bool("GICC_CHECKS", &c.checks);
  parse_bool("GICC_DISABLE_NVLS", &c.disable_nvls);
  parse_bool("GICC_DEBUG", &c.debug_puts);
  uint64_t heap = 0;
  if (parse_u64("GICC_SIGNAL_HEAP_BYTES", 64ull << 10, 1ull << 30, &heap)) c.signal_heap_bytes = heap;
  uint64_t v = 0;
  if (parse_u64("GICC_GEMM_GROUP_M", 1, 1024, &v)) c.gemm_group_m = (int)v;
  if (parse_u64("GICC_GEMM_L2_HINT", 0, 2, &v)) c.gemm_l2_hint = (int)v;
  if (parse_u64("GICC_GEMM_PAIR_GROUP_M", 1, 1024, &v)) c.gemm_pair_group_m = (int)v;
  if (parse_u64("GICC_GEMM_PAIR_L2_HINT", 0, 2, &v)) c.gemm_pair_l2_hint = (int)v;
  if (parse_u64("GICC_GEMM_PAIR_PREFETCH", 0, 64, &v)) c.gemm_pair_prefetch = (int)v;
  if (parse_u64("GICC_GEMM_PAIR_TMA_STORE", 0, 1, &v)) c.gemm_pair_tma_store = (int)v;
  return c;
}

std::string Config::summary() const {
  char buf[512];
  std::snprintf(buf, sizeof(buf),
                "gicc config: GICC_TIMEOUT_MS=%llu GICC_BOOTSTRAP_TIMEOUT_MS=%llu%s GICC_LOG_LEVEL=%s GICC_CHECKS=%d "
                "GICC_DISABLE_NVLS=%d GICC_DEBUG=%d GICC_SIGNAL_HEAP_BYTES=%zu%s GICC_GEMM_GROUP_M=%d "
                "GICC_GEMM_L2_HINT=%d",
                (unsigned long long)timeout_ms, (unsigned long long)bootstrap_timeout_ms,
                bootstrap_timeout_ms ? "" : " (default 120 s)", level_name(log_level), checks ? 1 : 0,
                disable_nvls ? 1 : 0, debug_puts ? 1 : 0, signal_heap_bytes,
                signal_heap_bytes ? "" : " (RuntimeOptions value)", gemm_group_m, gemm_l2_hint);
  return buf;
}

Config config() { return Config::from_env(); }

void set_log_rank(int rank) { g_rank = rank; }

void log(int level, const char* fmt, ...) {
  if (level > config().log_level) return;
  char msg[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  if (g_rank >= 0) std::fprintf(stderr, "[gicc r%d %s] %s\n", g_rank, level_name(level), msg);
  else std::fprintf(stderr, "[gicc %s] %s\n", level_name(level), msg);
}

NvtxRange::NvtxRange(const char* name) {
  std::call_once(g_domain_once, [] { g_domain = nvtxDomainCreateA("gicc"); });
  nvtxEventAttributes_t a{};
  a.version = NVTX_VERSION;
  a.size = NVTX_EVENT_ATTRIB_STRUCT_SIZE;
  a.messageType = NVTX_MESSAGE_TYPE_ASCII;
  a.message.ascii = name;
  nvtxDomainRangePushEx(g_domain, &a);
}

NvtxRange::~NvtxRange() { nvtxDomainRangePop(g_domain); }

}  // namespace gicc
