// pb_api.cpp -- error reporting and process-wide counters of the C ABI.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include "pb_internal.h"

namespace {
thread_local char g_err[512] = "";
thread_local bool g_capturing = false;
std::atomic<uint64_t> g_launches{0};
}  // namespace

int pb_set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

void pb_count_launch(uint64_t n) {
  if (!g_capturing) g_launches.fetch_add(n, std::memory_order_relaxed);
}
void pb_set_capturing(bool on) { g_capturing = on; }

extern "C" int pb_version(void) { return 10000; }

extern "C" int pb_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return PB_EINVAL;
  snprintf(buf, n, "%s", g_err);
  return PB_OK;
}

extern "C" uint64_t pb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }
