// Thread-local error messages for the C ABI.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "tcx_internal.h"

namespace tcx {
namespace {
thread_local std::string g_last_error;
}

tcx_status set_error(tcx_status code, const std::string& msg) {
  if (code != TCX_OK) g_last_error = msg;
  return code;
}

tcx_status set_errorf(tcx_status code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  return set_error(code, buf);
}

void clear_error() { g_last_error.clear(); }

namespace {
std::atomic<uint64_t> g_launches{0};
}
void note_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

}  // namespace tcx

extern "C" const char* tcx_last_error(void) { return tcx::g_last_error.c_str(); }

extern "C" uint64_t tcx_kernel_launch_count(void) { return tcx::g_launches.load(std::memory_order_relaxed); }

extern "C" const char* tcx_version(void) { return "tcx 0.1.0 (sm_100a)"; }
