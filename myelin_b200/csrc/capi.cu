// Error reporting and version for the myelin_b200 C ABI.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace mb {

static thread_local char g_last_error[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = '\0'; }

}  // namespace mb

extern "C" const char* mb_last_error(void) { return mb::g_last_error; }

extern "C" const char* mb_version(void) { return "myelin_b200 0.1.0 (sm_100a)"; }
