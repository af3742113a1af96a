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

namespace mb {
// Defined by the units that own bounded waits (async_copy.cuh declares them
// too); repeated here because this file has no device code of its own.
int scan_unit_status(bool clear);
int scan_fast_unit_status(bool clear);
int gemm_unit_status(bool clear);
cudaError_t scan_unit_wait_probe(uint32_t polls, cudaStream_t stream);
cudaError_t scan_fast_unit_wait_probe(uint32_t polls, cudaStream_t stream);
cudaError_t gemm_unit_wait_probe(uint32_t polls, cudaStream_t stream);
}  // namespace mb

// Every unit's word is read (and cleared when asked), so one call reports and
// resets all of them; the first non-zero code in unit order is returned.
extern "C" int mb_device_status(int clear) {
  int (*units[])(bool) = {mb::scan_unit_status, mb::scan_fast_unit_status,
                          mb::gemm_unit_status};
  int result = 0;
  bool failed = false;
  for (auto unit : units) {
    const int v = unit(clear != 0);
    if (v < 0) failed = true;
    else if (result == 0) result = v;
  }
  return failed ? -1 : result;
}

extern "C" int mb_debug_wait_timeout(int unit, int polls, void* stream) {
  MB_CHECK_ARG(polls > 0 && polls <= (1 << 16),
               "mb_debug_wait_timeout: polls must be in [1, 65536] (got %d)", polls);
  cudaStream_t s = mb::as_stream(stream);
  cudaError_t err;
  switch (unit) {
    case MB_UNIT_SCAN: err = mb::scan_unit_wait_probe(static_cast<uint32_t>(polls), s); break;
    case MB_UNIT_SCAN_FAST:
      err = mb::scan_fast_unit_wait_probe(static_cast<uint32_t>(polls), s);
      break;
    case MB_UNIT_GEMM: err = mb::gemm_unit_wait_probe(static_cast<uint32_t>(polls), s); break;
    default: mb::set_error("mb_debug_wait_timeout: unknown unit %d", unit); return 1;
  }
  if (err != cudaSuccess) {
    mb::set_error("mb_debug_wait_timeout: launch failed: %s", cudaGetErrorString(err));
    return 2;
  }
  return 0;
}
