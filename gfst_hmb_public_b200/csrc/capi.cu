// C-ABI housekeeping: status strings, per-thread last-error text, launch checks.
#include <stdarg.h>
#include <string.h>

#include "gfst_common.cuh"

namespace gfst {

namespace {
thread_local char g_last_error[512] = {0};
}

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return GFST_OK;
  set_last_error("%s: %s", what, cudaGetErrorString(e));
  return GFST_ERR_LAUNCH;
}

}  // namespace gfst

extern "C" const char* gfst_status_string(int status) {
  switch (status) {
    case GFST_OK: return "ok";
    case GFST_ERR_ARG: return "invalid argument";
    case GFST_ERR_SHAPE: return "unsupported shape";
    case GFST_ERR_ALIGN: return "misaligned pointer or pitch";
    case GFST_ERR_LAUNCH: return "kernel launch failed";
    case GFST_ERR_DEVICE: return "CUDA runtime error";
    case GFST_ERR_TIMEOUT: return "device-side wait timed out";
    case GFST_ERR_DTYPE: return "unsupported dtype";
    case GFST_ERR_NUMERIC: return "numerical routine did not converge";
    default: return "unknown status";
  }
}

extern "C" int gfst_abi_version(void) { return (1 << 16) | 0; }

extern "C" const char* gfst_last_error(void) { return gfst::g_last_error; }
