// capi.cu -- version, thread-local error reporting and launch checking for
// the libgsb200 C ABI (declared in include/gsb200.h).
#include <cstdarg>
#include <cstdio>

#include "gsb_common.cuh"

namespace gsb {

namespace {
thread_local char g_last_error[512] = "";
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

// Reports launch-configuration errors without synchronizing the stream.
int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return GSB_ERR_CUDA;
  }
  return GSB_OK;
}

}  // namespace gsb

GSB_EXPORT int gsb_abi_version(void) { return GSB_ABI_VERSION; }

GSB_EXPORT const char* gsb_last_error(void) { return gsb::g_last_error; }
