// capi.cu -- version, thread-local error reporting and launch checking for
// the libgsb200 C ABI (declared in include/gsb200.h).
#include <cstdarg>
#include <cstdio>
#include <cstring>

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

GSB_EXPORT int gsb_block_dim(const char* kernel_class) {
  using namespace gsb::launch;
  struct Entry {
    const char* name;
    int threads;
  };
  static const Entry table[] = {
      {"preprocess", PREPROCESS},
      {"preprocess_sh16", PREPROCESS_SH16},
      {"sh_colors_views", SH_COLORS_VIEWS},
      {"binning_scan", BINNING_SCAN},
      {"binning_emit", BINNING_EMIT},
      {"radix_sort", RADIX_SORT},
      {"render_forward", RENDER},
      {"render_backward", RENDER_BWD},
      {"render_backward_small_grid", RENDER},  // grids of fewer than 6,000 tiles
      {"backward_preprocess", PREPROCESS_BWD},
      {"backward_preprocess_sh16", PREPROCESS_BWD_SH16},
      {"sh_backward_views", SH_BACKWARD_VIEWS},
      {"ssim_fwd", SSIM},
      {"ssim_bwd", SSIM},
      // the reference's separate SSIM passes are one fused kernel per direction here
      {"ssim_fwd_h", SSIM},
      {"ssim_fwd_v", SSIM},
      {"ssim_bwd_h", SSIM},
      {"ssim_bwd_v", SSIM},
      {"knn_morton", KNN},
      {"knn_gather", KNN},
      {"knn_box_minmax", KNN},
      {"knn_box_dist", KNN},
      {"knn_search", KNN},
      {"adam", ADAM},
  };
  if (!kernel_class) return 0;
  for (const Entry& e : table)
    if (std::strcmp(e.name, kernel_class) == 0) return e.threads;
  return 0;
}
