// NVFP4 block-scaled GEMM (placeholder until the tcgen05 kind::mxf4nvf4 kernel lands).
#include "common.cuh"

extern "C" size_t rb2_nvfp4_gemm_workspace_size(int64_t, int64_t, int64_t) { return 0; }
extern "C" int rb2_nvfp4_gemm(const uint8_t*, const uint8_t*, const float*, const uint8_t*, const uint8_t*,
                              const float*, int64_t, int64_t, int64_t, void*, int, void*, size_t, void*) {
  rb2::set_error("nvfp4_gemm: not built");
  return RB2_EUNSUPPORTED;
}
