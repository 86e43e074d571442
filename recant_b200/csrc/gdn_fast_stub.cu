// Placeholder for the tensor-core GDN path until it lands: every entry reports "unsupported".
#include "gdn_common.cuh"

namespace rb2 {
size_t fast_workspace_size(int64_t, int64_t, int, int, int) { return 0; }
int fast_forward(const GdnProblem&, void*, void*, float*, cudaStream_t) {
  set_error("gdn: tensor-core path not built");
  return RB2_EUNSUPPORTED;
}
int fast_backward(const GdnProblem&, void*, const void*, const float*, void*, void*, void*, float*, void*,
                  float*, cudaStream_t) {
  set_error("gdn: tensor-core path not built");
  return RB2_EUNSUPPORTED;
}
}  // namespace rb2

extern "C" size_t rb2_nvfp4_gemm_workspace_size(int64_t, int64_t, int64_t) { return 0; }
extern "C" int rb2_nvfp4_gemm(const uint8_t*, const uint8_t*, const float*, const uint8_t*, const uint8_t*,
                              const float*, int64_t, int64_t, int64_t, void*, int, void*, size_t, void*) {
  rb2::set_error("nvfp4_gemm: not built");
  return RB2_EUNSUPPORTED;
}
