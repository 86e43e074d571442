// Affine state fold for segmented / context-parallel GDN.
//
// A run of chunks maps the 128 x 128 fp32 state affinely, S_out = M S_in + c, and the gradient
// transposed, dS_in = M^T dS_out + d. Given n such maps, the fold walks them in order (or in
// reverse, transposed) from a start value and records the value entering every map:
//   forward:    x_0 = s0;  x_{k+1} = M_k x_k + c_k              (k = 0 .. n-1)
//   transposed: x = s0;    x <- M_k^T x + c_k                   (k = n-1 .. 0)
// One CTA of 256 threads per (head, 32-column block of the state): the map M_k is staged in
// shared memory (row stride 129 floats, so rows of both M and M^T read without bank conflicts),
// the state block stays in shared memory, thread (i, half) owns 16 columns of row i. The next
// map is loaded into registers while the current step computes.
#include "common.cuh"

namespace rb2 {
namespace {

constexpr int kD = 128;
constexpr int kCols = 32;           // state columns per CTA (two 16-column halves)
constexpr int kHalf = 16;
constexpr int kThreads = 256;       // thread = (row i, column half)
constexpr int kMStride = kD + 1;
constexpr int kFoldSmem = (kD * kMStride + kD * kCols) * 4;
constexpr int kPf = kD * kD / 4 / kThreads;  // float4 of one map per thread (16)

__global__ void __launch_bounds__(kThreads) affine_fold_kernel(const float* __restrict__ M, const float* __restrict__ c,
                                                               const float* __restrict__ s0, int64_t n, int H,
                                                               int transpose, int identity_init,
                                                               float* __restrict__ states, float* __restrict__ final_out) {
  extern __shared__ float fsm[];
  float* ms = fsm;                    // [128][129]
  float* xs = fsm + kD * kMStride;    // [128][32] current value, columns [col0, col0 + 32)
  const int h = blockIdx.x, tid = threadIdx.x, i = tid & (kD - 1), half = tid >> 7;
  const int col0 = blockIdx.y * kCols, cx = half * kHalf;   // this thread's columns in xs
  const size_t mat = size_t(kD) * kD;
  const size_t hoff = size_t(h) * mat;
#pragma unroll
  for (int j = 0; j < kHalf; ++j) {
    const int col = col0 + cx + j;
    float v = 0.f;
    if (s0) v = s0[hoff + size_t(i) * kD + col];
    else if (identity_init) v = (i == col) ? 1.f : 0.f;
    xs[i * kCols + cx + j] = v;
  }
  // row i of A = M (A[i][r] = ms[i][r]) or M^T (A[i][r] = ms[r][i])
  const int a_row = transpose ? 1 : kMStride, a_col = transpose ? kMStride : 1;
  // the map of the next step is loaded into registers while this step computes
  float4 pf[kPf];
  auto fetch = [&](int64_t k) {
    const float4* mk = reinterpret_cast<const float4*>(M + size_t(k) * H * mat + hoff);
#pragma unroll
    for (int t = 0; t < kPf; ++t) pf[t] = mk[t * kThreads + tid];
  };
  if (n > 0) fetch(transpose ? n - 1 : 0);
  for (int64_t step = 0; step < n; ++step) {
    const int64_t k = transpose ? n - 1 - step : step;
    __syncthreads();  // xs written, ms free
#pragma unroll
    for (int t = 0; t < kPf; ++t) {
      const int e = 4 * (t * kThreads + tid), row = e >> 7, col = e & 127;
      float* d = ms + row * kMStride + col;
      d[0] = pf[t].x; d[1] = pf[t].y; d[2] = pf[t].z; d[3] = pf[t].w;
    }
    if (step + 1 < n) fetch(transpose ? k - 1 : k + 1);
    if (states) {
      float* dst = states + size_t(k) * H * mat + hoff + size_t(i) * kD + col0 + cx;
#pragma unroll
      for (int j = 0; j < kHalf; j += 4)
        *reinterpret_cast<float4*>(dst + j) = *reinterpret_cast<const float4*>(xs + i * kCols + cx + j);
    }
    float acc[kHalf];
    if (c) {
      const float* ck = c + size_t(k) * H * mat + hoff + size_t(i) * kD + col0 + cx;
#pragma unroll
      for (int j = 0; j < kHalf; j += 4) {
        const float4 v = *reinterpret_cast<const float4*>(ck + j);
        acc[j] = v.x; acc[j + 1] = v.y; acc[j + 2] = v.z; acc[j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < kHalf; ++j) acc[j] = 0.f;
    }
    __syncthreads();  // ms filled
#pragma unroll 4
    for (int r = 0; r < kD; ++r) {
      const float a = ms[i * a_row + r * a_col];
      const float* xr = xs + r * kCols + cx;
#pragma unroll
      for (int j = 0; j < kHalf; j += 4) {
        const float4 x4 = *reinterpret_cast<const float4*>(xr + j);
        acc[j] = fmaf(a, x4.x, acc[j]);
        acc[j + 1] = fmaf(a, x4.y, acc[j + 1]);
        acc[j + 2] = fmaf(a, x4.z, acc[j + 2]);
        acc[j + 3] = fmaf(a, x4.w, acc[j + 3]);
      }
    }
    __syncthreads();  // every thread has read xs
#pragma unroll
    for (int j = 0; j < kHalf; j += 4)
      *reinterpret_cast<float4*>(xs + i * kCols + cx + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
  }
  __syncthreads();
  if (final_out) {
    float* dst = final_out + hoff + size_t(i) * kD + col0 + cx;
#pragma unroll
    for (int j = 0; j < kHalf; j += 4)
      *reinterpret_cast<float4*>(dst + j) = *reinterpret_cast<const float4*>(xs + i * kCols + cx + j);
  }
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" int rb2_gdn_state_fold(const float* M, const float* c, const float* s0, int64_t n, int H, int d,
                                  int transpose, int identity_init, float* states, float* final_out, void* stream) {
  RB2_CHECK_ARG(d == kD, "gdn_state_fold: state dim must be 128 (got %d)", d);
  RB2_CHECK_ARG(n >= 0 && H >= 1 && H <= 65535, "gdn_state_fold: bad sizes n=%lld H=%d", (long long)n, H);
  RB2_CHECK_ARG(n == 0 || M != nullptr, "gdn_state_fold: null M");
  RB2_CHECK_ARG(states || final_out, "gdn_state_fold: no output");
  RB2_CHECK_ARG(!(s0 && identity_init), "gdn_state_fold: s0 and identity_init are exclusive");
  auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  RB2_CHECK_ARG(!misaligned(M) && !misaligned(c) && !misaligned(s0) && !misaligned(states) && !misaligned(final_out),
                "gdn_state_fold: pointers must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RB2_CUDA(cudaFuncSetAttribute(affine_fold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFoldSmem),
           "gdn_state_fold: smem attribute");
  ProfScope ps_("gdn_state_fold", s);
  affine_fold_kernel<<<dim3(H, kD / kCols), kThreads, kFoldSmem, s>>>(M, c, s0, n, H, transpose, identity_init, states,
                                                                 final_out);
  RB2_CHECK_LAUNCH("gdn_state_fold");
  return RB2_OK;
}
