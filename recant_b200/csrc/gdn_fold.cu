// Affine state fold for segmented / context-parallel GDN.
//
// A run of chunks maps the 128 x 128 fp32 state affinely, S_out = M S_in + c, and the gradient
// transposed, dS_in = M^T dS_out + d. Given n such maps, the fold walks them in order (or in
// reverse, transposed) from a start value and records the value entering every map:
//   forward:    x_0 = s0;  x_{k+1} = M_k x_k + c_k              (k = 0 .. n-1)
//   transposed: x = s0;    x <- M_k^T x + c_k                   (k = n-1 .. 0)
// One CTA of 256 threads per (head, 32-column block of the state), thread (ti, tj) owning the 4 x 4
// block rows 4 ti .. 4 ti + 3, columns 4 tj .. 4 tj + 3. Per step the map is staged in shared memory
// as given (row stride 132 floats: 16-byte aligned rows); when row r of the staged array is column r
// of the applied matrix A (A = G^T: the transposed modes), one step is 128 x (two 16-byte loads + 16
// FMAs) per thread; mode 0 (A = G) reads A's column from four rows instead. The state block stays in
// shared memory; the next map is fetched into registers while the current step computes. A prefix
// run of maps (whose entering values are not recorded) may precede the main maps in the same launch.
#include "common.cuh"

namespace rb2 {
namespace {

constexpr int kD = 128;
constexpr int kCols = 32;                     // state columns per CTA
constexpr int kThreads = 256;
constexpr int kMS = kD + 4;                   // staged map row stride (floats)
constexpr int kXS = kCols + 4;                // state block row stride (floats)
constexpr int kFoldSmem = (kD * kMS + kD * kXS) * 4;
constexpr int kPf = kD * kD / 4 / kThreads;   // float4 of one map per thread (16)

struct MapRun {
  const float* M;
  const float* c;
  int64_t n;
};

// mode 0: ascending k, A_k = M_k;  mode 1: descending k, A_k = M_k^T;  mode 2: ascending k, A_k = M_k^T
__global__ void __launch_bounds__(kThreads) affine_fold_kernel(MapRun pre, MapRun main_, const float* __restrict__ s0,
                                                               int H, int mode, int identity_init,
                                                               float* __restrict__ states, float* __restrict__ final_out) {
  extern __shared__ __align__(16) float fsm[];
  float* ms = fsm;                 // [128][132]
  float* xs = fsm + kD * kMS;      // [128][36]: the value, columns [col0, col0 + 32)
  const int h = blockIdx.x, tid = threadIdx.x, ti = tid >> 3, tj = tid & 7;
  const int col0 = blockIdx.y * kCols;
  const size_t mat = size_t(kD) * kD, hoff = size_t(h) * mat;
  const bool desc = mode == 1, a_rows = mode != 0;
  float x[4][4];  // this thread's block of the value entering the current step
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int row = 4 * ti + p, col = col0 + 4 * tj;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s0) v = *reinterpret_cast<const float4*>(s0 + hoff + size_t(row) * kD + col);
    else if (identity_init) v = make_float4(row == col, row == col + 1, row == col + 2, row == col + 3);
    x[p][0] = v.x; x[p][1] = v.y; x[p][2] = v.z; x[p][3] = v.w;
    *reinterpret_cast<float4*>(xs + row * kXS + 4 * tj) = v;
  }
  const int64_t total = pre.n + main_.n;
  // step s -> (run, map index): the prefix run first, each run in the mode's order
  auto map_of = [&](int64_t s, const float*& Mk, const float*& ck, int64_t& kmain) {
    const bool in_pre = s < pre.n;
    const MapRun& run = in_pre ? pre : main_;
    const int64_t j = in_pre ? s : s - pre.n;
    const int64_t k = desc ? run.n - 1 - j : j;
    Mk = run.M + size_t(k) * H * mat + hoff;
    ck = run.c ? run.c + size_t(k) * H * mat + hoff : nullptr;
    kmain = in_pre ? -1 : k;
  };
  float4 pf[kPf];
  auto fetch = [&](const float* Mk) {
    const float4* m4 = reinterpret_cast<const float4*>(Mk);
#pragma unroll
    for (int t = 0; t < kPf; ++t) pf[t] = m4[t * kThreads + tid];
  };
  const float* Mk;
  const float* ck;
  int64_t kmain;
  if (total > 0) {
    map_of(0, Mk, ck, kmain);
    fetch(Mk);
  }
  for (int64_t s = 0; s < total; ++s) {
    map_of(s, Mk, ck, kmain);
    __syncthreads();  // xs written, ms free
#pragma unroll
    for (int t = 0; t < kPf; ++t) {
      const int e = 4 * (t * kThreads + tid), row = e >> 7, col = e & 127;
      *reinterpret_cast<float4*>(ms + row * kMS + col) = pf[t];
    }
    if (s + 1 < total) {
      const float* Mn;
      const float* cn;
      int64_t kn;
      map_of(s + 1, Mn, cn, kn);
      fetch(Mn);
    }
    if (states && kmain >= 0) {
      float* dst = states + size_t(kmain) * H * mat + hoff + size_t(4 * ti) * kD + col0 + 4 * tj;
#pragma unroll
      for (int p = 0; p < 4; ++p)
        *reinterpret_cast<float4*>(dst + p * kD) = make_float4(x[p][0], x[p][1], x[p][2], x[p][3]);
    }
    float acc[4][4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ck) v = *reinterpret_cast<const float4*>(ck + size_t(4 * ti + p) * kD + col0 + 4 * tj);
      acc[p][0] = v.x; acc[p][1] = v.y; acc[p][2] = v.z; acc[p][3] = v.w;
    }
    __syncthreads();  // ms filled
    if (a_rows) {
#pragma unroll 4
      for (int r = 0; r < kD; ++r) {
        const float4 a = *reinterpret_cast<const float4*>(ms + r * kMS + 4 * ti);
        const float4 xv = *reinterpret_cast<const float4*>(xs + r * kXS + 4 * tj);
        const float av[4] = {a.x, a.y, a.z, a.w}, xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[p][q] = fmaf(av[p], xw[q], acc[p][q]);
      }
    } else {
#pragma unroll 4
      for (int r = 0; r < kD; ++r) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + r * kXS + 4 * tj);
        const float xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float av = ms[(4 * ti + p) * kMS + r];
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[p][q] = fmaf(av, xw[q], acc[p][q]);
        }
      }
    }
    __syncthreads();  // every thread has read xs
#pragma unroll
    for (int p = 0; p < 4; ++p) {
#pragma unroll
      for (int q = 0; q < 4; ++q) x[p][q] = acc[p][q];
      *reinterpret_cast<float4*>(xs + (4 * ti + p) * kXS + 4 * tj) = make_float4(acc[p][0], acc[p][1], acc[p][2], acc[p][3]);
    }
  }
  if (final_out) {
    float* dst = final_out + hoff + size_t(4 * ti) * kD + col0 + 4 * tj;
#pragma unroll
    for (int p = 0; p < 4; ++p)
      *reinterpret_cast<float4*>(dst + p * kD) = make_float4(x[p][0], x[p][1], x[p][2], x[p][3]);
  }
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" int rb2_gdn_state_fold_ex(const float* M, const float* c, int64_t n, const float* Mp, const float* cp,
                                     int64_t np, const float* s0, int H, int d, int mode, int identity_init,
                                     float* states, float* final_out, void* stream) {
  RB2_CHECK_ARG(d == kD, "gdn_state_fold: state dim must be 128 (got %d)", d);
  RB2_CHECK_ARG(n >= 0 && np >= 0 && H >= 1 && H <= 65535, "gdn_state_fold: bad sizes n=%lld np=%lld H=%d",
                (long long)n, (long long)np, H);
  RB2_CHECK_ARG(mode >= 0 && mode <= 2, "gdn_state_fold: mode must be 0, 1 or 2");
  RB2_CHECK_ARG((n == 0 || M != nullptr) && (np == 0 || Mp != nullptr), "gdn_state_fold: null M");
  RB2_CHECK_ARG(states || final_out, "gdn_state_fold: no output");
  RB2_CHECK_ARG(!(s0 && identity_init), "gdn_state_fold: s0 and identity_init are exclusive");
  auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  RB2_CHECK_ARG(!misaligned(M) && !misaligned(c) && !misaligned(Mp) && !misaligned(cp) && !misaligned(s0) &&
                    !misaligned(states) && !misaligned(final_out),
                "gdn_state_fold: pointers must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RB2_CUDA(cudaFuncSetAttribute(affine_fold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFoldSmem),
           "gdn_state_fold: smem attribute");
  ProfScope ps_("gdn_state_fold", s);
  affine_fold_kernel<<<dim3(H, kD / kCols), kThreads, kFoldSmem, s>>>(MapRun{Mp, cp, np}, MapRun{M, c, n}, s0, H, mode,
                                                                 identity_init, states, final_out);
  RB2_CHECK_LAUNCH("gdn_state_fold");
  return RB2_OK;
}

extern "C" int rb2_gdn_state_fold(const float* M, const float* c, const float* s0, int64_t n, int H, int d,
                                  int transpose, int identity_init, float* states, float* final_out, void* stream) {
  return rb2_gdn_state_fold_ex(M, c, n, nullptr, nullptr, 0, s0, H, d, transpose ? 1 : 0, identity_init, states,
                               final_out, stream);
}
