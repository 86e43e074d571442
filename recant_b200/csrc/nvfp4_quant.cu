// NVFP4 activation quantizer: randomized Hadamard (16-point) + e2m1 codes + e4m3 per-16 scales
// + fp32 global scale, bit-exact with the reference quantize(rht(x)).
//
// Reference semantics (recant/model/nvfp4.py):
//   rht            :23-31  sign flip by _SIGNS, butterflies with strides 1,2,4,8 as (a+b, a-b),
//                          x0.25, re-round to the input dtype
//   quantize       :76-91  s_g = max(|x|, 1e-30) / (6*448); s_b = min((amax16 / 6) / s_g, 448)
//                          -> e4m3 (RNE); denom = (s8 == 0 ? 1 : s8) * s_g; q = x / denom
//   _round_codes   :59-71  RN: idx = #{midpoints < |q|} (ties toward zero), +8 when q < 0;
//                          SR: unbiased choice between the two neighbouring grid points
//   _pack          :73-74  even element in the low nibble
//
// Design (2.5625 B/elt algorithmic for bf16): the global amax forces two passes.
// Pass 1 reads x, transforms each 16-block in registers and reduces the amax to one word.
// Pass 2 re-reads x in REVERSE block order so that the tail of x that pass 1 left in the
// 126 MB L2 is consumed first, recomputes the transform and writes codes and scales.
// Both passes are persistent grid-stride sweeps (SMs x resident CTAs): a thread handles one
// 16-element block at a time (a warp covers 512 contiguous elements) with the next block's load
// already in flight. Inputs of at most 2048 blocks run both passes in one CTA and one launch.
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "gated_norm.cuh"

namespace rb2 {
namespace {

constexpr int kThreads = 256;

// The raw bytes of one 16-element block (32 for bf16, 64 for fp32): loaded one block ahead of the
// block being transformed, so that every thread keeps a load in flight while it computes.
template <typename T>
struct Raw16 {
  uint4 w[sizeof(T) * 16 / 16];
};

template <typename T>
__device__ __forceinline__ void load_raw(const T* __restrict__ p, Raw16<T>& r) {
  const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < int(sizeof(T)); ++i) r.w[i] = __ldg(p4 + i);
}

__device__ __forceinline__ void unpack16(const Raw16<float>& r, float v[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[4 * i + 0] = __uint_as_float(r.w[i].x); v[4 * i + 1] = __uint_as_float(r.w[i].y);
    v[4 * i + 2] = __uint_as_float(r.w[i].z); v[4 * i + 3] = __uint_as_float(r.w[i].w);
  }
}

__device__ __forceinline__ void unpack16(const Raw16<__nv_bfloat16>& r, float v[16]) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t w[4] = {r.w[i].x, r.w[i].y, r.w[i].z, r.w[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j + 0] = __uint_as_float(w[j] << 16);
      v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
  }
}

// Two butterflies at once: (a0, a1) <- (a0, a1) + (b0, b1), (b0, b1) <- (a0, a1) - (b0, b1) as paired
// f32x2 operations (sm_100), each lane rounded exactly as the scalar add / sub.
__device__ __forceinline__ void bfly2(float& a0, float& a1, float& b0, float& b1) {
  unsigned long long a, b, sm, df;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(sm) : "l"(a), "l"(b));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(df) : "l"(a), "l"(b));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(sm));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(b0), "=f"(b1) : "l"(df));
}
__device__ __forceinline__ void mul2(float& a0, float& a1, float c) {
  unsigned long long a, k, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(k) : "f"(c));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(k));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(r));
}

// The 16-point randomized Hadamard transform of one block with the reference's operations in the
// reference's order (every element is the same chain of IEEE adds / subtracts as nvfp4.rht), the
// butterflies paired two at a time; `reround`: round the result to the input dtype, as rht does.
template <typename T>
__device__ __forceinline__ void transform16(float v[16], bool rot, bool reround = true) {
  if (rot) {
    // _SIGNS = [1,1,-1,1,-1,-1,-1,1,1,1,1,1,-1,-1,1,-1]
    v[2] = -v[2]; v[4] = -v[4]; v[5] = -v[5]; v[6] = -v[6];
    v[12] = -v[12]; v[13] = -v[13]; v[15] = -v[15];
#pragma unroll
    for (int i = 0; i < 16; i += 4) bfly2(v[i], v[i + 2], v[i + 1], v[i + 3]);  // stride 1: (i, i+1), (i+2, i+3)
#pragma unroll
    for (int s = 2; s < 16; s <<= 1) {
#pragma unroll
      for (int i = 0; i < 16; i += 2)
        if ((i & s) == 0) bfly2(v[i], v[i + 1], v[i + s], v[i + s + 1]);
    }
#pragma unroll
    for (int i = 0; i < 16; i += 2) mul2(v[i], v[i + 1], 0.25f);
    if (sizeof(T) == 2 && reround) {  // one paired conversion per two elements
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[i], v[i + 1]);
        const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
        v[i] = __uint_as_float(u << 16);
        v[i + 1] = __uint_as_float(u & 0xffff0000u);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
zero_word_kernel(unsigned int* w) { *w = 0u; }

// Pass 1: a grid-stride sweep (forward) over the blocks, one block in flight per thread ahead of
// the one being transformed; one atomicMax per CTA.
template <typename T>
__global__ void __launch_bounds__(kThreads)
amax_kernel(const T* __restrict__ x, int64_t n_blocks, int rot, unsigned int* __restrict__ gmax_bits) {
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  int64_t b = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  float m = 0.f;
  Raw16<T> cur;
  if (b < n_blocks) load_raw(x + b * 16, cur);
  for (; b < n_blocks; b += stride) {
    Raw16<T> nxt;
    if (b + stride < n_blocks) load_raw(x + (b + stride) * 16, nxt);
    float v[16];
    unpack16(cur, v);
    transform16<T>(v, rot != 0, false);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
    cur = nxt;
  }
  // rht re-rounds to the input dtype; rounding to nearest is monotone and symmetric, so the max of
  // the rounded magnitudes is the rounded max
  if (sizeof(T) == 2 && rot) m = __bfloat162float(__float2bfloat16_rn(m));
  m = warp_max(m);
  __shared__ float red[kThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.f;
    r = warp_max(r);
    // non-negative floats order like their bit patterns
    if (threadIdx.x == 0 && r > 0.f) atomicMax(gmax_bits, __float_as_uint(r));
  }
}

// Philox-4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw; SC'11).
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// e2m1 index for round-to-nearest with ties toward zero: the number of decision points 0.25, 0.75,
// 1.25, 1.75, 2.5, 3.5, 5 strictly below a = min(|q|, 6). Each point has at most two mantissa bits
// after the leading one, so with key = ceil(bits(a) / 2^21) (sign 0, 8 exponent bits, 2 mantissa
// bits, rounded up) a > point <=> key > key(point); the keys of the points are 500, 506, 509, 511,
// 513, 515, 517, and the index is a step function of key in [500, 518], read from a packed table
// of 4-bit entries.
__device__ __forceinline__ int e2m1_index(float a) {
  const uint32_t key = (__float_as_uint(a) + 0x1FFFFFu) >> 21;
  const uint32_t k = min(max(key, 500u), 518u) - 500u;  // 0 .. 18
  // entry k = #{points with key < 500 + k}
  constexpr uint64_t lo = 0x5544332221111110ull;        // k = 0 .. 15
  constexpr uint32_t hi = 0x766u;                        // k = 16 .. 18
  return k < 16 ? int((lo >> (4 * k)) & 0xF) : int((hi >> (4 * (k - 16))) & 0xF);
}

// floor(n / d) for n < 2^32 by one multiply and shift (Granlund & Montgomery, PLDI 1994):
// s = ceil(log2 d), m = ceil(2^(32+s) / d)
struct Divider {
  uint64_t m;
  uint32_t s;
};
inline Divider make_divider(uint32_t d) {
  uint32_t s = 0;
  while ((uint64_t(1) << s) < d) ++s;
  const unsigned __int128 num = (static_cast<unsigned __int128>(1) << (32 + s));
  return Divider{uint64_t((num + d - 1) / d), s};
}
__device__ __forceinline__ uint32_t divide(uint32_t n, Divider dv) {
  // m < 2^33: floor(n m / 2^32) = floor(n m_lo / 2^32) + n m_hi
  const uint64_t hi32 = ((uint64_t(n) * uint32_t(dv.m)) >> 32) + uint64_t(n) * (dv.m >> 32);
  return uint32_t(hi32 >> dv.s);
}

// SR: the upper of the two grid neighbours of a in [0, 6], as the index of the first of 0, .5, 1,
// 1.5, 2, 3, 4 that is not below a (at least 1): every such point is a multiple of 2^21 in the bit
// pattern, so with key = ceil(bits(a) / 2^21) the count is a step function of key in [504, 518],
// read from a packed table of 4-bit entries.
__device__ __forceinline__ int sr_upper(float a) {
  const uint32_t key = (__float_as_uint(a) + 0x1FFFFFu) >> 21;
  const uint32_t k = min(max(key, 504u), 518u) - 504u;  // 0 .. 14
  return int((0x776655443322221ull >> (4 * k)) & 0xFu);
}

// Codes and scale of block b from its raw bytes.
template <typename T>
__device__ __forceinline__ void quant_block(uint32_t b, const Raw16<T>& raw, int rot, int stochastic, uint64_t seed,
                                            float s_g, uint32_t groups, Divider by_groups,
                                            uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
                                            uint8_t* __restrict__ blocked) {
  float v[16];
  unpack16(raw, v);
  transform16<T>(v, rot != 0);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float s_b = fminf(__fdiv_rn(__fdiv_rn(amax, 6.0f), s_g), 448.0f);
  const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(s_b, __NV_SATFINITE, __NV_E4M3);
  const __half_raw hr = __nv_cvt_fp8_to_halfraw(s8, __NV_E4M3);
  const float sq = __half2float(__half(hr));
  const float denom = __fmul_rn(sq == 0.f ? 1.f : sq, s_g);
  // a' = |x| RN(1/denom) is within 2.5 ulp of the correctly rounded |x| / denom (two roundings of
  // relative size 2^-24 each, plus the quotient's own half ulp). Every decision point of the
  // rounding (RN: 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5; SR: the grid 0.5, 1, 1.5, 2, 3, 4, 6) lies on
  // a multiple of 2^21 in the bit pattern, so when the bits of a' are more than 8 away from such a
  // multiple (SR; RN tests the points themselves, below), a' and the exact quotient fall on the same
  // side of every point; otherwise the exact quotient is computed. q < 0 <=> x < 0 since denom > 0 (and -0
  // gives +0 / no sign bit in both); the sign is bit 3 of each nibble.
  const float rinv = __frcp_rn(denom);
  uint32_t packed[2] = {0u, 0u};
  if (stochastic) {
    // Unbiased choice between the grid neighbours lo < a <= hi with p = (a - lo) / (hi - lo); the
    // spacing hi - lo is a power of two, so the division is an exact multiply. p from a' differs from
    // p of the exact quotient by a few ulps, which moves no choice's probability by more than that.
    uint32_t rnd[16];
    const uint2 key = make_uint2(uint32_t(seed), uint32_t(seed >> 32));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 r = philox4x32_10(make_uint4(b, 0u, uint32_t(j), 0u), key);
      rnd[4 * j + 0] = r.x; rnd[4 * j + 1] = r.y; rnd[4 * j + 2] = r.z; rnd[4 * j + 3] = r.w;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float a = __fmul_rn(fabsf(v[i]), rinv);
      const uint32_t u = __float_as_uint(a);
      if (u != 0u && ((u + 8u) & 0x1FFFFFu) <= 16u) a = fabsf(__fdiv_rn(v[i], denom));
      a = fminf(a, 6.0f);
      const int hi = sr_upper(a);
      const float glo = hi <= 4 ? 0.5f * float(hi - 1) : float(hi - 3);
      const float inv = hi <= 4 ? 2.f : (hi < 7 ? 1.f : 0.5f);
      const float pr = __fmul_rn(__fsub_rn(a, glo), inv);
      const float r = float(rnd[i] >> 8) * (1.0f / 16777216.0f);
      const int idx = (r < pr) ? hi : hi - 1;
      packed[i >> 3] |= uint32_t(idx + (v[i] < 0.f ? 8 : 0)) << (4 * (i & 7));
    }
  } else {
    // RN: away from the decision points the index is the nearest grid point, which the hardware
    // pair conversion (cvt.rn.satfinite.e2m1x2, values above 6 saturating to 6) gives for two
    // magnitudes at once; at a decision point it rounds ties to even where the reference rounds
    // them toward zero, and those pairs take the exact path, which counts the points. A pair is near
    // a decision point when a' (1 - e) and a' (1 + e), e = 2^-19 (16 ulps, against a' being within
    // 2.5 ulps of the exact quotient), convert differently: the two then lie on either side of a
    // point; grid points and zeros convert alike on both sides and do not trigger.
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const float a0 = __fmul_rn(fabsf(v[i]), rinv), a1 = __fmul_rn(fabsf(v[i + 1]), rinv);
      uint32_t nib = __nv_cvt_float2_to_fp4x2(make_float2(a0, a1), __NV_E2M1, cudaRoundNearest);  // a0 low
      float l0 = a0, l1 = a1, h0 = a0, h1 = a1;
      mul2(l0, l1, 1.0f - 0x1p-19f);
      mul2(h0, h1, 1.0f + 0x1p-19f);
      const uint32_t nl = __nv_cvt_float2_to_fp4x2(make_float2(l0, l1), __NV_E2M1, cudaRoundNearest),
                     nh = __nv_cvt_float2_to_fp4x2(make_float2(h0, h1), __NV_E2M1, cudaRoundNearest);
      if (((nl ^ nh) & 0xFFu) != 0u) {
        const float e0 = fabsf(__fdiv_rn(v[i], denom)), e1 = fabsf(__fdiv_rn(v[i + 1], denom));
        nib = uint32_t(e2m1_index(fminf(e0, 6.0f))) | (uint32_t(e2m1_index(fminf(e1, 6.0f))) << 4);
      }
      nib |= (v[i] < 0.f ? 8u : 0u) | (v[i + 1] < 0.f ? 0x80u : 0u);
      packed[i >> 3] |= (nib & 0xFFu) << (4 * (i & 7));
    }
  }
  reinterpret_cast<uint2*>(codes)[b] = make_uint2(packed[0], packed[1]);
  scales[b] = uint8_t(s8);
  if (blocked) {
    const uint32_t r = divide(b, by_groups), c = b - r * groups;
    const size_t ncb = (groups + 3) / 4;
    const size_t off = ((r >> 7) * ncb + (c >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (c & 3);
    blocked[off] = uint8_t(s8);
  }
}

// Pass 2: a grid-stride sweep in REVERSE block order (the j-th block from the end), so that what
// pass 1 left in L2 is consumed first, with the next block's load in flight during each block.
template <typename T>
__global__ void __launch_bounds__(kThreads, 4)
quant_kernel(const T* __restrict__ x, uint32_t n_blocks, uint32_t groups, Divider by_groups, int rot,
             int stochastic, uint64_t seed, const unsigned int* __restrict__ gmax_bits,
             uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
             uint8_t* __restrict__ blocked, float* __restrict__ gscale_out) {
  const float gmax = fmaxf(__uint_as_float(*gmax_bits), 1e-30f);
  const float s_g = __fdiv_rn(gmax, 2688.0f);  // 6 * 448
  if (blockIdx.x == 0 && threadIdx.x == 0) *gscale_out = s_g;
  const uint32_t stride = gridDim.x * kThreads;
  uint32_t j = blockIdx.x * kThreads + threadIdx.x;
  Raw16<T> cur;
  if (j < n_blocks) load_raw(x + size_t(n_blocks - 1 - j) * 16, cur);
  for (; j < n_blocks; j += stride) {
    Raw16<T> nxt;
    if (j + stride < n_blocks) load_raw(x + size_t(n_blocks - 1 - (j + stride)) * 16, nxt);
    quant_block<T>(n_blocks - 1 - j, cur, rot, stochastic, seed, s_g, groups, by_groups, codes, scales, blocked);
    cur = nxt;
  }
}

// Inputs of at most kSmallBlocks blocks (the decode step quantizes one token per sequence): one CTA
// takes the amax and then quantizes, so the call is one launch instead of three. The same
// per-block code as the two passes; max is exact in any order, so the result is identical.
constexpr uint32_t kSmallBlocks = 2048;

template <typename T>
__global__ void __launch_bounds__(kThreads)
quant_small_kernel(const T* __restrict__ x, uint32_t n_blocks, uint32_t groups, Divider by_groups, int rot,
                   int stochastic, uint64_t seed, uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
                   uint8_t* __restrict__ blocked, size_t clear_bytes, float* __restrict__ gscale_out) {
  // zero the blocked scales first (their pads); the scales themselves are written after the barrier
  for (size_t i = threadIdx.x; i < clear_bytes; i += kThreads) blocked[i] = 0;
  float m = 0.f;
  for (uint32_t b = threadIdx.x; b < n_blocks; b += kThreads) {
    Raw16<T> raw;
    load_raw(x + size_t(b) * 16, raw);
    float v[16];
    unpack16(raw, v);
    transform16<T>(v, rot != 0);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
  }
  m = warp_max(m);
  __shared__ float red[kThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float gm = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) gm = fmaxf(gm, red[i]);
  const float s_g = __fdiv_rn(fmaxf(gm, 1e-30f), 2688.0f);  // 6 * 448
  if (threadIdx.x == 0) *gscale_out = s_g;
  for (uint32_t b = threadIdx.x; b < n_blocks; b += kThreads) {
    Raw16<T> raw;
    load_raw(x + size_t(b) * 16, raw);
    quant_block<T>(b, raw, rot, stochastic, seed, s_g, groups, by_groups, codes, scales, blocked);
  }
}

// CTAs of kThreads that fit on one SM (the persistent grids are SMs x this).
template <typename K>
int resident_ctas(K kernel) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, 0) != cudaSuccess || n < 1) n = 1;
  return n;
}

template <typename T>
void sweep_grids(int sms, int64_t n_blocks, unsigned* g_amax, unsigned* g_quant) {
  static const int occ_a = resident_ctas(amax_kernel<T>);
  static const int occ_q = resident_ctas(quant_kernel<T>);
  const int64_t need = (n_blocks + kThreads - 1) / kThreads;
  *g_amax = unsigned(need < int64_t(sms) * occ_a ? need : int64_t(sms) * occ_a);
  *g_quant = unsigned(need < int64_t(sms) * occ_q ? need : int64_t(sms) * occ_q);
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" size_t rb2_nvfp4_quantize_workspace_size(int64_t M, int64_t K) {
  (void)M; (void)K;
  return 256;
}

extern "C" int rb2_nvfp4_quantize(const void* x, int64_t M, int64_t K, int dtype, int use_rht,
                                  int stochastic, uint64_t seed, uint8_t* codes, uint8_t* scales,
                                  uint8_t* scales_blocked, float* gscale, void* ws,
                                  size_t ws_bytes, void* stream) {
  RB2_CHECK_ARG(M > 0 && K > 0 && K % 16 == 0, "nvfp4_quantize: need M, K > 0 and K %% 16 == 0 (M=%lld K=%lld)",
                (long long)M, (long long)K);
  RB2_CHECK_ARG(dtype == RB2_F32 || dtype == RB2_BF16, "nvfp4_quantize: dtype must be F32 or BF16");
  RB2_CHECK_ARG(M * (K / 16) < (int64_t(1) << 31), "nvfp4_quantize: more than 2^31 blocks of 16 (M=%lld K=%lld)",
                (long long)M, (long long)K);
  RB2_CHECK_ARG(x && codes && scales && gscale && ws, "nvfp4_quantize: null pointer");
  RB2_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(codes) & 7) == 0,
                "nvfp4_quantize: x must be 16-byte and codes 8-byte aligned");
  if (ws_bytes < rb2_nvfp4_quantize_workspace_size(M, K)) {
    set_error("nvfp4_quantize: workspace too small");
    return RB2_EWORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int* gmax = static_cast<unsigned int*>(ws);
  const int64_t n_blocks = M * (K / 16);
  const int64_t groups = K / 16;
  const Divider div = make_divider(uint32_t(groups));
  // the blocked layout pads rows to 128 and scale columns to 4; the pads must read as zero
  const bool pads = scales_blocked && (M % 128 != 0 || groups % 4 != 0);
  const size_t nb = size_t((M + 127) / 128) * size_t((groups + 3) / 4) * 512;
  if (n_blocks <= int64_t(kSmallBlocks)) {
    ProfScope ps_("nvfp4_quant_small", s);
    const size_t clear = pads ? nb : 0;
    if (dtype == RB2_BF16)
      quant_small_kernel<__nv_bfloat16><<<1, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                               uint32_t(n_blocks), uint32_t(groups), div, use_rht,
                                                               stochastic, seed, codes, scales, scales_blocked, clear,
                                                               gscale);
    else
      quant_small_kernel<float><<<1, kThreads, 0, s>>>(static_cast<const float*>(x), uint32_t(n_blocks),
                                                       uint32_t(groups), div, use_rht, stochastic, seed, codes, scales,
                                                       scales_blocked, clear, gscale);
    RB2_CHECK_LAUNCH("nvfp4_quantize: small");
    return RB2_OK;
  }
  { ProfScope ps_("nvfp4_zero", s); zero_word_kernel<<<1, 1, 0, s>>>(gmax); }
  RB2_CHECK_LAUNCH("nvfp4_quantize: zero");
  if (pads) RB2_CUDA(cudaMemsetAsync(scales_blocked, 0, nb, s), "nvfp4_quantize: clear blocked pads");
  int dev = 0, sms = 148;
  RB2_CUDA(cudaGetDevice(&dev), "nvfp4_quantize: device");
  RB2_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "nvfp4_quantize: SM count");
  unsigned ga = 1, gq = 1;
  if (dtype == RB2_BF16) {
    auto xp = static_cast<const __nv_bfloat16*>(x);
    sweep_grids<__nv_bfloat16>(sms, n_blocks, &ga, &gq);
    { ProfScope ps_("nvfp4_amax", s); amax_kernel<__nv_bfloat16><<<ga, kThreads, 0, s>>>(xp, n_blocks, use_rht, gmax); }
    ProfScope ps_("nvfp4_quant", s);
    quant_kernel<__nv_bfloat16><<<gq, kThreads, 0, s>>>(xp, uint32_t(n_blocks), uint32_t(groups), div, use_rht,
                                                        stochastic, seed, gmax, codes, scales, scales_blocked,
                                                        gscale);
  } else {
    auto xp = static_cast<const float*>(x);
    sweep_grids<float>(sms, n_blocks, &ga, &gq);
    { ProfScope ps_("nvfp4_amax", s); amax_kernel<float><<<ga, kThreads, 0, s>>>(xp, n_blocks, use_rht, gmax); }
    ProfScope ps_("nvfp4_quant", s);
    quant_kernel<float><<<gq, kThreads, 0, s>>>(xp, uint32_t(n_blocks), uint32_t(groups), div, use_rht, stochastic,
                                                seed, gmax, codes, scales, scales_blocked, gscale);
  }
  RB2_CHECK_LAUNCH("nvfp4_quantize");
  return RB2_OK;
}

// ------------------------------------------------------------------------------------------------
// The block's gated RMSNorm (RMSNormGated, recant/model/fused_ops.py:11-16: y = bf16(w bf16(x r))
// silu(z) over rows of 128, r = rsqrt(mean x^2 + eps)) fused with the first pass of the NVFP4
// quantizer of y, the out_proj input (layers.py:181 -> QLinear -> quantize_activation,
// nvfp4.py:144-149): the kernel writes y and r and reduces the global amax of rht(y) in the same
// pass, so the quantizer's second pass is the only other read of y.
// 16 threads per row (gated_norm.cuh: thread h holds elements 8h .. 8h + 7, the same arithmetic as
// the stand-alone norm kernel), so each 16-element block of the transform spans lanes 2b, 2b + 1:
// butterflies of stride 1, 2 and 4 stay in the thread, stride 8 pairs lanes l, l ^ 1 by a shuffle;
// the operations and their order are the reference's (as in transform16), so the amax is
// bit-identical to the stand-alone pass.
// ------------------------------------------------------------------------------------------------
namespace rb2 {
namespace {
__global__ void __launch_bounds__(256) gated_norm_amax_kernel(const __nv_bfloat16* __restrict__ x,
                                                              const __nv_bfloat16* __restrict__ z,
                                                              const float* __restrict__ w, int64_t rows, float eps,
                                                              int rot, __nv_bfloat16* __restrict__ y,
                                                              float* __restrict__ rstd, unsigned int* __restrict__ gmax_bits) {
  const int lane = threadIdx.x & 31, hl = lane & 15, jj = hl & 1;
  float w8[8];
  {
    const float4 a = reinterpret_cast<const float4*>(w)[2 * hl], b = reinterpret_cast<const float4*>(w)[2 * hl + 1];
    w8[0] = a.x; w8[1] = a.y; w8[2] = a.z; w8[3] = a.w; w8[4] = b.x; w8[5] = b.y; w8[6] = b.z; w8[7] = b.w;
  }
  // _SIGNS of elements 8 jj .. 8 jj + 7 of the block (negative at 2, 4, 5, 6, 12, 13, 15), bit t = element 8 jj + t
  const uint32_t neg = jj ? 0xB0u : 0x74u;
  float m = 0.f;
  const int64_t warp = (int64_t(blockIdx.x) * 256 + threadIdx.x) >> 5, nwarps = int64_t(gridDim.x) * 8;
  for (int64_t row0 = warp * 4 + (lane >> 4); row0 - (lane >> 4) < rows; row0 += nwarps * 4) {
    uint4 ux[2], uz[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t row = row0 + 2 * u;
      ux[u] = row < rows ? reinterpret_cast<const uint4*>(x + row * 128)[hl] : make_uint4(0, 0, 0, 0);
      uz[u] = row < rows ? reinterpret_cast<const uint4*>(z + row * 128)[hl] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t row = row0 + 2 * u;
      float x8[8], z8[8], v[8];
      gn_unpack8(ux[u], x8);
      gn_unpack8(uz[u], z8);
      const float r = gated_norm8(x8, z8, w8, eps, v);
      if (row < rows) {
        reinterpret_cast<uint4*>(y + row * 128)[hl] = gn_pack8(v);
        if (hl == 0 && rstd) rstd[row] = r;
      }
      if (rot) {
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = (neg >> t) & 1u ? -v[t] : v[t];
#pragma unroll
        for (int st = 1; st < 8; st <<= 1) {  // strides 1, 2, 4 inside the thread
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            if ((t & st) == 0) {
              const float a = v[t], b = v[t + st];
              v[t] = __fadd_rn(a, b);
              v[t + st] = __fsub_rn(a, b);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {  // stride 8: lanes l, l ^ 1; the lower lane keeps a + b
          const float o = __shfl_xor_sync(0xffffffffu, v[t], 1);
          v[t] = jj ? __fsub_rn(o, v[t]) : __fadd_rn(v[t], o);
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = gn_bf16_round(__fmul_rn(v[t], 0.25f));
      }
      if (row < rows) {
#pragma unroll
        for (int t = 0; t < 8; ++t) m = fmaxf(m, fabsf(v[t]));
      }
    }
  }
  m = warp_max(m);
  __shared__ float red[8];
  if (lane == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float q = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    q = warp_max(q);
    if (threadIdx.x == 0 && q > 0.f) atomicMax(gmax_bits, __float_as_uint(q));
  }
}
}  // namespace
}  // namespace rb2

extern "C" int rb2_gated_rmsnorm_nvfp4_fwd(const void* x, const void* z, const float* w, int64_t rows, int dim,
                                           float eps, void* y, float* rstd, int64_t M, int64_t K, int use_rht,
                                           uint8_t* codes, uint8_t* scales, uint8_t* scales_blocked, float* gscale,
                                           void* ws, size_t ws_bytes, void* stream) {
  RB2_CHECK_ARG(dim == 128, "gated_rmsnorm_nvfp4: row length must be 128 (got %d)", dim);
  RB2_CHECK_ARG(rows > 0 && M > 0 && K > 0 && K % 16 == 0 && rows * 128 == M * K,
                "gated_rmsnorm_nvfp4: rows x 128 must equal M x K with K %% 16 == 0 (rows=%lld M=%lld K=%lld)",
                (long long)rows, (long long)M, (long long)K);
  RB2_CHECK_ARG(M * (K / 16) < (int64_t(1) << 31), "gated_rmsnorm_nvfp4: more than 2^31 blocks of 16");
  RB2_CHECK_ARG(x && z && w && y && rstd && codes && scales && gscale && ws, "gated_rmsnorm_nvfp4: null pointer");
  RB2_CHECK_ARG(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(w) |
                  reinterpret_cast<uintptr_t>(y)) & 15) == 0 && (reinterpret_cast<uintptr_t>(codes) & 7) == 0,
                "gated_rmsnorm_nvfp4: x, z, w, y must be 16-byte and codes 8-byte aligned");
  if (ws_bytes < rb2_nvfp4_quantize_workspace_size(M, K)) {
    set_error("gated_rmsnorm_nvfp4: workspace too small");
    return RB2_EWORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int* gmax = static_cast<unsigned int*>(ws);
  const int64_t n_blocks = M * (K / 16), groups = K / 16;
  const Divider div = make_divider(uint32_t(groups));
  const bool pads = scales_blocked && (M % 128 != 0 || groups % 4 != 0);
  const size_t nb = size_t((M + 127) / 128) * size_t((groups + 3) / 4) * 512;
  { ProfScope ps_("nvfp4_zero", s); zero_word_kernel<<<1, 1, 0, s>>>(gmax); }
  RB2_CHECK_LAUNCH("gated_rmsnorm_nvfp4: zero");
  if (pads) RB2_CUDA(cudaMemsetAsync(scales_blocked, 0, nb, s), "gated_rmsnorm_nvfp4: clear blocked pads");
  int dev = 0, sms = 148;
  RB2_CUDA(cudaGetDevice(&dev), "gated_rmsnorm_nvfp4: device");
  RB2_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "gated_rmsnorm_nvfp4: SM count");
  {
    ProfScope ps_("block_gated_norm_amax", s);
    const int64_t need = (rows + 31) / 32;  // 8 warps x 4 rows per CTA step
    const unsigned g = unsigned(need < int64_t(sms) * 8 ? need : int64_t(sms) * 8);
    gated_norm_amax_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(z),
                                             w, rows, eps, use_rht, static_cast<__nv_bfloat16*>(y), rstd, gmax);
  }
  RB2_CHECK_LAUNCH("gated_rmsnorm_nvfp4: norm + amax");
  unsigned ga = 1, gq = 1;
  sweep_grids<__nv_bfloat16>(sms, n_blocks, &ga, &gq);
  {
    ProfScope ps_("nvfp4_quant", s);
    quant_kernel<__nv_bfloat16><<<gq, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(y), uint32_t(n_blocks),
                                                        uint32_t(groups), div, use_rht, 0, 0, gmax, codes, scales,
                                                        scales_blocked, gscale);
  }
  RB2_CHECK_LAUNCH("gated_rmsnorm_nvfp4: quantize");
  return RB2_OK;
}

namespace rb2 {
namespace {
__global__ void __launch_bounds__(256) block_scales_kernel(const uint8_t* __restrict__ scales, int64_t rows, int64_t cols,
                                                           uint8_t* __restrict__ blocked) {
  const int64_t n = rows * cols, ncb = (cols + 3) / 4;
  for (int64_t i = int64_t(blockIdx.x) * 256 + threadIdx.x; i < n; i += int64_t(gridDim.x) * 256) {
    const int64_t r = i / cols, c = i % cols;
    blocked[((r >> 7) * ncb + (c >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (c & 3)] = scales[i];
  }
}
}  // namespace
}  // namespace rb2

extern "C" int rb2_nvfp4_block_scales(const uint8_t* scales, int64_t rows, int64_t cols, uint8_t* blocked,
                                      void* stream) {
  RB2_CHECK_ARG(rows > 0 && cols > 0 && scales && blocked, "nvfp4_block_scales: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t nb = size_t((rows + 127) / 128) * size_t((cols + 3) / 4) * 512;
  RB2_CUDA(cudaMemsetAsync(blocked, 0, nb, s), "nvfp4_block_scales: clear");
  {
    ProfScope ps_("nvfp4_block_scales", s);
    block_scales_kernel<<<148 * 4, 256, 0, s>>>(scales, rows, cols, blocked);
  }
  RB2_CHECK_LAUNCH("nvfp4_block_scales");
  return RB2_OK;
}

// ------------------------------------------------------------------------------------------------
// Allocation-free variant of rb2_nvfp4_quantize.
//
// Some callers cannot hand the library a workspace: C or C++ code that embeds the library without
// a device allocator of its own, serving loops that run with the caching allocator frozen, and
// code paths where a cudaMalloc would synchronise the device or fail under a memory cap. For them
// the quantizer's only scratch -- the word that collects the global |x| maximum -- lives in a
// file-scope device array instead. That array exists once per GPU that loads the library and stays
// allocated until the process exits. Every call shares it: the kernel clears the word at the start
// of each call, and calls whose kernels overlap on the GPU (two streams at once) race on it.
// The scratch is one word for every shape, so no size is rejected today; the size check below
// guards the array's stated maximum should the quantizer ever need more.
// ------------------------------------------------------------------------------------------------
#include <cudaTypedefs.h>
#include <mutex>

namespace rb2 {
namespace {
constexpr size_t kQuantStaticScratchBytes = 256;
__device__ __align__(256) unsigned char g_quant_scratch[kQuantStaticScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchSlot {
  unsigned long long ctx_id = 0;  // the CUDA context the address belongs to (0: none yet)
  void* ptr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// Unique id of the calling thread's current context (ids are never reused, unlike handles), or 0.
unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_quant_scratch in the current context. In host code the name g_quant_scratch
// is only a host-side stand-in, so the address is looked up with cudaGetSymbolAddress on the first
// call that runs on a device, and again whenever that device's context has changed since (after a
// cudaDeviceReset the module is loaded anew and the old address is gone).
int static_scratch(void** out) {
  int dev = 0;
  RB2_CUDA(cudaGetDevice(&dev), "nvfp4_quantize_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("nvfp4_quantize_noalloc: device ordinal %d out of range", dev);
    return RB2_EINVAL;
  }
  const unsigned long long ctx = current_context_id();  // 0 before the thread's first CUDA call
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  if (!slot.ptr || ctx == 0 || slot.ctx_id != ctx) {
    void* p = nullptr;
    // (this also makes the device's primary context current if the thread had none yet)
    RB2_CUDA(cudaGetSymbolAddress(&p, g_quant_scratch), "nvfp4_quantize_noalloc: cudaGetSymbolAddress");
    slot.ptr = p;
    slot.ctx_id = current_context_id();
  }
  *out = slot.ptr;
  return RB2_OK;
}
}  // namespace
}  // namespace rb2

extern "C" int rb2_nvfp4_quantize_noalloc(const void* x, int64_t M, int64_t K, int dtype, int use_rht,
                                          int stochastic, uint64_t seed, uint8_t* codes, uint8_t* scales,
                                          uint8_t* scales_blocked, float* gscale, void* stream) {
  const size_t need = rb2_nvfp4_quantize_workspace_size(M, K);
  if (need > rb2::kQuantStaticScratchBytes) {  // unreachable today (one word for every shape); a guard
    rb2::set_error("nvfp4_quantize_noalloc: M=%lld K=%lld needs %zu bytes of scratch, more than the %zu-byte static "
                   "buffer; use rb2_nvfp4_quantize with a workspace",
                   (long long)M, (long long)K, need, rb2::kQuantStaticScratchBytes);
    return RB2_EWORKSPACE;
  }
  void* scratch = nullptr;
  const int rc = rb2::static_scratch(&scratch);
  if (rc) return rc;
  return rb2_nvfp4_quantize(x, M, K, dtype, use_rht, stochastic, seed, codes, scales, scales_blocked, gscale, scratch,
                            rb2::kQuantStaticScratchBytes, stream);
}
