// The gated RMSNorm of one 128-element row (RMSNormGated, recant/model/fused_ops.py:11-16):
// y = bf16(bf16(w bf16(x r)) silu(z)), r = rsqrt(mean x^2 + eps), shared by the stand-alone norm
// kernel (gdn_block.cu) and the norm fused with the NVFP4 quantizer's amax (nvfp4_quant.cu), so that
// both give bit-identical y and r. Layout: 16 threads per row, thread h (= lane & 15) holds
// elements 8h .. 8h + 7 (one 16-byte load per tensor); a warp covers two rows.
#pragma once

#include "common.cuh"

namespace rb2 {

__device__ __forceinline__ float gn_bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void gn_unpack8(const uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 gn_pack8(const float (&v)[8]) {
  uint32_t p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    p[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(p[0], p[1], p[2], p[3]);
}

// All 32 lanes call this (the row sum reduces over each half-warp). x8, z8: this thread's 8 inputs;
// w8: the norm weights of its 8 columns. Returns r; out: the 8 outputs (bf16 values as float).
__device__ __forceinline__ float gated_norm8(const float (&x8)[8], const float (&z8)[8], const float (&w8)[8], float eps,
                                             float (&out)[8]) {
  float ss = x8[0] * x8[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) ss = fmaf(x8[i], x8[i], ss);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss * (1.f / 128.f) + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float zs = z8[i] * (1.f / (1.f + __expf(-z8[i])));  // silu
    out[i] = gn_bf16_round(gn_bf16_round(w8[i] * gn_bf16_round(x8[i] * r)) * zs);
  }
  return r;
}

}  // namespace rb2
