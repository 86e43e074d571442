// Element-wise kernels of the GDN block around the chunked op (recant/model/layers.py:148-182):
//   causal depthwise conv (kernel 4, zero prefix) + SiLU over the qkv channels   layers.py:157-168
//   gates g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)               fused_ops.py:32-33,
//                                                                                 layers.py:154
//   gated RMSNorm y = w * bf16(x rsqrt(mean x^2 + eps)) * silu(z) per 128-row     fused_ops.py:11-16
// with the backward of each (the block's conv, gate and norm weights are frozen: only input
// gradients). All are HBM-bound: 16-byte loads and stores, fp32 arithmetic, the reference's
// roundings to bf16 where its eager code casts.
#include "common.cuh"
#include "gated_norm.cuh"

namespace rb2 {
namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x * sigm(x); }

constexpr int kConvK = 4;

// The conv's C channels, written to (or their gradients read from) up to three contiguous tensors:
// channels [0, s1) -> p0 (width s1), [s1, s2) -> p1, [s2, C) -> p2 (s1 = s2 = C: one tensor).
struct Split {
  bf16* p[3];
  int s1, s2, C;
  __device__ __forceinline__ bf16* at(int64_t tok, int c) const {
    if (c < s1) return p[0] + tok * s1 + c;
    if (c < s2) return p[1] + tok * (s2 - s1) + (c - s1);
    return p[2] + tok * (C - s2) + (c - s2);
  }
};
// One CTA: a tile of kTileT tokens x kTileC channels of one sequence. The tile and its 3-row halo
// are copied to shared memory with 16-byte cp.async (zero-filled before token 0 and past T), all
// copies in flight at once; each thread then works on one 4-channel group and a run of 8 rows
// (64 threads per row, 4 row groups; few registers, so 4 CTAs share an SM and hide the copies).
constexpr int kTileT = 32, kTileC = 256, kChunks = kTileC / 8, kGroups = kTileC / 4;
constexpr int kHalo = kConvK - 1;
constexpr int kRowGroups = 256 / kGroups, kRowsPer = kTileT / kRowGroups;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

__device__ __forceinline__ void load4(const bf16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  v[0] = __uint_as_float(u.x << 16); v[1] = __uint_as_float(u.x & 0xffff0000u);
  v[2] = __uint_as_float(u.y << 16); v[3] = __uint_as_float(u.y & 0xffff0000u);
}
__device__ __forceinline__ void store4(bf16* p, const float (&v)[4]) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}
__device__ __forceinline__ void load_taps4(const bf16* w, int c, float (&wt)[kConvK][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint2 u = *reinterpret_cast<const uint2*>(w + int64_t(c + i) * kConvK);
    wt[0][i] = __uint_as_float(u.x << 16); wt[1][i] = __uint_as_float(u.x & 0xffff0000u);
    wt[2][i] = __uint_as_float(u.y << 16); wt[3][i] = __uint_as_float(u.y & 0xffff0000u);
  }
}
// silu with a fast reciprocal (sigmoid to a few ulp; the output is rounded to bf16)
__device__ __forceinline__ float fsigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// 8 channels of token t < 0 from the cached prefix prev [B, C, 3] (token t = column 3 + t; the
// reference's LayerCache.conv_state, layers.py:159-166), or zeros without one
__device__ __forceinline__ void halo_from_prev(bf16* dst, const bf16* prev, int b, int C, int c, int t) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bf16 lo = prev[(int64_t(b) * C + c + 2 * i) * kHalo + kHalo + t];
    const bf16 hi = prev[(int64_t(b) * C + c + 2 * i + 1) * kHalo + kHalo + t];
    w[i] = uint32_t(__bfloat16_as_ushort(lo)) | (uint32_t(__bfloat16_as_ushort(hi)) << 16);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

struct TileIdx {
  int b, t0, c0, nchunk;
};
__device__ __forceinline__ TileIdx tile_of(int64_t tile, int T, int C) {
  const int ct = (C + kTileC - 1) / kTileC, tt = (T + kTileT - 1) / kTileT;
  TileIdx r;
  r.c0 = int(tile % ct) * kTileC;
  r.t0 = int((tile / ct) % tt) * kTileT;
  r.b = int(tile / (int64_t(ct) * tt));
  r.nchunk = min(kChunks, (C - r.c0) / 8);
  return r;
}

// y[b, t, c] = bf16(silu(bf16(sum_j w[c, j] x[b, t - 3 + j, c])))
__global__ void __launch_bounds__(256, 4) conv_silu_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                               const bf16* __restrict__ prev, int B, int T, int C,
                                                               Split y) {
  __shared__ __align__(16) bf16 xs[kTileT + kHalo][kTileC];  // row i = token t0 - 3 + i
  const TileIdx ti = tile_of(blockIdx.x, T, C);
  const bf16* xb = x + int64_t(ti.b) * T * C + ti.c0;
  for (int e = threadIdx.x; e < (kTileT + kHalo) * kChunks; e += 256) {
    const int r = e / kChunks, ch = e % kChunks, t = ti.t0 - kHalo + r;
    if (t < 0 && prev && ch < ti.nchunk) {
      halo_from_prev(&xs[r][ch * 8], prev, ti.b, C, ti.c0 + ch * 8, t);
      continue;
    }
    const bool ok = ch < ti.nchunk && t >= 0 && t < T;
    cp_async16(&xs[r][ch * 8], ok ? xb + int64_t(t) * C + ch * 8 : x, ok);
  }
  cp_async_wait_all();
  __syncthreads();
  const int g = threadIdx.x % kGroups, r0 = (threadIdx.x / kGroups) * kRowsPer;
  if (g >= 2 * ti.nchunk) return;
  const int c = ti.c0 + g * 4;
  float wt[kConvK][4];
  load_taps4(w, c, wt);
  float win[kConvK][4];
#pragma unroll
  for (int j = 0; j < kHalo; ++j) load4(&xs[r0 + j][g * 4], win[j]);
#pragma unroll
  for (int k = 0; k < kRowsPer; ++k) {
    const int t = ti.t0 + r0 + k;
    load4(&xs[r0 + k + kHalo][g * 4], win[kHalo]);
    float out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = wt[0][i] * win[0][i];
      a = fmaf(wt[1][i], win[1][i], a);
      a = fmaf(wt[2][i], win[2][i], a);
      a = fmaf(wt[3][i], win[3][i], a);
      const float u = bfr(a);
      out[i] = u * fsigm(u);
      win[0][i] = win[1][i]; win[1][i] = win[2][i]; win[2][i] = win[3][i];
    }
    if (t < T) store4(y.at(int64_t(ti.b) * T + t, c), out);
  }
}

// du[t] = bf16(dy[t] silu'(u[t])) (u recomputed, bf16 as in the forward) for t in [t0, t0 + 35);
// dx[t] = sum_j w[c, j] du[t + 3 - j] for t in [t0, t0 + 32)
__global__ void __launch_bounds__(256, 4) conv_silu_bwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                               const bf16* __restrict__ prev, Split dy, int B, int T,
                                                               int C, bf16* __restrict__ dx) {
  __shared__ __align__(16) bf16 xs[kTileT + 2 * kHalo][kTileC];  // row i = token t0 - 3 + i
  __shared__ __align__(16) bf16 ds[kTileT + kHalo][kTileC];      // row i = token t0 + i: dy, then du
  const TileIdx ti = tile_of(blockIdx.x, T, C);
  const bf16* xb = x + int64_t(ti.b) * T * C + ti.c0;
  for (int e = threadIdx.x; e < (kTileT + 2 * kHalo) * kChunks; e += 256) {
    const int r = e / kChunks, ch = e % kChunks, t = ti.t0 - kHalo + r;
    if (t < 0 && prev && ch < ti.nchunk) {
      halo_from_prev(&xs[r][ch * 8], prev, ti.b, C, ti.c0 + ch * 8, t);
      continue;
    }
    const bool ok = ch < ti.nchunk && t >= 0 && t < T;
    cp_async16(&xs[r][ch * 8], ok ? xb + int64_t(t) * C + ch * 8 : x, ok);
  }
  for (int e = threadIdx.x; e < (kTileT + kHalo) * kChunks; e += 256) {
    const int r = e / kChunks, ch = e % kChunks, t = ti.t0 + r;
    const bool ok = ch < ti.nchunk && t < T;
    cp_async16(&ds[r][ch * 8], ok ? static_cast<const bf16*>(dy.at(int64_t(ti.b) * T + t, ti.c0 + ch * 8)) : x, ok);
  }
  cp_async_wait_all();
  __syncthreads();
  const int g = threadIdx.x % kGroups, grp = threadIdx.x / kGroups;
  const bool active = g < 2 * ti.nchunk;
  const int c = ti.c0 + g * 4;
  float wt[kConvK][4];
  if (active) load_taps4(w, c, wt);
  // phase 1: 35 du rows over the row groups (9 rows each, the last one short); zero-filled dy gives du = 0
  constexpr int kDuRows = kTileT + kHalo, kPer = (kDuRows + kRowGroups - 1) / kRowGroups;
  if (active) {
    const int r0 = grp * kPer;
    float win[kConvK][4];
#pragma unroll
    for (int j = 0; j < kHalo; ++j) load4(&xs[r0 + j][g * 4], win[j]);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int r = r0 + k;
      if (r >= kDuRows) break;
      load4(&xs[r + kHalo][g * 4], win[kHalo]);
      float gr[4], du[4];
      load4(&ds[r][g * 4], gr);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float a = wt[0][i] * win[0][i];
        a = fmaf(wt[1][i], win[1][i], a);
        a = fmaf(wt[2][i], win[2][i], a);
        a = fmaf(wt[3][i], win[3][i], a);
        const float pre = bfr(a), sg = fsigm(pre);
        du[i] = gr[i] * sg * (1.f + pre * (1.f - sg));
        win[0][i] = win[1][i]; win[1][i] = win[2][i]; win[2][i] = win[3][i];
      }
      store4(&ds[r][g * 4], du);
    }
  }
  __syncthreads();
  // phase 2: dx rows r0 .. r0 + 7 from du rows r0 .. r0 + 10
  if (!active) return;
  const int r0 = grp * kRowsPer;
  float dw[kConvK][4];
#pragma unroll
  for (int j = 0; j < kHalo; ++j) load4(&ds[r0 + j][g * 4], dw[j]);
#pragma unroll
  for (int k = 0; k < kRowsPer; ++k) {
    const int t = ti.t0 + r0 + k;
    load4(&ds[r0 + k + kHalo][g * 4], dw[kHalo]);
    float out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = wt[0][i] * dw[3][i];
      a = fmaf(wt[1][i], dw[2][i], a);
      a = fmaf(wt[2][i], dw[1][i], a);
      a = fmaf(wt[3][i], dw[0][i], a);
      out[i] = a;
      dw[0][i] = dw[1][i]; dw[1][i] = dw[2][i]; dw[2][i] = dw[3][i];
    }
    if (t < T) store4(dx + (int64_t(ti.b) * T + t) * C + c, out);
  }
}

// The next call's prefix: the last 3 tokens of cat(prev, x) per channel, [B, C, 3] (layers.py:165-166).
// out may be prev (in-place update): a thread owns one channel and reads prev[T + j] before writing
// out[j], j ascending, so no entry is overwritten before it is read (no __restrict__ on the two).
__global__ void conv_state_kernel(const bf16* __restrict__ x, const bf16* prev, int B, int T, int C, bf16* out) {
  const int64_t n = int64_t(B) * C;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int c = int(i % C), b = int(i / C);
#pragma unroll
    for (int j = 0; j < kHalo; ++j) {
      const int p = T + j;  // position in cat(prev, x)
      bf16 val = __float2bfloat16_rn(0.f);
      if (p >= kHalo) val = x[(int64_t(b) * T + p - kHalo) * C + c];
      else if (prev) val = prev[i * kHalo + p];
      out[i * kHalo + j] = val;
    }
  }
}

// g = -exp(A_log[h]) softplus(a + dt_bias[h]) (fp32), beta = bf16(sigmoid(b)); softplus as torch
// (threshold 20: x > 20 -> x)
__global__ void __launch_bounds__(256) gates_fwd_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b,
                                                        const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                                                        int64_t n, int H, float* __restrict__ g, bf16* __restrict__ beta) {
  for (int64_t i = int64_t(blockIdx.x) * 256 + threadIdx.x; i < n; i += int64_t(gridDim.x) * 256) {
    const int h = int(i % H);
    const float x = __bfloat162float(a[i]) + dt_bias[h];
    const float sp = x > 20.f ? x : log1pf(expf(x));
    g[i] = -expf(A_log[h]) * sp;
    beta[i] = __float2bfloat16_rn(1.f / (1.f + expf(-__bfloat162float(b[i]))));
  }
}
// da = dg (-exp(A_log)) sigmoid(a + dt_bias); db = dbeta beta (1 - beta) with the forward's bf16 beta
__global__ void __launch_bounds__(256) gates_bwd_kernel(const bf16* __restrict__ a, const bf16* __restrict__ beta,
                                                        const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                                                        const float* __restrict__ dg, const bf16* __restrict__ dbeta,
                                                        int64_t n, int H, bf16* __restrict__ da, bf16* __restrict__ db) {
  for (int64_t i = int64_t(blockIdx.x) * 256 + threadIdx.x; i < n; i += int64_t(gridDim.x) * 256) {
    const int h = int(i % H);
    const float x = __bfloat162float(a[i]) + dt_bias[h];
    const float ds = x > 20.f ? 1.f : 1.f / (1.f + expf(-x));
    da[i] = __float2bfloat16_rn(dg[i] * -expf(A_log[h]) * ds);
    const float bt = __bfloat162float(beta[i]);
    db[i] = __float2bfloat16_rn(__bfloat162float(dbeta[i]) * bt * (1.f - bt));
  }
}

// one warp per row of 128 (4 per lane); rstd kept for the backward
__global__ void __launch_bounds__(256) gated_norm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z,
                                                             const float* __restrict__ w, int64_t rows, float eps,
                                                             bf16* __restrict__ y, float* __restrict__ rstd) {
  // 16 threads per row (gated_norm.cuh), two rows per warp, two row pairs per warp and step
  const int lane = threadIdx.x & 31, hl = lane & 15;
  float w8[8];
  {
    const float4 a = reinterpret_cast<const float4*>(w)[2 * hl], b = reinterpret_cast<const float4*>(w)[2 * hl + 1];
    w8[0] = a.x; w8[1] = a.y; w8[2] = a.z; w8[3] = a.w; w8[4] = b.x; w8[5] = b.y; w8[6] = b.z; w8[7] = b.w;
  }
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
      float x8[8], z8[8], o[8];
      gn_unpack8(ux[u], x8);
      gn_unpack8(uz[u], z8);
      const float r = gated_norm8(x8, z8, w8, eps, o);
      if (row < rows) {
        reinterpret_cast<uint4*>(y + row * 128)[hl] = gn_pack8(o);
        if (hl == 0 && rstd) rstd[row] = r;
      }
    }
  }
}
// out = bf16(w n) silu(z), n = bf16(x r): dz = dout bf16(w n) silu'(z); dn = dout w silu(z);
// dx = r (dn - xh mean(dn xh)), xh = x r
__global__ void __launch_bounds__(256) gated_norm_bwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z,
                                                             const float* __restrict__ w, const float* __restrict__ rstd,
                                                             const bf16* __restrict__ dout, int64_t rows,
                                                             bf16* __restrict__ dx, bf16* __restrict__ dz) {
  const int lane = threadIdx.x & 31;
  const float4 wv = reinterpret_cast<const float4*>(w)[lane];
  const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
  // four rows per warp and step, their loads issued together (the rows are short: 256 bytes each)
  constexpr int kU = 4;
  const int64_t warp = (int64_t(blockIdx.x) * 256 + threadIdx.x) >> 5, nwarps = int64_t(gridDim.x) * 8;
  for (int64_t row0 = warp * kU; row0 < rows; row0 += nwarps * kU) {
    uint2 uxs[kU], uzs[kU], uds[kU];
    float rs[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (row0 + u < rows) {
        uxs[u] = reinterpret_cast<const uint2*>(x + (row0 + u) * 128)[lane];
        uzs[u] = reinterpret_cast<const uint2*>(z + (row0 + u) * 128)[lane];
        uds[u] = reinterpret_cast<const uint2*>(dout + (row0 + u) * 128)[lane];
        rs[u] = rstd[row0 + u];
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t row = row0 + u;
      if (row >= rows) break;
      const uint2 ux = uxs[u], uz = uzs[u], ud = uds[u];
      const float xv[4] = {__uint_as_float(ux.x << 16), __uint_as_float(ux.x & 0xffff0000u),
                           __uint_as_float(ux.y << 16), __uint_as_float(ux.y & 0xffff0000u)};
      const float zv[4] = {__uint_as_float(uz.x << 16), __uint_as_float(uz.x & 0xffff0000u),
                           __uint_as_float(uz.y << 16), __uint_as_float(uz.y & 0xffff0000u)};
      const float gv[4] = {__uint_as_float(ud.x << 16), __uint_as_float(ud.x & 0xffff0000u),
                           __uint_as_float(ud.y << 16), __uint_as_float(ud.y & 0xffff0000u)};
      const float r = rs[u];
      float dn[4], dzv[4], dot = 0.f;
  #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float s = sigm(zv[i]);
        const float wn = bfr(wa[i] * bfr(xv[i] * r));
        dzv[i] = gv[i] * wn * s * (1.f + zv[i] * (1.f - s));
        dn[i] = gv[i] * wa[i] * zv[i] * s;
        dot += dn[i] * xv[i] * r;
      }
      dot = warp_sum(dot) * (1.f / 128.f);
      float dxv[4];
  #pragma unroll
      for (int i = 0; i < 4; ++i) dxv[i] = r * (dn[i] - xv[i] * r * dot);
      const __nv_bfloat162 a0 = __floats2bfloat162_rn(dxv[0], dxv[1]), a1 = __floats2bfloat162_rn(dxv[2], dxv[3]);
      const __nv_bfloat162 b0 = __floats2bfloat162_rn(dzv[0], dzv[1]), b1 = __floats2bfloat162_rn(dzv[2], dzv[3]);
      reinterpret_cast<uint2*>(dx + row * 128)[lane] =
          make_uint2(*reinterpret_cast<const uint32_t*>(&a0), *reinterpret_cast<const uint32_t*>(&a1));
      reinterpret_cast<uint2*>(dz + row * 128)[lane] =
          make_uint2(*reinterpret_cast<const uint32_t*>(&b0), *reinterpret_cast<const uint32_t*>(&b1));
    }
  }
}

unsigned grid_for(int64_t n, int per_block) {
  const int64_t g = (n + per_block - 1) / per_block;
  return unsigned(g < 148 * 16 ? (g > 0 ? g : 1) : 148 * 16);
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace rb2

using namespace rb2;

namespace rb2 {
namespace {
int make_split(void* p0, void* p1, void* p2, int s1, int s2, int C, Split* out) {
  RB2_CHECK_ARG(p0 && aligned16(p0), "conv_silu: null or misaligned output pointer");
  if (p1 == nullptr && p2 == nullptr) {
    *out = Split{{static_cast<bf16*>(p0), nullptr, nullptr}, C, C, C};
    return RB2_OK;
  }
  RB2_CHECK_ARG(p1 && p2 && aligned16(p1) && aligned16(p2), "conv_silu: null or misaligned split pointer");
  RB2_CHECK_ARG(0 < s1 && s1 < s2 && s2 < C && s1 % 8 == 0 && s2 % 8 == 0,
                "conv_silu: split points must be multiples of 8 with 0 < s1 < s2 < C");
  *out = Split{{static_cast<bf16*>(p0), static_cast<bf16*>(p1), static_cast<bf16*>(p2)}, s1, s2, C};
  return RB2_OK;
}
}  // namespace
}  // namespace rb2

extern "C" int rb2_conv_silu_fwd(const void* x, const void* w, const void* prev, int B, int T, int C, int K, void* y0,
                                 void* y1, void* y2, int s1, int s2, void* new_state, void* stream) {
  RB2_CHECK_ARG(K == kConvK, "conv_silu: kernel size must be 4 (got %d)", K);
  RB2_CHECK_ARG(B >= 1 && T >= 1 && C >= 8 && C % 8 == 0, "conv_silu: bad sizes B=%d T=%d C=%d", B, T, C);
  RB2_CHECK_ARG(x && w && aligned16(x) && (reinterpret_cast<uintptr_t>(w) & 7) == 0,
                "conv_silu: null or misaligned pointer");
  Split y;
  int rc = make_split(y0, y1, y2, s1, s2, C, &y);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = int64_t(B) * ((T + kTileT - 1) / kTileT) * ((C + kTileC - 1) / kTileC);
  RB2_CHECK_ARG(n < (int64_t(1) << 31), "conv_silu: too many tiles (%lld)", (long long)n);
  {
    ProfScope ps_("block_conv_silu_fwd", s);
    conv_silu_fwd_kernel<<<unsigned(n), 256, 0, s>>>(static_cast<const bf16*>(x), static_cast<const bf16*>(w),
                                                      static_cast<const bf16*>(prev), B, T, C, y);
  }
  RB2_CHECK_LAUNCH("conv_silu_fwd");
  if (new_state) {
    ProfScope ps_("block_conv_state", s);
    conv_state_kernel<<<grid_for(int64_t(B) * C, 256), 256, 0, s>>>(
        static_cast<const bf16*>(x), static_cast<const bf16*>(prev), B, T, C, static_cast<bf16*>(new_state));
    RB2_CHECK_LAUNCH("conv_state");
  }
  return RB2_OK;
}

extern "C" int rb2_conv_silu_bwd(const void* x, const void* w, const void* prev, const void* dy0, const void* dy1,
                                 const void* dy2, int s1, int s2, int B, int T, int C, int K, void* dx, void* stream) {
  RB2_CHECK_ARG(K == kConvK, "conv_silu: kernel size must be 4 (got %d)", K);
  RB2_CHECK_ARG(B >= 1 && T >= 1 && C >= 8 && C % 8 == 0, "conv_silu: bad sizes B=%d T=%d C=%d", B, T, C);
  RB2_CHECK_ARG(x && w && dx && aligned16(x) && aligned16(dx) && (reinterpret_cast<uintptr_t>(w) & 7) == 0,
                "conv_silu: null or misaligned pointer");
  Split dy;
  int rc = make_split(const_cast<void*>(dy0), const_cast<void*>(dy1), const_cast<void*>(dy2), s1, s2, C, &dy);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = int64_t(B) * ((T + kTileT - 1) / kTileT) * ((C + kTileC - 1) / kTileC);
  RB2_CHECK_ARG(n < (int64_t(1) << 31), "conv_silu: too many tiles (%lld)", (long long)n);
  ProfScope ps_("block_conv_silu_bwd", s);
  conv_silu_bwd_kernel<<<unsigned(n), 256, 0, s>>>(static_cast<const bf16*>(x), static_cast<const bf16*>(w),
                                                    static_cast<const bf16*>(prev), dy, B, T, C, static_cast<bf16*>(dx));
  RB2_CHECK_LAUNCH("conv_silu_bwd");
  return RB2_OK;
}

extern "C" int rb2_gdn_gates_fwd(const void* a, const void* b, const float* A_log, const float* dt_bias, int64_t n,
                                 int H, float* g, void* beta, void* stream) {
  RB2_CHECK_ARG(n >= 0 && H >= 1 && n % H == 0, "gdn_gates: bad sizes n=%lld H=%d", (long long)n, H);
  RB2_CHECK_ARG(n == 0 || (a && b && A_log && dt_bias && g && beta), "gdn_gates: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps_("block_gates_fwd", s);
  gates_fwd_kernel<<<grid_for(n, 256), 256, 0, s>>>(static_cast<const bf16*>(a), static_cast<const bf16*>(b), A_log,
                                                      dt_bias, n, H, g, static_cast<bf16*>(beta));
  RB2_CHECK_LAUNCH("gdn_gates_fwd");
  return RB2_OK;
}

extern "C" int rb2_gdn_gates_bwd(const void* a, const void* beta, const float* A_log, const float* dt_bias,
                                 const float* dg, const void* dbeta, int64_t n, int H, void* da, void* db,
                                 void* stream) {
  RB2_CHECK_ARG(n >= 0 && H >= 1 && n % H == 0, "gdn_gates: bad sizes n=%lld H=%d", (long long)n, H);
  RB2_CHECK_ARG(n == 0 || (a && beta && A_log && dt_bias && dg && dbeta && da && db), "gdn_gates: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps_("block_gates_bwd", s);
  gates_bwd_kernel<<<grid_for(n, 256), 256, 0, s>>>(static_cast<const bf16*>(a), static_cast<const bf16*>(beta), A_log,
                                                      dt_bias, dg, static_cast<const bf16*>(dbeta), n, H,
                                                      static_cast<bf16*>(da), static_cast<bf16*>(db));
  RB2_CHECK_LAUNCH("gdn_gates_bwd");
  return RB2_OK;
}

extern "C" int rb2_gated_rmsnorm_fwd(const void* x, const void* z, const float* w, int64_t rows, int dim, float eps,
                                     void* y, float* rstd, void* stream) {
  RB2_CHECK_ARG(dim == 128, "gated_rmsnorm: row length must be 128 (got %d)", dim);
  RB2_CHECK_ARG(rows >= 0, "gated_rmsnorm: bad row count");
  RB2_CHECK_ARG(rows == 0 || (x && z && w && y && aligned16(x) && aligned16(z) && aligned16(w) && aligned16(y)),
                "gated_rmsnorm: null or misaligned pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps_("block_gated_norm_fwd", s);
  gated_norm_fwd_kernel<<<grid_for(rows, 32), 256, 0, s>>>(static_cast<const bf16*>(x), static_cast<const bf16*>(z), w,
                                                           rows, eps, static_cast<bf16*>(y), rstd);
  RB2_CHECK_LAUNCH("gated_rmsnorm_fwd");
  return RB2_OK;
}

extern "C" int rb2_gated_rmsnorm_bwd(const void* x, const void* z, const float* w, const float* rstd, const void* dout,
                                     int64_t rows, int dim, void* dx, void* dz, void* stream) {
  RB2_CHECK_ARG(dim == 128, "gated_rmsnorm: row length must be 128 (got %d)", dim);
  RB2_CHECK_ARG(rows >= 0, "gated_rmsnorm: bad row count");
  RB2_CHECK_ARG(rows == 0 || (x && z && w && rstd && dout && dx && dz && aligned16(x) && aligned16(z) &&
                              aligned16(w) && aligned16(dout) && aligned16(dx) && aligned16(dz)),
                "gated_rmsnorm: null or misaligned pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps_("block_gated_norm_bwd", s);
  gated_norm_bwd_kernel<<<grid_for(rows, 32), 256, 0, s>>>(static_cast<const bf16*>(x), static_cast<const bf16*>(z), w,
                                                           rstd, static_cast<const bf16*>(dout), rows,
                                                           static_cast<bf16*>(dx), static_cast<bf16*>(dz));
  RB2_CHECK_LAUNCH("gated_rmsnorm_bwd");
  return RB2_OK;
}
