// NVFP4 block-scaled GEMM on tcgen05: out[M,N] = (A . B^T) * gA * gB.
//
// Replaces the GEMM_BACKENDS of recant/model/nvfp4.py:108-125 (_gemm_emulated, and
// _gemm_scaled_mm = torch._scaled_mm on cuBLASLt with the 128x4 blocked scale swizzle of
// _to_blocked, nvfp4.py:112-119). A = codes [M, K/2] (two e2m1 per byte, even element in the low
// nibble), B = codes [N, K/2]; per-16 e4m3 scales in the blocked layout; fp32 accumulation.
//
// Persistent CTAs (one per SM) walk 128 x 256 output tiles, warp-specialised. The scales are read
// in the blocked layout itself: its 512-byte atom (32 rows x 16 bytes: row r = the 4 scales of rows
// r, r+32, r+64, r+96 for one 64-element K step) is what each 32-lane quarter of the tensor memory
// holds, so one tcgen05.cp.32x128b.warpx4 (the copy engine writes the atom to all four quarters)
// moves a K step of one 128-row block, and no expanded image is built or read:
//   warp 0     producer: TMA (cp.async.bulk.tensor, SW128, no multicast) of the A and B code tiles
//              (128 bytes = 256 K-elements per row per stage) and 1-D bulk copies of the stage's
//              scale atoms (A's row block; B's two 128-row halves) into a 4-stage ring; completion
//              via mbarrier transaction counts;
//   warp 1     MMA: the atom copies into TMEM (lane m, 32-bit column m / 32 of a 4-column group holds
//              row m's scales: A one group per K step, B two (its halves); 12 copies per 4 K steps),
//              then one tcgen05.mma.kind::mxf4nvf4.block_scale.block16 (M=128, N=256, K=64) per K step;
//   warps 2-9  epilogue: TMEM -> registers (each warp: its sub-partition's 32 rows x 128 columns),
//              accumulator released, then * gA gB -> fp32 or bf16 rows while the next tile runs.

#include <atomic>

#include "tmap.cuh"

namespace rb2 {
namespace {

constexpr int BM = 128, BKB = 128;  // tile rows, K bytes per stage (= 256 e2m1)
constexpr int kThreads = 320;  // producer, MMA, 8 epilogue warps

// Tile shape: BN output columns, STAGES smem stages, ACC TMEM accumulator buffers. A stage is
// [A scale atoms | B scale atoms | A codes | B codes]: the atoms first, so that every scale copy
// reads well inside its own stage.
constexpr int kAtom = 512;  // the scales of one 128-row block for one 64-element K step

template <int BN_, int STAGES_, int ACC_>
struct GemmCfg {
  static constexpr int BN = BN_, STAGES = STAGES_, ACC = ACC_;
  static constexpr int A_BYTES = BM * BKB, B_BYTES = BN * BKB;
  static constexpr int SFA_BYTES = 4 * kAtom;                // [4 K steps][atom]
  static constexpr int SFB_BYTES = 2 * 4 * kAtom;            // [2 halves][4 K steps][atom]
  static constexpr int SFA_OFF = 0, SFB_OFF = SFA_BYTES, A_OFF = SFA_BYTES + SFB_BYTES, B_OFF = A_OFF + A_BYTES;
  static constexpr int STAGE_BYTES = B_OFF + B_BYTES;
  static constexpr int LORA_BYTES = BN * 16 * 2;             // the tile's LoRA B rows (r <= 16, bf16)
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;   // + LORA_BYTES for the LoRA variant
  static constexpr int SF_COL0 = ACC * BN;                   // TMEM: accumulators, then scale factors
  static_assert(BN == 256, "B's scales are two 128-row halves");
  static_assert(SF_COL0 + 16 + 32 <= 512, "TMEM budget");
  static_assert(A_OFF % 1024 == 0 && B_OFF % 1024 == 0 && STAGE_BYTES % 1024 == 0, "SW128 alignment");
  static_assert(SMEM + LORA_BYTES <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(tc::smem_u32(smem_dst)),
      "l"(map), "r"(x), "r"(y), "r"(tc::smem_u32(bar))
      : "memory");
}
// smem descriptor of one scale atom (32 rows x 16 bytes) as the source of tcgen05.cp.32x128b, no
// swizzle: 8-row x 16-byte core matrices, consecutive row groups 128 bytes apart (SBO); a single
// 16-byte column, so the leading-dimension offset is unused
__device__ __forceinline__ uint64_t desc_sf_atom(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFF);
  d |= uint64_t(1) << 16;                     // LBO (unused)
  d |= uint64_t(128 >> 4) << 32;              // SBO
  d |= uint64_t(1) << 46;
  return d;                                   // layout type 0 = no swizzle
}
// the atom into 4 consecutive columns of all 128 lanes: lane 32 q + r gets atom row r, q = 0..3
__device__ __forceinline__ void tmem_cp_sf_atom(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// kind::mxf4nvf4 instruction descriptor: e2m1 x e2m1, ue4m3 scales, K-major A and B, dense K=64
__host__ __device__ constexpr uint32_t idesc_nvf4(int M, int N) {
  return (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1 : 0), "r"(sfa_tmem), "r"(sfb_tmem));
}

// 32 lanes x 32 columns of 32-bit TMEM into registers, without waiting (tcgen05.wait::ld follows)
__device__ __forceinline__ void tmem_ld32_raw(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

// Persistent: CTA c handles tiles c, c + gridDim.x, ... (tile t -> row block t / ntn, column block
// t % ntn, so concurrently running CTAs share A row blocks in L2). The producer streams stages
// across tile boundaries; the single TMEM accumulator is handed between the MMA warp and the
// epilogue warps with acc_full / acc_empty.
// Optional low-rank term added in the epilogue: out = y + s * h B^T with h [M, r] (row stride ldh)
// and B [N, r] bf16, r 8 or 16 -- QLinear's LoRA (layers.py:65-70, 86-97) with h = x A^T computed
// by the caller, rounded as the reference rounds it when the output is bf16:
//   mode 0 (grouped_linear's addmm, layers.py:86-97): y rounded to bf16, plus s (h B^T) rounded to
//          bf16, the sum rounded (torch.addmm on the GPU: cuBLAS rounds the scaled product first);
//   mode 1 (QLinear.forward, layers.py:65-70): y, h B^T and (h B^T) s each rounded to bf16, then
//          their sum rounded.
struct Lora {
  const __nv_bfloat16* h;
  const __nv_bfloat16* b;
  int64_t ldh;
  int r;
  float s;
  int mode;
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void unpack8(const uint4 u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <class C, bool kLora>
__global__ void __launch_bounds__(kThreads, 1)
nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb, int nrb_b, const float* __restrict__ ga,
                  const float* __restrict__ gb, int M, int N, int K, void* __restrict__ out, int out_bf16,
                  Lora lora, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023);
  constexpr int BN = C::BN, STAGES = C::STAGES, ACC = C::ACC;
  constexpr int A_BYTES = C::A_BYTES, B_BYTES = C::B_BYTES, STAGE_BYTES = C::STAGE_BYTES;
  __shared__ uint64_t full[STAGES], empty[STAGES], acc_full[ACC], acc_empty[ACC];
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int ksteps = K / 64;                       // 64-element MMA steps
  const int nstages = (ksteps + 3) / 4;            // 4 steps per stage
  const int ntm = (M + BM - 1) / BM, ntn = (N + BN - 1) / BN, ntiles = ntm * ntn;

  if (w == 1) {
    tc::tmem_alloc(&tmem_base, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < ACC; ++b) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 8);   // one arrival per epilogue warp
    }
    tc::fence_mbar_init();
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;

  if (w == 0) {
    if (l == 0) {  // ---------------- producer ----------------
      int g = 0;   // global stage counter
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int tm = t / ntn, tn = t % ntn;
        for (int kt = 0; kt < nstages; ++kt, ++g) {
          const int s = g % STAGES;
          if (!(ok = tc::mbar_wait(&empty[s], ((g / STAGES) & 1) ^ 1, err, 201))) break;
          unsigned char* st = sm + s * STAGE_BYTES;
          const int steps = min(4, ksteps - 4 * kt);
          // blocked scales: atom (row block, K step) at (row block * K steps + K step) * 512; B's second
          // half is absent past the last row block (its output columns are not stored)
          const uint32_t sf = uint32_t(steps) * kAtom;
          const bool half1 = 2 * tn + 1 < nrb_b;
          tc::mbar_expect_tx(&full[s], A_BYTES + B_BYTES + sf * (half1 ? 3u : 2u));
          tma_load_2d(st + C::A_OFF, &map_a, kt * BKB, tm * BM, &full[s]);
          tma_load_2d(st + C::B_OFF, &map_b, kt * BKB, tn * BN, &full[s]);
          tc::bulk_load(st + C::SFA_OFF, sfa + (size_t(tm) * ksteps + 4 * kt) * kAtom, sf, &full[s]);
          tc::bulk_load(st + C::SFB_OFF, sfb + (size_t(2 * tn) * ksteps + 4 * kt) * kAtom, sf, &full[s]);
          if (half1)
            tc::bulk_load(st + C::SFB_OFF + 4 * kAtom, sfb + (size_t(2 * tn + 1) * ksteps + 4 * kt) * kAtom, sf, &full[s]);
        }
      }
    }
  } else if (w == 1) {
    if (l == 0) {  // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_nvf4(BM, BN);
      const uint32_t t_sfa = tbase + C::SF_COL0, t_sfb = t_sfa + 16;
      int g = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++local) {
        const int ab = local % ACC;
        const uint32_t t_acc = tbase + ab * BN;
        if (!(ok = tc::mbar_wait(&acc_empty[ab], ((local / ACC) & 1) ^ 1, err, 204))) break;
        tc::fence_after_sync();
        for (int kt = 0; kt < nstages; ++kt, ++g) {
          const int s = g % STAGES;
          if (!(ok = tc::mbar_wait(&full[s], (g / STAGES) & 1, err, 202))) break;
          tc::fence_after_sync();
          const uint32_t st = tc::smem_u32(sm + s * STAGE_BYTES);
          const int steps = min(4, ksteps - 4 * kt);
          // descriptors built once per stage; their address fields advance in 16-byte units
          const uint64_t d_sfa = desc_sf_atom(st + C::SFA_OFF), d_sfb = desc_sf_atom(st + C::SFB_OFF),
                         d_a = tc::desc_kmajor_sw128(st + C::A_OFF), d_b = tc::desc_kmajor_sw128(st + C::B_OFF);
          constexpr uint32_t kA = kAtom >> 4, kH = 4 * kAtom >> 4;  // one atom; one B half (16-byte units)
          if (steps == 4) {  // every stage but a ragged last one: straight-line issue
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {   // K step kk: A -> columns 4kk .. 4kk + 3, B halves -> 8kk .. 8kk + 7
              tmem_cp_sf_atom(t_sfa + 4 * kk, d_sfa + kk * kA);
              tmem_cp_sf_atom(t_sfb + 8 * kk, d_sfb + kk * kA);
              tmem_cp_sf_atom(t_sfb + 8 * kk + 4, d_sfb + kH + kk * kA);
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_nvf4(t_acc, d_a + 2 * kk, d_b + 2 * kk, idesc, t_sfa + 4 * kk, t_sfb + 8 * kk, kt > 0 || kk > 0);
          } else {
            for (int kk = 0; kk < steps; ++kk) {
              tmem_cp_sf_atom(t_sfa + 4 * kk, d_sfa + kk * kA);
              tmem_cp_sf_atom(t_sfb + 8 * kk, d_sfb + kk * kA);
              tmem_cp_sf_atom(t_sfb + 8 * kk + 4, d_sfb + kH + kk * kA);
            }
            for (int kk = 0; kk < steps; ++kk)
              mma_nvf4(t_acc, d_a + 2 * kk, d_b + 2 * kk, idesc, t_sfa + 4 * kk, t_sfb + 8 * kk, kt > 0 || kk > 0);
          }
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&acc_full[ab]);
      }
    }
  } else {  // ---------------- epilogue: warps 2..9 ----------------
    // warp w reads TMEM lanes 32 (w % 4) .. + 31 (its sub-partition) and half (w - 2) / 4 of the
    // columns into registers, hands the accumulator back at once, then scales and stores, so the
    // stores overlap the next tile's main loop
    const int q = w & 3, half = (w - 2) >> 2;
    constexpr int HC = BN / 2;
    const float scale = ga[0] * gb[0];
    int local = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++local) {
      const int tm = t / ntn, tn = t % ntn;
      const int ab = local % ACC;
      const uint32_t lane_addr = tbase + (uint32_t(32 * q) << 16) + ab * BN + half * HC;
      // a timed-out wait is recorded in err; the warp still walks every tile (with garbage) so that
      // all 8 epilogue warps meet the same named barriers, each after bounded waits only
      const bool live = tc::mbar_wait(&acc_full[ab], (local / ACC) & 1, err, 203);
      tc::fence_after_sync();
      uint32_t r[HC / 32][32];
#pragma unroll
      for (int c = 0; c < HC / 32; ++c) tmem_ld32_raw(lane_addr + 32 * c, r[c]);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      tc::fence_before_sync();
      __syncwarp();
      if (l == 0) mbar_arrive(&acc_empty[ab]);
      __nv_bfloat16* lb = reinterpret_cast<__nv_bfloat16*>(sm + STAGES * STAGE_BYTES);
      if constexpr (kLora) {  // the tile's B rows, zero-padded to 16 values -> shared memory (named barrier 1)
        asm volatile("bar.sync 1, 256;" ::: "memory");  // the previous tile's readers are done
        for (int e = tid - 64; e < BN * 2; e += 256) {
          const int rr = e >> 1, cc = e & 1, n = tn * BN + rr;
          uint4 v4 = make_uint4(0, 0, 0, 0);
          if (n < N && 8 * cc < lora.r) v4 = __ldg(reinterpret_cast<const uint4*>(lora.b + size_t(n) * lora.r) + cc);
          reinterpret_cast<uint4*>(lb)[e] = v4;
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
      const int row = tm * BM + 32 * q + l;
      if (!live || row >= M) continue;
      float hf[16];  // this row's h (LoRA), zero past r
      if constexpr (kLora) {
        unpack8(__ldg(reinterpret_cast<const uint4*>(lora.h + size_t(row) * lora.ldh)), hf);
        if (lora.r > 8) {
          unpack8(__ldg(reinterpret_cast<const uint4*>(lora.h + size_t(row) * lora.ldh + 8)), hf + 8);
        } else {
#pragma unroll
          for (int i = 8; i < 16; ++i) hf[i] = 0.f;
        }
      }
#pragma unroll
      for (int c = 0; c < HC / 32; ++c) {
        const int col0 = tn * BN + half * HC + 32 * c;
        if (col0 >= N) break;
        // r[c][j] <- the output value (fp32 bits)
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          float v = __uint_as_float(r[c][jj]) * scale;
          if constexpr (kLora) {  // every lane reads the same B row: shared-memory broadcast
            const uint4* bp = reinterpret_cast<const uint4*>(lb + (half * HC + 32 * c + jj) * 16);
            float bf[8];
            unpack8(bp[0], bf);
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) d = fmaf(hf[i], bf[i], d);
            unpack8(bp[1], bf);
#pragma unroll
            for (int i = 0; i < 8; ++i) d = fmaf(hf[8 + i], bf[i], d);
            if (!out_bf16) v = fmaf(lora.s, d, v);
            else if (lora.mode == 0) v = bf16r(v) + bf16r(lora.s * d);  // addmm as cuBLAS rounds it
            else v = bf16r(v) + bf16r(bf16r(d) * lora.s);
          }
          r[c][jj] = __float_as_uint(v);
        }
        if (out_bf16) {
          __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + size_t(row) * N + col0;
          if (col0 + 32 <= N && (N % 8) == 0) {
#pragma unroll
            for (int jj = 0; jj < 32; jj += 8) {
              const uint4 pk = make_uint4(
                  tc::pack_bf16(__uint_as_float(r[c][jj]), __uint_as_float(r[c][jj + 1])),
                  tc::pack_bf16(__uint_as_float(r[c][jj + 2]), __uint_as_float(r[c][jj + 3])),
                  tc::pack_bf16(__uint_as_float(r[c][jj + 4]), __uint_as_float(r[c][jj + 5])),
                  tc::pack_bf16(__uint_as_float(r[c][jj + 6]), __uint_as_float(r[c][jj + 7])));
              *reinterpret_cast<uint4*>(o + jj) = pk;
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              if (col0 + jj < N) o[jj] = __float2bfloat16_rn(__uint_as_float(r[c][jj]));
          }
        } else {
          float* o = static_cast<float*>(out) + size_t(row) * N + col0;
          if (col0 + 32 <= N && (N % 4) == 0) {
#pragma unroll
            for (int jj = 0; jj < 32; jj += 4)
              *reinterpret_cast<float4*>(o + jj) = make_float4(__uint_as_float(r[c][jj]), __uint_as_float(r[c][jj + 1]),
                                                               __uint_as_float(r[c][jj + 2]), __uint_as_float(r[c][jj + 3]));
          } else {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              if (col0 + jj < N) o[jj] = __uint_as_float(r[c][jj]);
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (w == 1) tc::tmem_dealloc(tbase, 512);
}

// ------------------------------------------------------------------------------------------------
// SM-pair variant (cta_group::2): a cluster of two CTAs computes one 256 x 256 output tile. Each CTA
// holds its own 128 rows of A and its own 128-row half of B in shared memory; the pair's MMA
// (M = 256, N = 256, K = 64), issued by the even CTA, reads both CTAs' operands and writes each CTA's
// 128 accumulator rows (all 256 columns) into that CTA's tensor memory. A CTA thus reads only half of
// B from L2 where a one-SM 128 x 256 tile reads all of it: 8 KB instead of 12 KB of codes per 128 x
// 256 x 64 MMA step, and L2 -> SM traffic is what bounds the one-SM kernel at large shapes.
//   both CTAs, warp 0: TMA of the CTA's A rows, B half and scale atoms (A: its own row block; B: both
//     128-row halves, since each CTA's accumulator spans all 256 columns); the .cta_group::2 loads
//     count their bytes on the even CTA's `full` barrier (plain loads, no multicast);
//   even CTA, warp 10: per K step three atom copies into both CTAs' tensor memory
//     (tcgen05.cp.cta_group::2), into one of NSF scale sets in turn, handed to the MMA thread
//     through `sf_full` / `sf_free` (issued from one thread, copies and MMAs run one after the
//     other; from two threads the copies of later stages overlap the MMAs);
//   even CTA, warp 1: one pair MMA per K step; commits arrive on both CTAs' `empty`, `acc_full`;
//   both CTAs, warps 2-9: the epilogue of the CTA's 128 rows; each warp releases the accumulator by
//     an arrival on the even CTA's `acc_empty` (8 warps x 2 CTAs).
// The scale atoms are read through 3-D tensor maps over the blocked layout, [row block][K step][128
// u32]: a stage's 4 K steps of one row block are one box, and K steps or row blocks past the end
// read as zero.
namespace pair {
constexpr int ROWS = 128;                                   // rows of A and of B per CTA
constexpr int STAGES = 5;
constexpr int A_BYTES = ROWS * BKB, B_BYTES = ROWS * BKB;
constexpr int SFA_OFF = 0, SFB_OFF = 4 * kAtom, A_OFF = SFB_OFF + 8 * kAtom, B_OFF = A_OFF + A_BYTES;
constexpr int STAGE_BYTES = B_OFF + B_BYTES;                // 38 KB
constexpr int STAGE_TX = A_BYTES + B_BYTES + 12 * kAtom;    // bytes one CTA loads per stage
constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
constexpr int NSF = 4;         // scale sets in tensor memory (stage g uses set g % NSF)
constexpr int SF_COL0 = 256;  // TMEM: accumulator 0-255, scale sets of 48 columns from 256
static_assert(SF_COL0 + NSF * 48 <= 512, "TMEM budget");
constexpr int THREADS = kThreads + 32;                      // + warp 10: the scale-copy issuer
static_assert(A_OFF % 1024 == 0 && B_OFF % 1024 == 0 && STAGE_BYTES % 1024 == 0, "SW128 alignment");
static_assert(SMEM <= 227 * 1024, "shared memory");
}  // namespace pair

__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the shared::cluster address of the variable at local shared address `saddr` in CTA `rank`
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
// every thread of both CTAs
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(smem_dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
// tile of this CTA's rows into its own shared memory; the bytes are counted on `bar`, a
// shared::cluster address (the even CTA's barrier)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_cp_sf_atom_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void mma_nvf4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t sfa_tmem, uint32_t sfb_tmem, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1 : 0), "r"(sfa_tmem), "r"(sfb_tmem));
}
// arrives on `bar` (same shared offset) in both CTAs of the pair once the issuing thread's earlier
// pair MMAs and copies have completed
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          tc::smem_u32(bar)),
      "h"(uint16_t(3))
      : "memory");
}
// arrives on `bar` in this CTA only
__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(tc::smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// scales 32 accumulator values (fp32 bits) and stores them to out[row][col0 ...], columns < N
__device__ __forceinline__ void store_out32(uint32_t (&r)[32], float scale, void* out, int out_bf16, int row, int col0,
                                            int N) {
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) r[jj] = __float_as_uint(__uint_as_float(r[jj]) * scale);
  if (out_bf16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + size_t(row) * N + col0;
    if (col0 + 32 <= N && (N % 8) == 0) {
#pragma unroll
      for (int jj = 0; jj < 32; jj += 8)
        *reinterpret_cast<uint4*>(o + jj) = make_uint4(
            tc::pack_bf16(__uint_as_float(r[jj]), __uint_as_float(r[jj + 1])),
            tc::pack_bf16(__uint_as_float(r[jj + 2]), __uint_as_float(r[jj + 3])),
            tc::pack_bf16(__uint_as_float(r[jj + 4]), __uint_as_float(r[jj + 5])),
            tc::pack_bf16(__uint_as_float(r[jj + 6]), __uint_as_float(r[jj + 7])));
    } else {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        if (col0 + jj < N) o[jj] = __float2bfloat16_rn(__uint_as_float(r[jj]));
    }
  } else {
    float* o = static_cast<float*>(out) + size_t(row) * N + col0;
    if (col0 + 32 <= N && (N % 4) == 0) {
#pragma unroll
      for (int jj = 0; jj < 32; jj += 4)
        *reinterpret_cast<float4*>(o + jj) = make_float4(__uint_as_float(r[jj]), __uint_as_float(r[jj + 1]),
                                                         __uint_as_float(r[jj + 2]), __uint_as_float(r[jj + 3]));
    } else {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        if (col0 + jj < N) o[jj] = __uint_as_float(r[jj]);
    }
  }
}

// Persistent: cluster c (CTAs 2c, 2c + 1) handles 256 x 256 tiles c, c + clusters, ... (row-major
// over the tile grid). Every wait is bounded; a timed-out wait records its code in *err.
__global__ void __launch_bounds__(pair::THREADS, 1)
nvfp4_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_sfa, const __grid_constant__ CUtensorMap map_sfb,
                       const float* __restrict__ ga, const float* __restrict__ gb, int M, int N, int K,
                       void* __restrict__ out, int out_bf16, int* __restrict__ err) {
  using namespace pair;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t full[STAGES], empty[STAGES], acc_full, acc_empty, drain, sf_full[NSF], sf_free[NSF], cp_drain;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const uint32_t rank = cta_rank_in_cluster();
  const int cluster = int(blockIdx.x >> 1), nclusters = int(gridDim.x >> 1);
  const int ksteps = K / 64, nstages = (ksteps + 3) / 4;
  const int ntn = (N + 255) / 256, ntiles = ((M + 255) / 256) * ntn;

  if (w == 1) {  // the same warp in both CTAs: the pair's allocation covers both tensor memories
    tmem_alloc_pair(&tmem_base, 512);
    tmem_relinquish_pair();
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(&acc_full, 1);
    tc::mbar_init(&acc_empty, 16);
    tc::mbar_init(&drain, 1);
    for (int b = 0; b < NSF; ++b) {
      tc::mbar_init(&sf_full[b], 1);
      tc::mbar_init(&sf_free[b], 1);
    }
    tc::mbar_init(&cp_drain, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised before any load or arrival can reach them
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;

  if (w == 0) {
    if (l == 0) {  // ---------------- producer (both CTAs) ----------------
      int g = 0;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters) {
        const int tm = t / ntn, tn = t % ntn;
        for (int kt = 0; kt < nstages; ++kt, ++g) {
          const int s = g % STAGES;
          if (!(ok = tc::mbar_wait(&empty[s], ((g / STAGES) & 1) ^ 1, err, 211))) break;
          const uint32_t st = tc::smem_u32(sm + s * STAGE_BYTES), fb = cluster_addr(tc::smem_u32(&full[s]), 0);
          if (rank == 0) tc::mbar_expect_tx(&full[s], 2 * STAGE_TX);  // both CTAs' bytes
          tma_load_2d_pair(st + A_OFF, &map_a, kt * BKB, tm * 256 + ROWS * int(rank), fb);
          tma_load_2d_pair(st + B_OFF, &map_b, kt * BKB, tn * 256 + ROWS * int(rank), fb);
          tma_load_3d_pair(st + SFA_OFF, &map_sfa, 0, 4 * kt, 2 * tm + int(rank), fb);
          tma_load_3d_pair(st + SFB_OFF, &map_sfb, 0, 4 * kt, 2 * tn, fb);
          tma_load_3d_pair(st + SFB_OFF + 4 * kAtom, &map_sfb, 0, 4 * kt, 2 * tn + 1, fb);
        }
      }
    }
  } else if (w == 1) {
    if (l == 0 && rank == 0) {  // ---------------- MMA issuer (even CTA) ----------------
      constexpr uint32_t idesc = idesc_nvf4(256, 256);
      int g = 0, local = 0;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters, ++local) {
        if (!(ok = tc::mbar_wait(&acc_empty, (local & 1) ^ 1, err, 214))) break;
        tc::fence_after_sync();
        for (int kt = 0; kt < nstages; ++kt, ++g) {
          const int s = g % STAGES, b = g % NSF;
          if (!(ok = tc::mbar_wait(&full[s], (g / STAGES) & 1, err, 212))) break;
          if (!(ok = tc::mbar_wait(&sf_full[b], (g / NSF) & 1, err, 216))) break;  // the stage's scales are in TMEM
          tc::fence_after_sync();
          const uint32_t st = tc::smem_u32(sm + s * STAGE_BYTES);
          const int steps = min(4, ksteps - 4 * kt);
          const uint32_t t_sfa = tbase + SF_COL0 + b * 48, t_sfb = t_sfa + 16;
          const uint64_t d_a = tc::desc_kmajor_sw128(st + A_OFF), d_b = tc::desc_kmajor_sw128(st + B_OFF);
          for (int kk = 0; kk < steps; ++kk)
            mma_nvf4_pair(tbase, d_a + 2 * kk, d_b + 2 * kk, idesc, t_sfa + 4 * kk, t_sfb + 8 * kk, kt > 0 || kk > 0);
          mma_commit_pair(&empty[s]);
          mma_commit_pair_local(&sf_free[b]);  // the scale set may be overwritten once these MMAs are done
        }
        mma_commit_pair(&acc_full);
      }
      mma_commit_pair(&drain);  // completes once every MMA issued above has
    }
  } else if (w == 10) {
    if (l == 0 && rank == 0) {  // ---------------- scale-copy issuer (even CTA) ----------------
      // copies a stage's scale atoms into scale set g % NSF of both CTAs' tensor memory, up to NSF - 1
      // stages ahead of the MMAs
      int g = 0;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters) {
        for (int kt = 0; kt < nstages; ++kt, ++g) {
          const int s = g % STAGES, b = g % NSF;
          if (!(ok = tc::mbar_wait(&full[s], (g / STAGES) & 1, err, 217))) break;
          if (!(ok = tc::mbar_wait(&sf_free[b], ((g / NSF) & 1) ^ 1, err, 218))) break;
          tc::fence_after_sync();
          const uint32_t st = tc::smem_u32(sm + s * STAGE_BYTES);
          const int steps = min(4, ksteps - 4 * kt);
          const uint32_t t_sfa = tbase + SF_COL0 + b * 48, t_sfb = t_sfa + 16;
          const uint64_t d_sfa = desc_sf_atom(st + SFA_OFF), d_sfb = desc_sf_atom(st + SFB_OFF);
          constexpr uint32_t kA = kAtom >> 4, kH = 4 * kAtom >> 4;  // one atom; one B half (16-byte units)
          for (int kk = 0; kk < steps; ++kk) {  // K step kk: A -> columns 4kk .. 4kk + 3, B halves -> 8kk .. 8kk + 7
            tmem_cp_sf_atom_pair(t_sfa + 4 * kk, d_sfa + kk * kA);
            tmem_cp_sf_atom_pair(t_sfb + 8 * kk, d_sfb + kk * kA);
            tmem_cp_sf_atom_pair(t_sfb + 8 * kk + 4, d_sfb + kH + kk * kA);
          }
          mma_commit_pair_local(&sf_full[b]);
        }
      }
      mma_commit_pair_local(&cp_drain);
      tc::mbar_wait(&cp_drain, 0, err, 219);  // no copy of this thread is still in flight
    }
  } else {  // ---------------- epilogue: warps 2..9 of both CTAs ----------------
    static_assert(pair::THREADS == 11 * 32, "warps 0, 1 and 10 are handled above");
    const int q = w & 3, half = (w - 2) >> 2;
    const float scale = ga[0] * gb[0];
    const uint32_t ae = cluster_addr(tc::smem_u32(&acc_empty), 0);
    int local = 0;
    for (int t = cluster; t < ntiles; t += nclusters, ++local) {
      const int tm = t / ntn, tn = t % ntn;
      const uint32_t lane_addr = tbase + (uint32_t(32 * q) << 16) + half * 128;
      if (!tc::mbar_wait(&acc_full, local & 1, err, 213)) break;  // (no named barriers: leaving is safe)
      tc::fence_after_sync();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_raw(lane_addr + 32 * c, r[c]);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      tc::fence_before_sync();
      __syncwarp();
      if (l == 0) mbar_arrive_cluster(ae);
      const int row = tm * 256 + ROWS * int(rank) + 32 * q + l;
      if (row >= M) continue;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int col0 = tn * 256 + half * 128 + 32 * c;
        if (col0 >= N) break;
        store_out32(r[c], scale, out, out_bf16, row, col0, N);
      }
    }
  }
  if (w == 1 && l == 0) tc::mbar_wait(&drain, 0, err, 215);  // the pair's MMAs no longer touch either CTA
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the other may still signal its barriers
  tc::fence_after_sync();
  if (w == 1) tmem_dealloc_pair(tbase, 512);
}

// 2-D byte tensor [rows][cols_bytes], box [box_rows][128 bytes], 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols_bytes, int box_rows) {
  auto fn = tmap_encoder();
  if (!fn) {
    set_error("nvfp4_gemm: cuTensorMapEncodeTiled unavailable");
    return RB2_ECUDA;
  }
  cuuint64_t dims[2] = {cuuint64_t(cols_bytes), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols_bytes)};
  cuuint32_t box[2] = {128u, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("nvfp4_gemm: cuTensorMapEncodeTiled failed (%d)", int(r));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

// The blocked scales of `rows` rows as a 3-D u32 tensor [row block][K step][128] (one 512-byte atom
// per (row block, K step)), box [1][4][128]: the four K steps of one row block that a stage uses.
int make_map_sf(CUtensorMap* map, const void* base, int64_t rows, int64_t K) {
  auto fn = tmap_encoder();
  if (!fn) {
    set_error("nvfp4_gemm: cuTensorMapEncodeTiled unavailable");
    return RB2_ECUDA;
  }
  const int64_t nrb = (rows + 127) / 128, ks = K / 64;
  cuuint64_t dims[3] = {128u, cuuint64_t(ks), cuuint64_t(nrb)};
  cuuint64_t strides[2] = {cuuint64_t(kAtom), cuuint64_t(ks) * kAtom};
  cuuint32_t box[3] = {128u, 4u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("nvfp4_gemm: cuTensorMapEncodeTiled (scales) failed (%d)", int(r));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

// How many two-CTA clusters of the pair kernel can be resident at once on device `dev` (queried
// once per device; 0 if the query fails, in which case the one-SM kernel is used).
int pair_clusters(int dev) {
  static std::atomic<int> cache[64];  // value + 1; 0 = not yet queried (concurrent first calls agree)
  if (dev < 0 || dev >= 64) return 0;
  const int known = cache[dev].load(std::memory_order_relaxed);
  if (known > 0) return known - 1;
  int n = 0;
  bool failed = true;
  if (cudaFuncSetAttribute(nvfp4_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pair::SMEM) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(pair::THREADS);
    cfg.dynamicSmemBytes = pair::SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    failed = cudaOccupancyMaxActiveClusters(&n, nvfp4_gemm_pair_kernel, &cfg) != cudaSuccess;
  }
  if (failed) {
    n = 0;
    cudaGetLastError();  // the failed query's error is not left for the next launch check
  }
  cache[dev].store(n + 1, std::memory_order_relaxed);
  return n;
}

}  // namespace
}  // namespace rb2

using namespace rb2;

namespace {
// the blocked scale layout: [row block of 128][K step of 64][512-byte atom]
int64_t blocked_bytes(int64_t rows, int64_t K) { return (rows + 127) / 128 * (K / 64) * kAtom; }
}  // namespace

// workspace: the kernel's status word (the scales are read in place)
extern "C" size_t rb2_nvfp4_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  (void)M; (void)N; (void)K;
  return 1024;
}

extern "C" int rb2_nvfp4_gemm_ex(const uint8_t* a_codes, const uint8_t* a_scales_blocked, const float* a_gscale,
                                 const uint8_t* b_codes, const uint8_t* b_scales_blocked, const float* b_gscale,
                                 const uint8_t* b_images, const void* lora_h, int64_t lora_ldh, const void* lora_b,
                                 int lora_r, float lora_scale, int lora_mode, int64_t M, int64_t N, int64_t K, void* out,
                                 int out_dtype, void* ws, size_t ws_bytes, void* stream) {
  RB2_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % 64 == 0, "nvfp4_gemm: need M, N > 0 and K %% 64 == 0 (K=%lld)",
                (long long)K);
  RB2_CHECK_ARG(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31), "nvfp4_gemm: size");
  RB2_CHECK_ARG(a_codes && b_codes && a_scales_blocked && b_scales_blocked && a_gscale && b_gscale && out && ws,
                "nvfp4_gemm: null pointer");
  RB2_CHECK_ARG(out_dtype == RB2_F32 || out_dtype == RB2_BF16, "nvfp4_gemm: out_dtype");
  RB2_CHECK_ARG((reinterpret_cast<uintptr_t>(a_codes) & 15) == 0 && (reinterpret_cast<uintptr_t>(b_codes) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(a_scales_blocked) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(b_scales_blocked) & 15) == 0,
                "nvfp4_gemm: operands must be 16-byte aligned");
  if (ws_bytes < rb2_nvfp4_gemm_workspace_size(M, N, K)) {
    set_error("nvfp4_gemm: workspace too small");
    return RB2_EWORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap ma, mb;
  int rc;
  using Wide = GemmCfg<256, 4, 1>;
  const int BN = Wide::BN;
  if ((rc = make_map(&ma, a_codes, M, K / 2, BM))) return rc;
  if ((rc = make_map(&mb, b_codes, N, K / 2, BN))) return rc;
  RB2_CUDA(cudaMemsetAsync(ws, 0, sizeof(int), s), "nvfp4_gemm: clear status");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  dim3 grid(unsigned(ntiles < sms ? ntiles : sms));
  // B's precomputed scales (rb2_nvfp4_gemm_b_images) are its blocked scales, read in place like A's
  const uint8_t* sfb = b_images ? b_images : b_scales_blocked;
  RB2_CHECK_ARG((reinterpret_cast<uintptr_t>(b_images) & 15) == 0, "nvfp4_gemm: b_images must be 16-byte aligned");
  RB2_CHECK_ARG(lora_h == nullptr ||
                    (lora_b && lora_r > 0 && lora_r <= 16 && lora_r % 8 == 0 && lora_ldh >= lora_r && lora_ldh % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(lora_h) & 15) == 0 && (reinterpret_cast<uintptr_t>(lora_b) & 15) == 0),
                "nvfp4_gemm: LoRA needs r in {8, 16}, a row stride that is a multiple of 8 and 16-byte aligned h, B");
  RB2_CHECK_ARG(lora_mode == 0 || lora_mode == 1, "nvfp4_gemm: lora_mode must be 0 or 1");
  const Lora lora{static_cast<const __nv_bfloat16*>(lora_h), static_cast<const __nv_bfloat16*>(lora_b), lora_ldh,
                  lora_r, lora_scale, lora_mode};
  {
    ProfScope ps_("nvfp4_gemm", s);
    if (lora.h) {
      RB2_CUDA(cudaFuncSetAttribute(nvfp4_gemm_kernel<Wide, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Wide::SMEM + Wide::LORA_BYTES),
               "nvfp4_gemm: smem attribute");
      nvfp4_gemm_kernel<Wide, true><<<grid, kThreads, Wide::SMEM + Wide::LORA_BYTES, s>>>(
          ma, mb, a_scales_blocked, sfb, int((N + 127) / 128), a_gscale, b_gscale, int(M), int(N), int(K), out,
          out_dtype == RB2_BF16, lora,
          static_cast<int*>(ws));
    } else {
      RB2_CUDA(cudaFuncSetAttribute(nvfp4_gemm_kernel<Wide, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Wide::SMEM),
               "nvfp4_gemm: smem attribute");
      nvfp4_gemm_kernel<Wide, false><<<grid, kThreads, Wide::SMEM, s>>>(
          ma, mb, a_scales_blocked, sfb, int((N + 127) / 128), a_gscale, b_gscale, int(M), int(N), int(K), out,
          out_dtype == RB2_BF16, lora,
          static_cast<int*>(ws));
    }
  }
  RB2_CHECK_LAUNCH("nvfp4_gemm");
  return RB2_OK;
}

extern "C" int rb2_nvfp4_gemm(const uint8_t* a_codes, const uint8_t* a_scales_blocked, const float* a_gscale,
                              const uint8_t* b_codes, const uint8_t* b_scales_blocked, const float* b_gscale,
                              int64_t M, int64_t N, int64_t K, void* out, int out_dtype, void* ws, size_t ws_bytes,
                              void* stream) {
  return rb2_nvfp4_gemm_ex(a_codes, a_scales_blocked, a_gscale, b_codes, b_scales_blocked, b_gscale, nullptr, nullptr,
                           0, nullptr, 0, 0.f, 0, M, N, K, out, out_dtype, ws, ws_bytes, stream);
}

// The same product on SM pairs (cta_group::2, 256 x 256 tiles). Correct at every shape the one-SM
// kernel takes, but slower at the shapes measured (16384 x 12288 x 4096: 0.56 ms against 0.46 ms):
// per SM it moves the same tensor-memory scale copies as the one-SM kernel, and its pair MMA and
// copies each take longer per SM than their one-SM counterparts.
extern "C" int rb2_nvfp4_gemm_pair(const uint8_t* a_codes, const uint8_t* a_scales_blocked, const float* a_gscale,
                                   const uint8_t* b_codes, const uint8_t* b_scales_blocked, const float* b_gscale,
                                   int64_t M, int64_t N, int64_t K, void* out, int out_dtype, void* ws, size_t ws_bytes,
                                   void* stream) {
  RB2_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % 64 == 0, "nvfp4_gemm_pair: need M, N > 0 and K %% 64 == 0 (K=%lld)",
                (long long)K);
  RB2_CHECK_ARG(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31), "nvfp4_gemm_pair: size");
  RB2_CHECK_ARG(a_codes && b_codes && a_scales_blocked && b_scales_blocked && a_gscale && b_gscale && out && ws,
                "nvfp4_gemm_pair: null pointer");
  RB2_CHECK_ARG(out_dtype == RB2_F32 || out_dtype == RB2_BF16, "nvfp4_gemm_pair: out_dtype");
  RB2_CHECK_ARG((reinterpret_cast<uintptr_t>(a_codes) & 15) == 0 && (reinterpret_cast<uintptr_t>(b_codes) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(a_scales_blocked) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(b_scales_blocked) & 15) == 0,
                "nvfp4_gemm_pair: operands must be 16-byte aligned");
  if (ws_bytes < rb2_nvfp4_gemm_workspace_size(M, N, K)) {
    set_error("nvfp4_gemm_pair: workspace too small");
    return RB2_EWORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0;
  cudaGetDevice(&dev);
  const int clusters = pair_clusters(dev);
  if (clusters <= 0) {
    set_error("nvfp4_gemm_pair: no two-CTA cluster of this kernel fits on the device");
    return RB2_ECUDA;
  }
  int rc;
  CUtensorMap pa, pb, psa, psb;
  if ((rc = make_map(&pa, a_codes, M, K / 2, pair::ROWS)) || (rc = make_map(&pb, b_codes, N, K / 2, pair::ROWS)) ||
      (rc = make_map_sf(&psa, a_scales_blocked, M, K)) || (rc = make_map_sf(&psb, b_scales_blocked, N, K)))
    return rc;
  RB2_CUDA(cudaMemsetAsync(ws, 0, sizeof(int), s), "nvfp4_gemm_pair: clear status");
  const int64_t ptiles = ((M + 255) / 256) * ((N + 255) / 256);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(2 * (ptiles < clusters ? ptiles : clusters)));
  cfg.blockDim = dim3(pair::THREADS);
  cfg.dynamicSmemBytes = pair::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  {
    ProfScope ps_("nvfp4_gemm_pair", s);
    RB2_CUDA(cudaLaunchKernelEx(&cfg, nvfp4_gemm_pair_kernel, pa, pb, psa, psb, a_gscale, b_gscale, int(M), int(N),
                                int(K), out, int(out_dtype == RB2_BF16), static_cast<int*>(ws)),
             "nvfp4_gemm_pair: launch");
  }
  RB2_CHECK_LAUNCH("nvfp4_gemm_pair");
  return RB2_OK;
}

extern "C" size_t rb2_nvfp4_gemm_b_images_size(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0) return 0;
  return size_t(blocked_bytes(N, K));
}

// The B operand's scales as the kernel reads them, kept with a frozen weight: the kernel reads the
// blocked layout in place, so this is a copy of the blocked scales (kept for callers that cache it).
extern "C" int rb2_nvfp4_gemm_b_images(const uint8_t* b_scales_blocked, int64_t N, int64_t K, void* out,
                                       size_t out_bytes, void* stream) {
  RB2_CHECK_ARG(N > 0 && K > 0 && K % 64 == 0 && N < (int64_t(1) << 31) && K < (int64_t(1) << 31),
                "nvfp4_gemm_b_images: need N > 0 and K %% 64 == 0");
  RB2_CHECK_ARG(b_scales_blocked && out && (reinterpret_cast<uintptr_t>(b_scales_blocked) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                "nvfp4_gemm_b_images: null or misaligned pointer");
  const size_t nb = size_t(blocked_bytes(N, K));
  if (out_bytes < nb) {
    set_error("nvfp4_gemm_b_images: output too small");
    return RB2_EWORKSPACE;
  }
  RB2_CUDA(cudaMemcpyAsync(out, b_scales_blocked, nb, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)),
           "nvfp4_gemm_b_images: copy");
  return RB2_OK;
}
