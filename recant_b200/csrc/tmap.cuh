// TMA tensor maps (cp.async.bulk.tensor, no multicast) over the caller's token-major tensors.
//
// A [tokens][heads][128] bf16 tensor is described as a 3-D map with dims (128, heads, tokens) and a
// box of (64, 1, 64): one box is the 64 tokens x 64 columns of one head, landing as a 64-row,
// 128-byte-swizzled slab in shared memory, i.e. one half of a K-major SW128 operand tile. Rows past
// the end of the tensor are zero-filled by the TMA unit; rows past the end of a sequence inside the
// tensor are zeroed by the caller after the load.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "tc.cuh"

namespace rb2 {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// bf16 [tokens][heads][128]; base 16-byte aligned
inline int make_rows_map(CUtensorMap* map, const void* base, int64_t tokens, int heads) {
  auto fn = tmap_encoder();
  if (!fn) {
    set_error("gdn: cuTensorMapEncodeTiled unavailable");
    return RB2_ECUDA;
  }
  cuuint64_t dims[3] = {128u, cuuint64_t(heads), cuuint64_t(tokens > 0 ? tokens : 1)};
  cuuint64_t strides[2] = {cuuint64_t(128 * 2), cuuint64_t(heads) * 128 * 2};
  cuuint32_t box[3] = {64u, 1u, 64u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gdn: cuTensorMapEncodeTiled failed (%d)", int(r));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

namespace tc {
// One 64 x 64 box (columns x0 .. x0+63 of head `head`, tokens t0 .. t0+63) into a 1024-aligned slab.
// x0 is 0 or 64 (128-byte aligned innermost coordinate).
__device__ __forceinline__ void tma_rows(void* smem_dst, const CUtensorMap* map, int x0, int head, int t0,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(smem_dst)),
      "l"(map), "r"(x0), "r"(head), "r"(t0), "r"(smem_u32(bar))
      : "memory");
}
// 64 rows x 128 columns of one head into a SW128 tile whose slabs are `slab_bytes` apart, rows
// starting at `row0` (0 or 64): 16 KB on `bar`
__device__ __forceinline__ void tma_rows128(unsigned char* tile, int slab_bytes, int row0, const CUtensorMap* map,
                                            int head, int t0, uint64_t* bar) {
  tma_rows(tile + row0 * 128, map, 0, head, t0, bar);
  tma_rows(tile + slab_bytes + row0 * 128, map, 64, head, t0, bar);
}
// zero rows [L, 64) of such a 64-row block (whole 128-byte rows, so the swizzle does not matter)
__device__ __forceinline__ void zero_rows_tail(unsigned char* tile, int slab_bytes, int row0, int L, int nthr) {
  const int n = (64 - L) * 16;
  for (int idx = int(threadIdx.x); idx < n; idx += nthr) {
    const int rr = row0 + L + (idx >> 4), c = idx & 15;
    *reinterpret_cast<uint4*>(tile + (c >> 3) * slab_bytes + rr * 128 + (c & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
}
}  // namespace tc
}  // namespace rb2
