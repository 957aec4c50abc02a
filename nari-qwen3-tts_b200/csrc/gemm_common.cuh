// Helpers shared by the weight-streaming GEMMs (gemm.cu: bf16, gemm_fp8.cu:
// FP8 block-scaled): contiguous bulk copies, the 3-D X tensor load, thread-
// block cluster barriers and distributed shared memory, the SwiGLU epilogue
// and the driver's tensor-map encoder.
#pragma once

#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace nqt {
namespace gemm_detail {

// Contiguous global -> shared copy completing on an mbarrier (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// X slabs [slab, slab + group) of the 3-D view {k in slab, rows, slabs}, rows from `row0` (one copy per stage)
__device__ __forceinline__ void tma_load_x(void* dst, const CUtensorMap* map, uint64_t* bar, int row0, int slab) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(0), "r"(row0), "r"(slab)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Cluster barrier, split: every thread of every CTA arrives once, then waits once (release / acquire at
// cluster scope), alternating.  Whole converged warps only (.aligned): call sites reconverge first.
__device__ __forceinline__ void cluster_arrive() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  __syncwarp();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Contiguous copy from this CTA's shared memory into a peer's, completing `bar_cluster_addr`'s
// transaction count there (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster_addr, const void* src, uint32_t bytes,
                                                  uint32_t bar_cluster_addr) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster_addr),
               "r"(smem_addr(src)), "r"(bytes), "r"(bar_cluster_addr)
               : "memory");
}

// Named barrier of the four epilogue warps (warps 2-5).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// silu(g) * u with the fast (approximate, ~2 ulp) division: the result is rounded to bf16 right after
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.f + __expf(-g)) * u; }

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

inline PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// X [rows, K] (row pitch `ld_bytes`) viewed as {128 B of k, rows, K-slabs of 128 B} with box
// {128 B, box_rows, group}: one copy brings `group` K slabs, each [box_rows x 128 B] with the 128-byte
// swizzle, one after another.  `elem` is the element type (bf16: 64 per slab, uint8: 128 per slab).
inline int encode_x_slabs(CUtensorMap* map, CUtensorMapDataType elem, int elem_bytes, const void* base, int rows,
                          int64_t slabs, int64_t ld_bytes, int box_rows, int group) {
  auto encode = get_encode();
  if (encode == nullptr) return NQT_ERR_CUDA;
  const int per_slab = 128 / elem_bytes;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(per_slab), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(slabs)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld_bytes), 128};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(per_slab), static_cast<cuuint32_t>(box_rows),
                       static_cast<cuuint32_t>(group)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, elem, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NQT_OK : NQT_ERR_CUDA;
}

// Shared memory to request so that no SM holds more CTAs than TMEM columns for (512 / tmem_cols
// CTAs at most): a CTA blocked in tcgen05.alloc while its cluster peers wait at a cluster barrier
// would deadlock.  An SM has 228 KB; the runtime reserves 1 KB per CTA.
inline int tmem_smem_floor(int tmem_cols) {
  const int fit = 512 / tmem_cols;  // CTAs whose columns fit at once
  return 233472 / (fit + 1) - 1024 + 16;
}

}  // namespace gemm_detail
}  // namespace nqt
