// Weight-streaming GEMM for the decoder projections (sm_100a, tcgen05 + TMA).
//
//   Y[M, N] = X[M, K] . W[N, K]^T        (nn.Linear: W row-major [out, in])
//
// M (tokens of the step: 64 talker rows, 256 code-predictor rows) is small and
// N x K (the weights) is large, so the kernel is a stream over W.  The MMA
// operands are swapped: a 128-row tile of W is the MMA's M, the whole token
// batch is the MMA's N (padded to 16 by the TMA zero fill), and the fp32
// accumulator D^T[128 x Mpad] lives in TMEM.
//
// W is packed once, at load time, into 16 KB units [N / 128][K / 64][128 rows
// x 128 B] stored contiguously and already in the 128-byte-swizzled order the
// MMA reads (16-byte chunk c of row r at chunk c ^ (r % 8)).  The units of all
// tiles form one array, and a persistent grid of one CTA per SM splits it into
// equal contiguous ranges (stream-K): every SM streams the same number of
// bytes with one bulk copy per stage, whatever N / 128 is.  A CTA's range
// covers pieces of one to a few tiles; a tile covered by one CTA is written
// directly, a tile shared by several is summed with fp32 reductions into a
// zeroed L2-resident workspace (16-byte reductions, token-contiguous rows),
// and the CTA that arrives last (a per-tile ticket) writes the output and
// zeroes its part of the workspace again.  X
// (the step's activations, L2-resident) comes through a 2-D tensor map (box
// 64 x Mpad, 128-byte swizzle).
//
// Warp roles (6 warps): 0 copy producer, 1 TMEM owner + MMA issuer (two TMEM
// accumulators, so the next tile piece accumulates while the epilogue drains
// the previous one), 2-5 the epilogue (warp w reads TMEM lanes 32 (w % 4) ..).
// Epilogues:
//   plain    Y = bf16(acc)
//   bias     Y = bf16(acc + bias)                       (nn.Linear with bias)
//   silu_mul W rows interleaved in 64-row blocks [gate 64 | up 64]; output
//            column f of block b is silu(g) * u of rows 128 b + f, 128 b + 64 + f,
//            with g and u rounded to bf16 first (the unfused gate_up GEMM
//            followed by silu_and_mul); Y is [M, N / 2].
// Every wait is bounded and reports NQT_DEV_TIMEOUT.  The kernel is launched
// with programmatic stream serialization: the W stages of the prologue are
// fetched before griddepcontrol.wait, everything that touches X, Y or the
// workspace after it.  The workspace is one per device, so calls on a device
// are ordered on one stream.
//
// Replaces the torch/cuBLAS projections of the decoder layers
// (model/layers.py:195-270, model/components.py:300-356) and the sm90-only
// fused gate/up path (executor/optimizations.py:22-47).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace nqt {
namespace {

constexpr int kTileN = 128;                    // W rows per tile (MMA M)
constexpr int kBlockK = 64;                    // K per unit (one 128-byte swizzle row)
constexpr int kThreads = 6 * 32;
constexpr int kWBytes = kTileN * kBlockK * 2;  // 16 KB per unit
constexpr int kXsBytes = 32 * kTileN * 2;      // epilogue staging: 32 tokens x 128 bf16
constexpr int kMaxWsFloats = 4 << 20;          // split-tile workspace, fp32 [N][round_up(M, 4)]
constexpr int kMaxTiles = 1024;

__device__ __align__(16) float g_ws[kMaxWsFloats];  // zero at load; each split tile's last CTA zeroes it again
__device__ int g_ws_ticket[kMaxTiles];  // CTAs done per split tile; reset by the last one

enum Epilogue : int { kPlain = 0, kBias = 1, kSiluMul = 2 };

struct GemmArgs {
  const uint8_t* wpack;
  __nv_bfloat16* y;
  int64_t ldy;
  const __nv_bfloat16* bias;
  int32_t* status;
  float* ws;
  int* ticket;
  int m, n, k;
  int mpad;  // MMA N: m rounded up to 16
  int epilogue;
  int stages;
  int kbt;      // K units per tile
  int units;    // tiles * kbt
  int vec_out;  // y rows 16-byte aligned: vector stores
  int ldws;     // workspace row pitch: m rounded up to 4
};

__host__ __device__ constexpr int x_bytes(int mpad) { return mpad * kBlockK * 2; }
__host__ __device__ constexpr int stage_bytes(int mpad) { return kWBytes + x_bytes(mpad); }

// Units [first_unit(c), first_unit(c + 1)) belong to CTA c of G.
__device__ __forceinline__ int first_unit(int c, int units, int G) {
  return static_cast<int>((static_cast<int64_t>(c) * units) / G);
}
// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of(int u, int units, int G) {
  return static_cast<int>(((static_cast<int64_t>(u) + 1) * G - 1) / units);
}

// Contiguous global -> shared copy completing on an mbarrier (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Writes rows [0, 32) of the staging buffer (32 tokens x `cols` bf16, row pitch 128) to Y[m0 + r][col0 ..].
__device__ __forceinline__ void store_staged(const GemmArgs& a, const __nv_bfloat16* xs, int m0, int col0, int cols,
                                             int et) {
  if (a.vec_out) {
    const int per_row = cols / 8;
    for (int i = et; i < 32 * per_row; i += 128) {
      const int r = i / per_row, ch = i % per_row;
      if (m0 + r < a.m) {
        *reinterpret_cast<uint4*>(a.y + static_cast<int64_t>(m0 + r) * a.ldy + col0 + ch * 8) =
            *reinterpret_cast<const uint4*>(xs + r * kTileN + ch * 8);
      }
    }
  } else {
    for (int i = et; i < 32 * cols; i += 128) {
      const int r = i / cols, c = i % cols;
      if (m0 + r < a.m) a.y[static_cast<int64_t>(m0 + r) * a.ldy + col0 + c] = xs[r * kTileN + c];
    }
  }
}

// A tile written by one CTA: TMEM -> bf16 (epilogue) -> staging -> Y.
__device__ void direct_epilogue(const GemmArgs& a, uint32_t t_row, int row, int tile, __nv_bfloat16* xs, int et) {
  const int n0 = tile * kTileN;
  const float bias = a.epilogue == kBias ? __bfloat162float(a.bias[n0 + row]) : 0.f;
  for (int c = 0; c < a.mpad && c < a.m; c += 32) {
    uint32_t r[32];
    tc::ld_32x32b_x32(t_row + c, r);
    tc::wait_ld();
    if (a.epilogue == kSiluMul) {
      // up rows (64..127) stage bf16(up); gate rows combine
      if (row >= 64) {
#pragma unroll
        for (int e = 0; e < 32; ++e) xs[e * kTileN + 64 + (row - 64)] = __float2bfloat16_rn(__uint_as_float(r[e]));
      }
      epi_bar();
      if (row < 64) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float g = bf16_round(__uint_as_float(r[e]));
          const float u = __bfloat162float(xs[e * kTileN + 64 + row]);
          xs[e * kTileN + row] = __float2bfloat16_rn(silu_mul(g, u));
        }
      }
      epi_bar();
      store_staged(a, xs, c, tile * 64, 64, et);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) xs[e * kTileN + row] = __float2bfloat16_rn(__uint_as_float(r[e]) + bias);
      epi_bar();
      store_staged(a, xs, c, n0, kTileN, et);
    }
    epi_bar();
  }
}

// The last CTA of a split tile: workspace -> epilogue -> Y, and the workspace
// back to zero.  Thread et owns workspace row n0 + et (its tokens contiguous);
// sixteen 16-byte loads are in flight before the first is used.
__device__ void finish_split_tile(const GemmArgs& a, int tile, int et) {
  const int n0 = tile * kTileN;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  if (a.epilogue == kSiluMul) {
    if (et >= 64) return;  // gate thread et also takes up row et + 64
    float* g = a.ws + static_cast<int64_t>(n0 + et) * a.ldws;
    float* u = g + 64 * static_cast<int64_t>(a.ldws);
    __nv_bfloat16* dst = a.y + tile * 64 + et;
    for (int c0 = 0; c0 < a.ldws; c0 += 32) {
      float4 gv[8], uv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (c0 + 4 * q < a.ldws) {
          gv[q] = __ldcg(reinterpret_cast<const float4*>(g + c0 + 4 * q));
          uv[q] = __ldcg(reinterpret_cast<const float4*>(u + c0 + 4 * q));
        }
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (c0 + 4 * q < a.ldws) {
          __stcg(reinterpret_cast<float4*>(g + c0 + 4 * q), zero);
          __stcg(reinterpret_cast<float4*>(u + c0 + 4 * q), zero);
          const float gg[4] = {gv[q].x, gv[q].y, gv[q].z, gv[q].w};
          const float uu[4] = {uv[q].x, uv[q].y, uv[q].z, uv[q].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = c0 + 4 * q + e;
            if (m < a.m)
              dst[static_cast<int64_t>(m) * a.ldy] = __float2bfloat16_rn(silu_mul(bf16_round(gg[e]), bf16_round(uu[e])));
          }
        }
      }
    }
  } else {
    float* src = a.ws + static_cast<int64_t>(n0 + et) * a.ldws;
    const float bias = a.epilogue == kBias ? __bfloat162float(a.bias[n0 + et]) : 0.f;
    __nv_bfloat16* dst = a.y + n0 + et;
    for (int c0 = 0; c0 < a.ldws; c0 += 64) {
      float4 v[16];
#pragma unroll
      for (int q = 0; q < 16; ++q)
        if (c0 + 4 * q < a.ldws) v[q] = __ldcg(reinterpret_cast<const float4*>(src + c0 + 4 * q));
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        if (c0 + 4 * q < a.ldws) {
          __stcg(reinterpret_cast<float4*>(src + c0 + 4 * q), zero);
          const float vv[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = c0 + 4 * q + e;
            if (m < a.m) dst[static_cast<int64_t>(m) * a.ldy] = __float2bfloat16_rn(vv[e] + bias);
          }
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap xmap, GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = a.stages;
  const int sb = stage_bytes(a.mpad);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + ST * sb);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * sb + kXsBytes);
  uint64_t* empty = full + ST;
  uint64_t* done = empty + ST;  // [2] accumulator b complete
  uint64_t* tfree = done + 2;   // [2] accumulator b drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfree + 2);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int u0 = first_unit(blockIdx.x, a.units, G);
  const int u1 = first_unit(blockIdx.x + 1, a.units, G);
  const int nu = u1 - u0;
  uint32_t tmem_cols = 32;
  while (tmem_cols < static_cast<uint32_t>(2 * a.mpad)) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&done[b], 1);
      mbar_init(&tfree[b], 4);
    }
    fence_barrier_init();
    // W does not depend on the previous kernel: start streaming it at once
    const int pro = nu < ST ? nu : ST;
    for (int j = 0; j < pro; ++j) {
      mbar_arrive_expect_tx(&full[j], sb);
      bulk_load(smem + j * sb, a.wpack + static_cast<int64_t>(u0 + j) * kWBytes, kWBytes, &full[j]);
    }
  }
  // barrier 2: the mbarrier initialisation (warp 0 arrives without waiting) and the TMEM address
  // (allocated by warp 1) reach warps 1-5; the producer never waits for the allocation
  if (warp == 0) {
    __syncwarp();
    asm volatile("bar.arrive 2, %0;" ::"n"(kThreads) : "memory");
  } else {
    if (warp == 1) {
      tc::tmem_alloc(tmem_slot, tmem_cols);
      tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory");
    tc::fence_after_sync();
  }
  const uint32_t tmem = warp == 0 ? 0u : *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0 && nu > 0) {
      prefetch_tensormap(&xmap);
      const int pro = nu < ST ? nu : ST;
      grid_dependency_wait();
      for (int j = 0; j < pro; ++j)
        tma_load_2d(smem + j * sb + kWBytes, &xmap, &full[j], ((u0 + j) % a.kbt) * kBlockK, 0);
      int issued = pro;
      for (int j = pro; j < nu; ++j) {
        const int s = j % ST;
        if (!mbar_wait(&empty[s], ((j / ST) - 1) & 1, a.status)) break;
        mbar_arrive_expect_tx(&full[s], sb);
        bulk_load(smem + s * sb, a.wpack + static_cast<int64_t>(u0 + j) * kWBytes, kWBytes, &full[s]);
        tma_load_2d(smem + s * sb + kWBytes, &xmap, &full[s], ((u0 + j) % a.kbt) * kBlockK, 0);
        issued = j + 1;
      }
      // every copy issued has landed before the CTA leaves (bounded)
      for (int j = issued > ST ? issued - ST : 0; j < issued; ++j) mbar_wait(&full[j % ST], (j / ST) & 1, a.status);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16_f32(kTileN, a.mpad, false, false);
      int j = 0, seg = 0;
      bool ok = true;
      for (int u = u0; u < u1 && ok; ++seg) {
        const int tile = u / a.kbt;
        const int seg_end = min(u1, (tile + 1) * a.kbt);
        const int b = seg & 1;
        if (seg >= 2 && !mbar_wait(&tfree[b], ((seg - 2) >> 1) & 1, a.status)) break;
        tc::fence_after_sync();
        const uint32_t acc = tmem + b * a.mpad;
        const int seg_begin = u;
        for (; u < seg_end; ++u, ++j) {
          const int s = j % ST;
          if (!mbar_wait(&full[s], (j / ST) & 1, a.status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t w_addr = smem_addr(smem + s * sb);
          const uint32_t x_addr = w_addr + kWBytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t da = tc::smem_desc_sw128(w_addr + kk * 32, 16, 1024);
            const uint64_t db = tc::smem_desc_sw128(x_addr + kk * 32, 16, 1024);
            tc::mma_f16_ss(acc, da, db, idesc, (u > seg_begin || kk > 0) ? 1u : 0u);
          }
          tc::commit(&empty[s]);
        }
        tc::commit(&done[b]);  // arrives once every MMA above has completed
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps
    grid_dependency_wait();
    const int et = threadIdx.x - 64;  // 0..127
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // tile row = TMEM lane
    int seg = 0;
    for (int u = u0; u < u1; ++seg) {
      const int tile = u / a.kbt;
      const int seg_end = min(u1, (tile + 1) * a.kbt);
      const int b = seg & 1;
      const bool done_ok = mbar_wait(&done[b], (seg >> 1) & 1, a.status);
      tc::fence_after_sync();
      const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * a.mpad;
      const int c_first = cta_of(tile * a.kbt, a.units, G);
      const int c_last = cta_of((tile + 1) * a.kbt - 1, a.units, G);
      if (c_first == c_last) {
        if (done_ok) direct_epilogue(a, t_row, row, tile, xs, et);
      } else {
        // partial sum of a shared tile: 16-byte fp32 reductions into workspace row n0 + row, then the ticket
        float* ws_row = a.ws + static_cast<int64_t>(tile * kTileN + row) * a.ldws;
        for (int c = 0; c < a.mpad && c < a.m; c += 32) {
          uint32_t r[32];
          tc::ld_32x32b_x32(t_row + c, r);
          tc::wait_ld();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (c + 4 * q < a.m && done_ok) {
              red_add_v4(ws_row + c + 4 * q, __uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                         __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
            }
          }
        }
        __threadfence();
        epi_bar();
        if (et == 0) {
          const int arrived = atomicAdd(&a.ticket[tile], 1);
          const bool last = arrived == c_last - c_first;
          if (last) a.ticket[tile] = 0;
          *s_last = last ? 1 : 0;
        }
        epi_bar();
        if (*s_last) {
          __threadfence();
          finish_split_tile(a, tile, et);
        }
        epi_bar();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[b]);
      u = seg_end;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, tmem_cols);
  }
}

// One 16-byte chunk per thread: chunk (tile, kb, r, c) of the packed layout.
__global__ void pack_kernel(const __nv_bfloat16* w, int64_t ldw, int n, int k, int interleave, __nv_bfloat16* out) {
  const int kbt = k / kBlockK;
  const int64_t total = static_cast<int64_t>(n / kTileN) * kbt * kTileN * 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i & 7);
    const int r = static_cast<int>((i >> 3) % kTileN);
    const int64_t tkb = (i >> 3) / kTileN;  // tile * kbt + kb
    const int kb = static_cast<int>(tkb % kbt);
    const int tile = static_cast<int>(tkb / kbt);
    int src_row = tile * kTileN + r;
    if (interleave) src_row = r < 64 ? tile * 64 + r : n / 2 + tile * 64 + (r - 64);
    const uint4 v = *reinterpret_cast<const uint4*>(w + src_row * ldw + kb * kBlockK + c * 8);
    *reinterpret_cast<uint4*>(out + (tkb * kTileN + r) * kBlockK + ((c ^ (r & 7)) * 8)) = v;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// 2-D K-major map of a row-major bf16 matrix [rows, cols] with leading dimension ld, box {64, box_rows}.
int encode_2d(CUtensorMap* map, const void* base, int rows, int cols, int64_t ld, int box_rows) {
  auto encode = get_encode();
  if (encode == nullptr) return NQT_ERR_CUDA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NQT_OK : NQT_ERR_CUDA;
}

int smem_bytes(int mpad, int stages) {
  return 1024 + stages * stage_bytes(mpad) + kXsBytes + (2 * stages + 4) * 8 + 16;
}

struct Workspace {
  float* ws = nullptr;
  int* ticket = nullptr;
};

// Per-device addresses of the static workspace (looked up once per device).
int workspace(Workspace* out) {
  static std::mutex mu;
  static Workspace cache[64];
  static bool have[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NQT_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (!have[dev]) {
    void* p = nullptr;
    void* q = nullptr;
    if (cudaGetSymbolAddress(&p, g_ws) != cudaSuccess || cudaGetSymbolAddress(&q, g_ws_ticket) != cudaSuccess) {
      set_last_message("gemm: workspace symbol lookup failed");
      return NQT_ERR_CUDA;
    }
    cache[dev].ws = static_cast<float*>(p);
    cache[dev].ticket = static_cast<int*>(q);
    have[dev] = true;
  }
  *out = cache[dev];
  return NQT_OK;
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_gemm_pack_weight(const void* w, int64_t ldw, int n, int k, int interleave_gate_up, void* packed,
                                    void* stream) {
  if (!w || !packed || n < kTileN || k < kBlockK || n % kTileN || k % kBlockK || ldw < k) return NQT_ERR_ARG;
  if (interleave_gate_up && n % (2 * kTileN)) return NQT_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(packed) & 15u) || (ldw * 2) % 16)
    return NQT_ERR_ARG;
  const int64_t chunks = static_cast<int64_t>(n) * k / 8;
  const int grid = static_cast<int>((chunks + 255) / 256 < 65535 ? (chunks + 255) / 256 : 65535);
  pack_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const __nv_bfloat16*>(w), ldw, n, k,
                                                   interleave_gate_up, static_cast<__nv_bfloat16*>(packed));
  return check_launch("gemm_pack_weight");
}

extern "C" int nqt_gemm_bf16(const void* x, int64_t ldx, const void* wpacked, void* y, int64_t ldy,
                             const void* bias, int m, int n, int k, int epilogue, int ctas, int32_t* status,
                             void* stream) {
  if (!x || !wpacked || !y) return NQT_ERR_ARG;
  if (m < 1 || m > 256 || n < kTileN || k < kBlockK) return NQT_ERR_ARG;
  if (n % kTileN != 0 || k % kBlockK != 0) return NQT_ERR_UNSUPPORTED;
  if (epilogue < kPlain || epilogue > kSiluMul || (epilogue == kBias && bias == nullptr)) return NQT_ERR_ARG;
  // TMA / bulk copies: 16-byte aligned bases and row pitches
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(wpacked) & 15u) || (ldx * 2) % 16 ||
      ldx < k)
    return NQT_ERR_ARG;
  const int out_cols = epilogue == kSiluMul ? n / 2 : n;
  if (ldy < out_cols) return NQT_ERR_ARG;
  const int tiles = n / kTileN;
  const int ldws = (m + 3) / 4 * 4;
  if (tiles > kMaxTiles || static_cast<int64_t>(ldws) * n > kMaxWsFloats) return NQT_ERR_CAPACITY;
  const int mpad = (m + 15) / 16 * 16;
  const int kbt = k / kBlockK;
  const int units = tiles * kbt;
  // one CTA per SM (the shared-memory ring keeps it so), never more CTAs than units
  if (ctas <= 0) ctas = num_sms();
  if (ctas > units) ctas = units;
  int stages = 8;
  while (stages > 2 && smem_bytes(mpad, stages) > 227 * 1024) --stages;
  const int smem = smem_bytes(mpad, stages);
  if (smem > 227 * 1024) return NQT_ERR_UNSUPPORTED;
  Workspace wsp;
  if (workspace(&wsp) != NQT_OK) return NQT_ERR_CUDA;

  CUtensorMap xmap;
  if (encode_2d(&xmap, x, m, k, ldx, mpad) != NQT_OK) {
    set_last_message("gemm: cuTensorMapEncodeTiled failed");
    return NQT_ERR_CUDA;
  }
  const int vec_out = (reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (ldy * 2) % 16 == 0;
  GemmArgs a{static_cast<const uint8_t*>(wpacked), static_cast<__nv_bfloat16*>(y), ldy,
             static_cast<const __nv_bfloat16*>(bias), status, wsp.ws, wsp.ticket, m, n, k, mpad, epilogue, stages,
             kbt, units, vec_out, ldws};
  static std::once_flag once;
  std::call_once(once,
                 [] { cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024); });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, gemm_kernel, xmap, a);
  if (err != cudaSuccess) {
    set_last_error("gemm", err);
    return NQT_ERR_CUDA;
  }
  return NQT_OK;
}
