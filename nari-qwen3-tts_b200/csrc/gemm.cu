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
// MMA reads (16-byte chunk c of row r at chunk c ^ (r % 8)), so a stage is one
// bulk copy.  X (the step's activations, L2-resident) comes through a 2-D
// tensor map (box 64 x Mpad, 128-byte swizzle).
//
// Work split.  The grid is (N / 128 tiles) x S, one thread-block cluster of S
// CTAs per tile (S <= 8, chosen so the grid is about one CTA per SM): CTA r
// of a cluster streams the r-th contiguous K slice of the tile, with every
// stage of a short slice in flight at once.  The S fp32 partials are summed
// through distributed shared memory: each CTA parks its partial D^T
// token-major in its own shared memory, and after a cluster barrier CTA r
// reduces tokens [r m / S, (r+1) m / S) over the S partials (16-byte remote
// loads), applies the epilogue and writes Y.  No global workspace, atomics or
// second pass.
//
// Warp roles (6 warps): 0 copy producer, 1 TMEM owner + MMA issuer, 2-5 the
// epilogue (warp w reads TMEM lanes 32 (w % 4) ..).  Epilogues:
//   plain    Y = bf16(acc)
//   bias     Y = bf16(acc + bias)                       (nn.Linear with bias)
//   silu_mul W rows interleaved in 64-row blocks [gate 64 | up 64]; output
//            column f of block b is silu(g) * u of rows 128 b + f, 128 b + 64 + f,
//            with g and u rounded to bf16 first (the unfused gate_up GEMM
//            followed by silu_and_mul); Y is [M, N / 2].
// Every mbarrier wait is bounded and reports NQT_DEV_TIMEOUT; on a timeout a
// thread skips its remaining work but still reaches every cluster barrier, so
// no CTA leaves while a peer may read its shared memory.  The kernel is
// launched with programmatic stream serialization: the W copies are issued
// before griddepcontrol.wait (the weights do not depend on the previous
// kernel), X, Y and everything after them come after it.
//
// Replaces the torch/cuBLAS projections of the decoder layers
// (model/layers.py:195-270, model/components.py:300-356) and the sm90-only
// fused gate/up path (executor/optimizations.py:22-47).
#include <mutex>

#include "common.cuh"
#include "gemm_common.cuh"
#include "tcgen05.cuh"

namespace nqt {
namespace {

using namespace gemm_detail;

constexpr int kTileN = 128;                    // W rows per tile (MMA M)
constexpr int kBlockK = 64;                    // K per unit (one 128-byte swizzle row)
constexpr int kThreads = 6 * 32;
constexpr int kWBytes = kTileN * kBlockK * 2;  // 16 KB per unit
constexpr int kMaxSplit = 8;                   // portable cluster size
constexpr int kSmemBudget = 227 * 1024;
constexpr int kMaxGroup = 4;   // K units per stage: one W copy of up to 64 KB, one X copy
constexpr int kMaxStages = 8;

enum Epilogue : int { kPlain = 0, kBias = 1, kSiluMul = 2 };

struct GemmArgs {
  const uint8_t* wpack;
  __nv_bfloat16* y;
  int64_t ldy;
  const __nv_bfloat16* bias;
  int32_t* status;
  int m, n, k;
  int mpad;  // MMA N: m rounded up to 16
  int epilogue;
  int stages;
  int kbt;    // K units per tile
  int own;    // tokens per cluster rank, own_tokens(m, S)
  int group;    // K units per stage (one W bulk copy, one X tensor load)
  int vec_out;  // y and its row pitch 8-byte aligned: 4-column vector stores
};

__host__ __device__ constexpr int x_bytes(int mpad) { return mpad * kBlockK * 2; }
// a stage: `group` W units [group][128 x 128 B] then their X slabs [group][mpad x 128 B]
__host__ __device__ constexpr int stage_bytes(int mpad, int group) { return group * (kWBytes + x_bytes(mpad)); }
// Tokens each CTA of a cluster of S finishes, and the receive buffer that holds every sender's fp32
// slice of them: [S senders][own tokens][128 rows].  The sender parks its whole partial the same way,
// [S * own tokens][128 rows], over its drained stage ring.
__host__ __device__ constexpr int own_tokens(int m, int S) { return (m + S - 1) / S; }
__host__ __device__ constexpr int park_bytes(int m, int S) { return S * own_tokens(m, S) * kTileN * 4; }
// a CTA alone (S = 1) sums nothing and reads its own parked partial
__host__ __device__ constexpr int recv_bytes(int m, int S) { return S > 1 ? park_bytes(m, S) : 0; }
__host__ __device__ constexpr int ring_bytes(int mpad, int group, int m, int S, int stages) {
  return stages * stage_bytes(mpad, group) > park_bytes(m, S) ? stages * stage_bytes(mpad, group)
                                                               : park_bytes(m, S);
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap xmap, GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = a.stages;
  const int G = a.group;
  const int sb = stage_bytes(a.mpad, G);
  const int xoff = G * kWBytes;  // X slabs after the stage's W units
  const int S = gridDim.y;
  const int own = a.own;  // tokens per owner CTA (padded to 4)
  const int ring = ring_bytes(a.mpad, G, a.m, S, ST);
  float* park = reinterpret_cast<float*>(smem);           // [S * own tokens][128 rows], over the drained ring
  // [S senders][own tokens][128 rows]; a CTA alone reads its park directly
  float* recv = S > 1 ? reinterpret_cast<float*>(smem + ring) : park;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring + recv_bytes(a.m, S));
  uint64_t* empty = full + ST;
  uint64_t* done = empty + ST;   // the accumulator is complete
  uint64_t* recv_bar = done + 1; // every sender's slice of this CTA's tokens has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int rank = static_cast<int>(cluster_rank());  // == blockIdx.y: cluster dims (1, S, 1)
  const int kb0 = rank * a.kbt / S, kb1 = (rank + 1) * a.kbt / S;
  const int nu = kb1 - kb0;           // >= 1: S <= kbt
  const int nl = (nu + G - 1) / G;     // stage loads
  const uint8_t* wsrc = a.wpack + (static_cast<int64_t>(tile) * a.kbt + kb0) * kWBytes;
  uint32_t tmem_cols = 32;
  while (tmem_cols < static_cast<uint32_t>(a.mpad)) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(recv_bar, 1);
    fence_barrier_init();
    // the one arrival on recv_bar; the peers' copies complete its transaction count
    if (S > 1) mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(recv_bytes(a.m, S)));
    // W does not depend on the previous kernel: start streaming it at once; X (the previous
    // kernel's output) once that kernel has completed.  Load i carries units [i G, i G + g) of the
    // slice; its X box always holds G slabs (past the slice: unused, past K: zero fill).
    const int pro = nl < ST ? nl : ST;
    for (int i = 0; i < pro; ++i) {
      const int g = nu - i * G < G ? nu - i * G : G;
      mbar_arrive_expect_tx(&full[i], g * kWBytes + G * x_bytes(a.mpad));
      bulk_load(smem + i * sb, wsrc + static_cast<int64_t>(i) * G * kWBytes, g * kWBytes, &full[i]);
    }
    prefetch_tensormap(&xmap);
    grid_dependency_wait();
    for (int i = 0; i < pro; ++i) tma_load_x(smem + i * sb + xoff, &xmap, &full[i], 0, kb0 + i * G);
  }
  // the next kernel may be scheduled now and stream its own weights while this one finishes
  grid_dependents_launch();
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, tmem_cols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();  // also orders every thread after thread 0's dependency wait (Y may be written)
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  cluster_arrive();  // this CTA's barriers are initialised and recv_bar armed (release)
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const int pro = nl < ST ? nl : ST;  // issued with the barrier initialisation
      for (int i = pro; i < nl && ok; ++i) {
        const int s = i % ST;
        if (!mbar_wait(&empty[s], ((i / ST) - 1) & 1, a.status)) {
          ok = false;
          break;
        }
        const int g = nu - i * G < G ? nu - i * G : G;
        mbar_arrive_expect_tx(&full[s], g * kWBytes + G * x_bytes(a.mpad));
        bulk_load(smem + s * sb, wsrc + static_cast<int64_t>(i) * G * kWBytes, g * kWBytes, &full[s]);
        tma_load_x(smem + s * sb + xoff, &xmap, &full[s], 0, kb0 + i * G);
      }
    }
    cluster_wait();
    cluster_arrive_relaxed();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16_f32(kTileN, a.mpad, false, false);
      for (int i = 0; i < nl; ++i) {
        const int s = i % ST;
        if (!mbar_wait(&full[s], (i / ST) & 1, a.status)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const int g = nu - i * G < G ? nu - i * G : G;
        for (int u = 0; u < g; ++u) {
          const uint32_t w_addr = smem_addr(smem + s * sb + u * kWBytes);
          const uint32_t x_addr = smem_addr(smem + s * sb + xoff + u * x_bytes(a.mpad));
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t da = tc::smem_desc_sw128(w_addr + kk * 32, 16, 1024);
            const uint64_t db = tc::smem_desc_sw128(x_addr + kk * 32, 16, 1024);
            tc::mma_f16_ss(tmem, da, db, idesc, (i > 0 || u > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc::commit(&empty[s]);
      }
      tc::commit(done);  // arrives once every MMA above has completed
    }
    cluster_wait();
    cluster_arrive_relaxed();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // tile row = TMEM lane
    ok = mbar_wait(done, 0, a.status);
    tc::fence_after_sync();
    // park the partial token-major: park[tok][row] (conflict-free), zeros past the accumulator
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int padded = S * own;
    for (int c = 0; c < padded; c += 64) {  // two 32-column TMEM loads in flight per wait
      uint32_t r[2][32];
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (c + 32 * h < padded && c + 32 * h < static_cast<int>(tmem_cols)) tc::ld_32x32b_x32(t_row + c + 32 * h, r[h]);
      tc::wait_ld();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const bool have = c + 32 * h < static_cast<int>(tmem_cols) && ok;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int tok = c + 32 * h + e;
          if (tok < padded) park[tok * kTileN + row] = have ? __uint_as_float(r[h][e]) : 0.f;
        }
      }
    }
    fence_proxy_async_smem();  // the parked partial is read by the bulk copies (async proxy)
    epi_bar();
    cluster_wait();  // every peer's recv_bar is armed
    if (threadIdx.x == 64 && S > 1) {
      // owner o gets tokens [o * own, o * own + own) of this partial in its slot [rank]
      const uint32_t slice = static_cast<uint32_t>(own * kTileN * 4);
      const uint32_t dst = smem_addr(recv) + static_cast<uint32_t>(rank) * slice;
      const uint32_t bar = smem_addr(recv_bar);
      for (int o = 0; o < S; ++o)
        bulk_copy_to_peer(map_rank(dst, o), park + o * own * kTileN, slice, map_rank(bar, o));
    }
    // receive this CTA's tokens [rank * own, rank * own + own) from every sender, sum, epilogue, store
    const bool got = S == 1 || mbar_wait(recv_bar, 0, a.status);
    cluster_arrive_relaxed();  // everything addressed to this CTA has landed (its sources are read)
    const int t0 = rank * own;
    const int nt = a.m - t0 < own ? a.m - t0 : own;
    const bool silu = a.epilogue == kSiluMul;
    // thread = one fixed quad of 4 tile rows (silu: 4 gate rows and their up rows) and every
    // (128 / quads)-th token; four tokens per pass as independent load -> sum -> store chains (one
    // warp per scheduler has nothing else to hide their latency behind)
    const uint32_t recv_s = smem_addr(recv);
    const uint32_t slice_stride = static_cast<uint32_t>(own * kTileN * 4);  // bytes between senders
    const int quads = silu ? 16 : 32;
    const int q = row % quads;
    const int tstep = kTileN / quads;  // tokens covered by one pass of the 128 threads
    const int col = silu ? tile * 64 + 4 * q : tile * kTileN + 4 * q;
    float4 bias4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.epilogue == kBias) {
      bias4.x = __bfloat162float(a.bias[col]);
      bias4.y = __bfloat162float(a.bias[col + 1]);
      bias4.z = __bfloat162float(a.bias[col + 2]);
      bias4.w = __bfloat162float(a.bias[col + 3]);
    }
    __nv_bfloat16* const ybase = a.y + col;
    const int64_t ldy = a.ldy;
    const bool vec = a.vec_out != 0;
    for (int tb = row / quads; tb < nt; tb += 4 * tstep) {
      float4 g[4], u[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) g[k] = u[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s2 = 0; s2 < S; ++s2) {
        const uint32_t base = recv_s + s2 * slice_stride + static_cast<uint32_t>((tb * kTileN + 4 * q) * 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (tb + k * tstep < nt) {
            const uint32_t src = base + static_cast<uint32_t>(k * tstep * kTileN * 4);
            const float4 gv = ld_shared_v4(src);
            g[k].x += gv.x, g[k].y += gv.y, g[k].z += gv.z, g[k].w += gv.w;
            if (silu) {
              const float4 uv = ld_shared_v4(src + 64 * 4);
              u[k].x += uv.x, u[k].y += uv.y, u[k].z += uv.z, u[k].w += uv.w;
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int t = tb + k * tstep;
        if (t >= nt || !got) continue;
        float v0, v1, v2, v3;
        if (silu) {
          v0 = silu_mul(bf16_round(g[k].x), bf16_round(u[k].x));
          v1 = silu_mul(bf16_round(g[k].y), bf16_round(u[k].y));
          v2 = silu_mul(bf16_round(g[k].z), bf16_round(u[k].z));
          v3 = silu_mul(bf16_round(g[k].w), bf16_round(u[k].w));
        } else {
          v0 = g[k].x + bias4.x, v1 = g[k].y + bias4.y, v2 = g[k].z + bias4.z, v3 = g[k].w + bias4.w;
        }
        __nv_bfloat16* dst = ybase + static_cast<int64_t>(t0 + t) * ldy;
        const __nv_bfloat162 lo = __floats2bfloat162_rn(v0, v1), hi = __floats2bfloat162_rn(v2, v3);
        if (vec) {
          uint2 pk;
          pk.x = *reinterpret_cast<const uint32_t*>(&lo);
          pk.y = *reinterpret_cast<const uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(dst) = pk;
        } else {
          dst[0] = lo.x;
          dst[1] = lo.y;
          dst[2] = hi.x;
          dst[3] = hi.y;
        }
      }
    }
  }
  // every CTA has received all it was sent: no store of this CTA is still in flight when it leaves
  cluster_wait();
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

int smem_bytes(int mpad, int group, int m, int S, int stages) {
  return 1024 + ring_bytes(mpad, group, m, S, stages) + recv_bytes(m, S) + (2 * stages + 2) * 8 + 16;
}

// Clusters of S CTAs with `smem` bytes each that the current device holds at once (cached).
int max_active_clusters(int S, int smem) {
  static std::mutex mu;
  static int dev_cached = -1;
  static int cache[kMaxSplit + 1][64] = {};  // [S][smem in 4 KB steps]
  int dev = 0;
  cudaGetDevice(&dev);
  const int bucket = smem / 4096 < 64 ? smem / 4096 : 63;
  std::lock_guard<std::mutex> lock(mu);
  if (dev != dev_cached) {
    for (auto& row : cache)
      for (int& v : row) v = 0;
    dev_cached = dev;
  }
  int& v = cache[S][bucket];
  if (v == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, S, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = S;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = 1 << 20;  // unknown: do not shrink the split
    }
    v = n;
  }
  return v;
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
                             const void* bias, int m, int n, int k, int epilogue, int split, int32_t* status,
                             void* stream) {
  if (!x || !wpacked || !y) return NQT_ERR_ARG;
  if (m < 1 || m > 256 || n < kTileN || k < kBlockK) return NQT_ERR_ARG;
  if (n % kTileN != 0 || k % kBlockK != 0) return NQT_ERR_UNSUPPORTED;
  if (epilogue < kPlain || epilogue > kSiluMul || (epilogue == kBias && bias == nullptr)) return NQT_ERR_ARG;
  if (split < 0 || split > kMaxSplit) return NQT_ERR_ARG;
  // TMA / bulk copies: 16-byte aligned bases and row pitches
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(wpacked) & 15u) || (ldx * 2) % 16 ||
      ldx < k)
    return NQT_ERR_ARG;
  const int out_cols = epilogue == kSiluMul ? n / 2 : n;
  if (ldy < out_cols) return NQT_ERR_ARG;
  const int tiles = n / kTileN;
  if (tiles > 65535) return NQT_ERR_UNSUPPORTED;
  const int mpad = (m + 15) / 16 * 16;
  const int kbt = k / kBlockK;
  // K split = cluster size: the largest power of two (<= 8, <= K units per tile) that keeps the grid
  // within one CTA per SM and within the clusters the GPU can hold at once
  int S = split;
  if (S == 0) {
    S = 1;
    while (S * 2 <= kMaxSplit && S * 2 <= kbt && tiles * S * 2 <= num_sms()) S *= 2;
  }
  if (S > kbt) S = kbt;
  // TMEM holds 512 columns per SM.  A CTA blocked in tcgen05.alloc while its cluster peers wait at the
  // cluster barrier would deadlock, so shared memory is padded until no SM can hold more CTAs than
  // their columns fit: at least cols/512 of the SM's 228 KB, plus the 1 KB the runtime reserves per CTA.
  int tmem_cols = 32;
  while (tmem_cols < mpad) tmem_cols <<= 1;
  const int tmem_floor = tmem_cols * (233472 / 512);
  // per split: K units per stage (up to kMaxGroup: few, large copies), then as many stages as fit
  struct Plan {
    int group, stages, smem;
  };
  auto plan_for = [&](int s_split) {
    Plan pl;
    const int per_cta = (kbt + s_split - 1) / s_split;  // K units of the longest slice
    pl.group = per_cta < kMaxGroup ? per_cta : kMaxGroup;
    // keep two stages in flight when the slice has two loads' worth (a lone stage serialises copy and MMA)
    const int want = per_cta > pl.group ? 2 : 1;
    while (pl.group > 1 && smem_bytes(mpad, pl.group, m, s_split, want) > kSmemBudget) --pl.group;
    const int loads = (per_cta + pl.group - 1) / pl.group;
    pl.stages = loads < kMaxStages ? loads : kMaxStages;
    while (pl.stages > 1 && smem_bytes(mpad, pl.group, m, s_split, pl.stages) > kSmemBudget) --pl.stages;
    const int sm = smem_bytes(mpad, pl.group, m, s_split, pl.stages);
    pl.smem = sm > tmem_floor ? sm : tmem_floor;
    return pl;
  };
  // a split whose park and receive buffers do not fit beside one stage runs unsplit
  if (plan_for(S).smem > kSmemBudget) S = 1;
  Plan pl = plan_for(S);
  if (pl.smem > kSmemBudget) return NQT_ERR_UNSUPPORTED;
  static std::once_flag once;
  std::call_once(once,
                 [] { cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget); });
  // an automatic split whose clusters do not all fit at once runs a second wave: halve it until they do
  while (split == 0 && S > 1 && tiles > max_active_clusters(S, pl.smem)) {
    S /= 2;
    pl = plan_for(S);
    if (pl.smem > kSmemBudget) return NQT_ERR_UNSUPPORTED;
  }

  CUtensorMap xmap;
  if (encode_x_slabs(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, m, k / kBlockK, ldx * 2, mpad, pl.group) !=
      NQT_OK) {
    set_last_message("gemm: cuTensorMapEncodeTiled failed");
    return NQT_ERR_CUDA;
  }
  GemmArgs a{static_cast<const uint8_t*>(wpacked), static_cast<__nv_bfloat16*>(y), ldy,
             static_cast<const __nv_bfloat16*>(bias), status, m, n, k, mpad, epilogue, pl.stages, kbt,
             own_tokens(m, S), pl.group,
             (reinterpret_cast<uintptr_t>(y) & 7u) == 0 && ldy % 4 == 0 ? 1 : 0};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, S, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  attrs[1].id = cudaLaunchAttributeClusterDimension;
  attrs[1].val.clusterDim.x = 1;
  attrs[1].val.clusterDim.y = S;
  attrs[1].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, gemm_kernel, xmap, a);
  if (err != cudaSuccess) {
    set_last_error("gemm", err);
    return NQT_ERR_CUDA;
  }
  return NQT_OK;
}
