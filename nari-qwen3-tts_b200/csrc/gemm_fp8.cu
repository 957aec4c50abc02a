// FP8 (e4m3) block-scaled weight-streaming GEMM for the talker's gate/up
// projection, and the quantisers that feed it (sm_100a, tcgen05
// kind::f8f6f4 + TMA).
//
//   Y[M, N] = sum over 128-wide K blocks b of
//             (Xq[:, b] . Wq[:, b]^T) * sx[b, token] * sw[weight row / 128, b]
//
// The reference's production executor requires this for every talker layer
// (executor/build.py:73 -> executor/optimizations.py:22-47), on a path that only
// starts on sm90: the gate/up weight is quantised once into 128 x 128 blocks with
// power-of-two scales (model/layers.py:11-25) and the bf16 activations are
// quantised per token per 128-element block inside the library GEMM
// (model/layers.py:242-256, flashinfer fp8_blockscale_gemm_sm90, bf16 input).
// The rules are in fp8.cuh.
//
// Weight quantiser (load time): one CTA per 128 x 128 block, written in the
// reference's layout (q [N, K] row-major, scales [N/128, K/128] fp32).
// Activation quantiser: one warp per (token, 128-block); scales stored
// K-block-major [K/128][ld] (a block's tokens contiguous).  The talker step
// uses the same rule fused into the post-attention add + RMSNorm (norm.cu).
//
// GEMM.  The quantised weight is packed at load time into 16 KB units
// [N/128 tiles][K/128][128 rows x 128 B] in the MMA's 128-byte-swizzled order
// (one bulk copy each).  A tile of 128 weight rows is the MMA's M and a chunk of
// up to 128 tokens its N (grid z: one chunk per 128 tokens).  One SM pulls only
// ~35-40 GB/s (about 58 with two CTAs on it), so the stream needs every SM: the
// K range of a tile is split over S CTAs (grid y), S chosen so that the busiest
// SM streams the fewest K blocks - the talker's gate/up (96 tiles x 16 K blocks)
// runs as 3 x 96 CTAs, two per SM, all resident at once.
//
// Scale promotion: each K block's four K=32 MMAs accumulate into their own TMEM
// buffer (a ring of up to 8), and the four epilogue warps (one weight row per
// thread) fold every finished block into fp32 registers,
//     acc[t] = fma(block[t], sx[b, t] * sw[row block, b], acc[t]),
// then hand the buffer back to the MMA issuer, so the promotion overlaps the
// weight stream.  The scale products are staged in shared memory once per CTA.
//
// Split-K sum (S > 1): every CTA first takes its tile's ticket.  The others write
// their fp32 partial [tokens][128 rows] to a global workspace (L2-resident) and
// count it in on the tile's `written` counter; the CTA that completes the ticket
// parks its own partial in shared memory, waits (bounded) until the others have
// written - they all hold tickets already, so they are resident and finish
// unconditionally - returns both counters to zero, brings their partials into its
// drained stage ring with bulk copies and adds all S in rank order (so the result
// does not depend on which CTA finished last), then runs the epilogue.
// Epilogues: plain (Y = bf16) and SwiGLU, Y = silu(bf16 g) * bf16 u (the unfused
// GEMM followed by silu_and_mul), on gate/up rows packed in 32-row groups
// [gate 16 | up 16] (a tile holds gate and up rows 64 t .. 64 t + 63): lanes l and
// l + 16 of a warp hold a gate row and its up row, swap half of their tokens with
// one shuffle each and finish the other half.
//
// Warp roles (6 warps): 0 copy producer, 1 TMEM owner + MMA issuer, 2-5 scale
// promotion and epilogue.  Every mbarrier wait is bounded and reports
// NQT_DEV_TIMEOUT; a thread that gives up skips its remaining work (a CTA still
// counts in on its ticket, so the tickets return to zero), and before the CTA
// exits one thread waits for the copies it issued that were never consumed.
// Launched with programmatic stream serialization: the weight copies are issued
// before griddepcontrol.wait, X and its scales after it.
#include <mutex>

#include "common.cuh"
#include "fp8.cuh"
#include "gemm_common.cuh"
#include "tcgen05.cuh"

namespace nqt {
namespace {

using namespace gemm_detail;

constexpr int kTileN = 128;                // weight rows per tile (MMA M)
constexpr int kBlockK = 128;               // e4m3 elements per unit row (128 B) = one scale block
constexpr int kThreads = 6 * 32;
constexpr int kWBytes = kTileN * kBlockK;  // 16 KB per unit
constexpr int kMaxSplit = 8;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kPairBudget = 233472 / 2 - 1024;  // two CTAs per SM
constexpr int kMaxGroup = 4;
constexpr int kMaxStages = 8;
constexpr int kMaxBufs = 8;  // TMEM accumulator buffers (one K block each)

enum Epilogue : int { kPlain = 0, kSiluMul = 2 };  // the numbering of nqt_gemm_bf16

struct Fp8Args {
  const uint8_t* wpack;
  const float* wscale;  // [N / 128][kbt], blocks of the unpacked row order
  const float* xscale;  // [kbt][ld_xs]
  int64_t ld_xs;
  __nv_bfloat16* y;
  int64_t ldy;
  float* partials;   // [chunks][tiles][S][MP][128] (S > 1)
  int32_t* tickets;  // [2][chunks][tiles] (S > 1): tickets, then written counters; zero between launches
  int32_t* status;
  int m, n, kbt;
  int epilogue, interleave;
  int stages, group, bufs;
  uint32_t tmem_cols;
  int vec16;  // y 16-byte aligned with a row pitch of a multiple of 8: 16-byte stores
};

__host__ __device__ constexpr int x_bytes(int mp) { return mp * kBlockK; }
// a stage: `group` W units [group][128 x 128 B] then their X slabs [group][mp x 128 B]
__host__ __device__ constexpr int stage_bytes(int mp, int group) { return group * (kWBytes + x_bytes(mp)); }
// the drained ring is reused by the split-K sum (two partials [mp][128] fp32 at least: the own one and a copy)
// and then by the staged output tile ([mp][128] bf16 at most)
__host__ __device__ constexpr int ring_bytes(int mp, int group, int stages) {
  return stages * stage_bytes(mp, group) > mp * 1024 ? stages * stage_bytes(mp, group) : mp * 1024;
}
// per-CTA scale products sx[b, t] * sw[half, b] as [2 halves][units][mp]
__host__ __device__ constexpr int tables_bytes(int mp, int units) { return 2 * units * mp * 4; }
__host__ __device__ constexpr int smem_bytes(int mp, int group, int stages, int units, int bufs) {
  return 1024 + ring_bytes(mp, group, stages) + tables_bytes(mp, units) + (2 * stages + 2 * bufs + 2) * 8 + 16;
}

template <int MP, int MINB>
__global__ void __launch_bounds__(kThreads, MINB)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap xmap, Fp8Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = a.stages, G = a.group, R = a.bufs;
  const int S = gridDim.y;
  const int sb = stage_bytes(MP, G);
  const int xoff = G * kWBytes;
  const int units_max = (a.kbt + S - 1) / S;
  float* s_sc = reinterpret_cast<float*>(smem + ring_bytes(MP, G, ST));  // [2][units_max][MP]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_sc + 2 * units_max * MP);
  uint64_t* empty = full + ST;
  uint64_t* accf = empty + ST;  // a K block's accumulator buffer is complete (MMA commit)
  uint64_t* acce = accf + R;    // ... and has been read by the four epilogue warps
  uint64_t* done = acce + R;    // every MMA of this CTA has completed
  uint64_t* sumbar = done + 1;  // split K: the other CTAs' partials have landed in the ring
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sumbar + 1);
  volatile int* s_consumed = reinterpret_cast<volatile int*>(tmem_slot + 1);  // loads the MMA issuer took
  volatile int* s_issued = s_consumed + 1;                                    // loads the producer issued
  volatile int* s_last = s_issued + 1;                                        // this CTA completes the ticket

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int rank = blockIdx.y;
  const int t0 = blockIdx.z * MP;  // first token of this chunk
  const int kb0 = rank * a.kbt / S, kb1 = (rank + 1) * a.kbt / S;
  const int nu = kb1 - kb0;  // >= 1: S <= kbt
  const int nl = (nu + G - 1) / G;
  const uint8_t* wsrc = a.wpack + (static_cast<int64_t>(tile) * a.kbt + kb0) * kWBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < R; ++r) {
      mbar_init(&accf[r], 1);
      mbar_init(&acce[r], 4);
    }
    mbar_init(done, 1);
    mbar_init(sumbar, 1);
    fence_barrier_init();
    // the weights do not depend on the previous kernel: stream them at once; X once it has completed
    const int pro = nl < ST ? nl : ST;
    for (int i = 0; i < pro; ++i) {
      const int g = nu - i * G < G ? nu - i * G : G;
      mbar_arrive_expect_tx(&full[i], g * kWBytes + G * x_bytes(MP));
      bulk_load(smem + i * sb, wsrc + static_cast<int64_t>(i) * G * kWBytes, g * kWBytes, &full[i]);
    }
    prefetch_tensormap(&xmap);
    grid_dependency_wait();
    for (int i = 0; i < pro; ++i) tma_load_x(smem + i * sb + xoff, &xmap, &full[i], t0, kb0 + i * G);
    *s_consumed = 0;
    *s_issued = pro;
  }
  grid_dependents_launch();
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, a.tmem_cols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();  // also orders every thread after thread 0's dependency wait (X scales, Y, tickets)
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = nl < ST ? nl : ST;
      for (int i = issued; i < nl; ++i) {
        const int s = i % ST;
        if (!mbar_wait(&empty[s], ((i / ST) - 1) & 1, a.status)) break;
        const int g = nu - i * G < G ? nu - i * G : G;
        mbar_arrive_expect_tx(&full[s], g * kWBytes + G * x_bytes(MP));
        bulk_load(smem + s * sb, wsrc + static_cast<int64_t>(i) * G * kWBytes, g * kWBytes, &full[s]);
        tma_load_x(smem + s * sb + xoff, &xmap, &full[s], t0, kb0 + i * G);
        issued = i + 1;
      }
      *s_issued = issued;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_e4m3_f32(kTileN, MP);
      bool run = true;
      for (int i = 0; i < nl && run; ++i) {
        const int s = i % ST;
        if (!mbar_wait(&full[s], (i / ST) & 1, a.status)) break;
        *s_consumed = i + 1;
        tc::fence_after_sync();
        const int g = nu - i * G < G ? nu - i * G : G;
        for (int u = 0; u < g; ++u) {
          const int b = i * G + u;
          const int buf = b % R;
          // the buffer's previous block has been read out by the epilogue warps
          if (b >= R && !mbar_wait(&acce[buf], ((b / R) - 1) & 1, a.status)) {
            run = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * MP);
          const uint32_t w_addr = smem_addr(smem + s * sb + u * kWBytes);
          const uint32_t x_addr = smem_addr(smem + s * sb + xoff + u * x_bytes(MP));
#pragma unroll
          for (int kk = 0; kk < kBlockK / 32; ++kk) {
            const uint64_t da = tc::smem_desc_sw128(w_addr + kk * 32, 16, 1024);
            const uint64_t db = tc::smem_desc_sw128(x_addr + kk * 32, 16, 1024);
            tc::mma_f8_ss(d, da, db, idesc, kk > 0 ? 1u : 0u);
          }
          tc::commit(&accf[buf]);
        }
        tc::commit(&empty[s]);
      }
      tc::commit(done);
      mbar_wait(done, 0, a.status);  // no MMA of this CTA still runs when its TMEM is freed
    }
  } else {
    // ---------------------------------------------------------------- scale promotion + epilogue
    // scale products sx[b, t] * sw[half, b], staged once; four independent loads in flight per thread
    const int et = threadIdx.x - 64;  // 0 .. 127
    const int brow0 = a.interleave ? tile / 2 : tile;
    const int brow1 = a.interleave ? a.n / 256 + tile / 2 : tile;
    for (int base = 0; base < nu * MP; base += 4 * 128) {
      float sx[4], w0[4], w1[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int idx = base + et + j * 128;
        const int b = idx / MP, t = t0 + idx - b * MP;
        sx[j] = w0[j] = w1[j] = 0.f;
        if (idx < nu * MP) {
          if (t < a.m) sx[j] = __ldg(a.xscale + static_cast<int64_t>(kb0 + b) * a.ld_xs + t);
          w0[j] = __ldg(a.wscale + static_cast<int64_t>(brow0) * a.kbt + kb0 + b);
          w1[j] = __ldg(a.wscale + static_cast<int64_t>(brow1) * a.kbt + kb0 + b);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int idx = base + et + j * 128;
        if (idx < nu * MP) {
          const int b = idx / MP, c = idx - b * MP;
          s_sc[b * MP + c] = sx[j] * w0[j];
          s_sc[(units_max + b) * MP + c] = sx[j] * w1[j];
        }
      }
    }
    epi_bar();
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // tile row = TMEM lane
    const int half = (a.interleave && lane >= 16) ? 1 : 0;  // gate / up row (weight-scale block row)
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float acc[MP];
#pragma unroll
    for (int e = 0; e < MP; ++e) acc[e] = 0.f;
    bool ok = true;
    constexpr int kChunk = MP < 64 ? MP : 64;  // columns read per TMEM wait
    for (int b = 0; b < nu; ++b) {
      const int buf = b % R;
      if (!mbar_wait(&accf[buf], (b / R) & 1, a.status)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const float* scb = s_sc + (half * units_max + b) * MP;
#pragma unroll
      for (int h = 0; h < MP; h += kChunk) {
        uint32_t r0[32], r1[32];
        const uint32_t taddr = t_row + static_cast<uint32_t>(buf * MP + h);
        tc::ld_32x32b_x32(taddr, r0);
        if (kChunk == 64) tc::ld_32x32b_x32(taddr + 32, r1);
        tc::wait_ld();
        if (h + kChunk >= MP) {  // the whole buffer is in registers: give it back
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[buf]);
        }
#pragma unroll
        for (int e = 0; e < kChunk; e += 4) {
          const float4 sc4 = *reinterpret_cast<const float4*>(scb + h + e);
          const uint32_t* src = e < 32 ? r0 + e : r1 + (e - 32);
          acc[h + e] = fmaf(__uint_as_float(src[0]), sc4.x, acc[h + e]);
          acc[h + e + 1] = fmaf(__uint_as_float(src[1]), sc4.y, acc[h + e + 1]);
          acc[h + e + 2] = fmaf(__uint_as_float(src[2]), sc4.z, acc[h + e + 2]);
          acc[h + e + 3] = fmaf(__uint_as_float(src[3]), sc4.w, acc[h + e + 3]);
        }
      }
    }
    if (!ok) {
#pragma unroll
      for (int e = 0; e < MP; ++e) acc[e] = 0.f;
    }
    bool last = true;
    if (S > 1) {
      // split K: take the tile's ticket first.  The CTA that completes it sums; the others write their partial
      // to the workspace and count it in on the tile's `written` counter.  The summing CTA waits for that
      // count only on CTAs that already hold a ticket (resident, and writing unconditionally), so the wait
      // ends; it keeps its own partial in shared memory, off the global round trip.
      const int64_t slot = static_cast<int64_t>(blockIdx.z) * gridDim.x + tile;
      const int64_t slots = static_cast<int64_t>(gridDim.z) * gridDim.x;
      int32_t* ticket = a.tickets + slot;
      int32_t* written = a.tickets + slots + slot;
      float* parts = a.partials + slot * S * MP * kTileN;
      constexpr uint32_t kPart = MP * kTileN * 4;  // bytes of one partial
      // the drained ring holds `cap` partials: the own one in the last slot, copies in the others
      const int cap = ring_bytes(MP, G, ST) / static_cast<int>(kPart);
      float* own = reinterpret_cast<float*>(smem + (cap - 1) * kPart);
      if (threadIdx.x == 64) *s_last = atomicAdd(ticket, 1) == S - 1 ? 1 : 0;
      epi_bar();
      last = *s_last != 0;
      if (!last) {
#pragma unroll
        for (int e = 0; e < MP; ++e) __stcg(parts + (rank * MP + e) * kTileN + row, acc[e]);
        epi_bar();  // the CTA's stores happen before thread 64's release below
        if (threadIdx.x == 64) {
          __threadfence();
          atomicAdd(written, 1);
        }
      } else {
#pragma unroll
        for (int e = 0; e < MP; ++e) own[e * kTileN + row] = acc[e];
        if (threadIdx.x == 64) {
          bool ready = false;
          const uint64_t start = global_timer_ns();
          while (true) {
            if (ld_acquire_gpu(written) >= S - 1) {
              ready = true;
              break;
            }
            if (global_timer_ns() - start > kWaitLimitNs) break;
          }
          if (!ready) report(a.status, NQT_DEV_TIMEOUT);
          *ticket = 0;  // every CTA of this tile has counted in on both: reset for the next launch
          *written = 0;
          fence_proxy_async_global();  // the acquired partials are read by the bulk copies below
        }
        // every partial is added in rank order (the own one from shared memory), `cap - 1` copies per
        // round: the sum does not depend on which CTA completed the ticket
#pragma unroll
        for (int e = 0; e < MP; ++e) acc[e] = 0.f;
        const int per_round = cap - 1;
        int p = 0, round = 0;
        while (p < S) {
          // partials p .. q - 1 this round: up to per_round copies, the own one free
          int q = p, copies = 0;
          while (q < S && (q == rank || copies < per_round)) copies += q++ != rank ? 1 : 0;
          if (copies > 0) {
            epi_bar();  // (first round: the own partial is parked; later: the previous round is read)
            if (threadIdx.x == 64) {
              mbar_arrive_expect_tx(sumbar, static_cast<uint32_t>(copies) * kPart);
              for (int r = p, j = 0; r < q; ++r)
                if (r != rank) bulk_load(smem + (j++) * kPart, parts + static_cast<int64_t>(r) * MP * kTileN, kPart,
                                         sumbar);
            }
          } else {
            epi_bar();
          }
          const bool got = copies == 0 || mbar_wait(sumbar, round & 1, a.status);
          for (int r = p, j = 0; r < q && got; ++r) {
            const float* src = (r == rank ? own : reinterpret_cast<const float*>(smem + (j++) * kPart)) + row;
#pragma unroll
            for (int e = 0; e < MP; ++e) acc[e] += src[e * kTileN];
          }
          if (copies > 0) ++round;
          p = q;
        }
      }
    }
    if (last) {
      const int mt = a.m - t0 < MP ? a.m - t0 : MP;  // tokens of this chunk
      // the output tile is staged in the drained ring as [MP tokens][cols] bf16, then leaves in 16-byte pieces
      // of its token rows (scattered 2-byte stores from the owning threads cost several times more)
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem);
      const int cols = a.epilogue == kSiluMul ? 64 : kTileN;
      if (a.epilogue == kSiluMul) {
        // lane l < 16 holds a gate row and lane l + 16 the up row of the same output column: the gate lane
        // finishes tokens [0, MP/2), the up lane tokens [MP/2, MP), each sending the other the value it needs
        constexpr int kHalf = MP / 2;
        const bool gate = lane < 16;
        const int c = quarter * 16 + (lane & 15);
        const int tok0 = gate ? 0 : kHalf;
#pragma unroll
        for (int e = 0; e < kHalf; ++e) {
          // gate lane sends gate[e + kHalf] and keeps gate[e]; up lane sends up[e] and keeps up[e + kHalf]
          const float other = __shfl_xor_sync(kFull, gate ? acc[e + kHalf] : acc[e], 16);
          const float g = gate ? acc[e] : other;
          const float u = gate ? other : acc[e + kHalf];
          stage[(tok0 + e) * 64 + c] = __float2bfloat16_rn(silu_mul(bf16_round(g), bf16_round(u)));
        }
      } else {
#pragma unroll
        for (int e = 0; e < MP; ++e) stage[e * kTileN + row] = __float2bfloat16_rn(acc[e]);
      }
      epi_bar();
      const int pieces = cols / 8;  // 16-byte pieces per token row
      __nv_bfloat16* ybase = a.y + static_cast<int64_t>(t0) * a.ldy + tile * cols;
      for (int idx = et; idx < mt * pieces; idx += 128) {
        const int t = idx / pieces, pc = idx - t * pieces;
        const uint4 v = *reinterpret_cast<const uint4*>(stage + t * cols + pc * 8);
        __nv_bfloat16* dst = ybase + static_cast<int64_t>(t) * a.ldy + pc * 8;
        if (a.vec16) {
          *reinterpret_cast<uint4*>(dst) = v;
        } else {
          const __nv_bfloat16* e8 = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
          for (int j = 0; j < 8; ++j) dst[j] = e8[j];
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) {
    // a wait that gave up can leave issued copies unconsumed: they land before the CTA exits
    const int issued = *s_issued;
    for (int i = *s_consumed; i < issued; ++i) mbar_wait(&full[i % ST], (i / ST) & 1, a.status);
  }
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, a.tmem_cols);
  }
}

// One CTA per 128 x 128 weight block, two threads per row (64 elements each).
__global__ void __launch_bounds__(256) quantize_weight_blocks_kernel(const __nv_bfloat16* w, int64_t ldw, int kbt,
                                                                     uint8_t* q, int64_t ldq, float* scale) {
  __shared__ float s_max[8];
  const int br = blockIdx.y, bc = blockIdx.x;
  const int r = threadIdx.x >> 1, part = threadIdx.x & 1;
  const __nv_bfloat16* src = w + static_cast<int64_t>(br * 128 + r) * ldw + bc * 128 + part * 64;
  uint4 v[8];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = reinterpret_cast<const uint4*>(src)[j];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v[j]);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(e[i])));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = amax;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, s_max[i]);
  const int e = fp8::weight_block_exponent(amax);
  const float inv = fp8::exp2_int(-e);  // w / 2^e, exactly
  uint8_t* dst = q + static_cast<int64_t>(br * 128 + r) * ldq + bc * 128 + part * 64;
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&v[j]);
    const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&v[j + 1]);
    uint4 out;
    out.x = fp8::e4m3x4(__bfloat162float(e0[0]) * inv, __bfloat162float(e0[1]) * inv, __bfloat162float(e0[2]) * inv,
                        __bfloat162float(e0[3]) * inv);
    out.y = fp8::e4m3x4(__bfloat162float(e0[4]) * inv, __bfloat162float(e0[5]) * inv, __bfloat162float(e0[6]) * inv,
                        __bfloat162float(e0[7]) * inv);
    out.z = fp8::e4m3x4(__bfloat162float(e1[0]) * inv, __bfloat162float(e1[1]) * inv, __bfloat162float(e1[2]) * inv,
                        __bfloat162float(e1[3]) * inv);
    out.w = fp8::e4m3x4(__bfloat162float(e1[4]) * inv, __bfloat162float(e1[5]) * inv, __bfloat162float(e1[6]) * inv,
                        __bfloat162float(e1[7]) * inv);
    reinterpret_cast<uint4*>(dst)[j / 2] = out;
  }
  if (threadIdx.x == 0) scale[static_cast<int64_t>(br) * kbt + bc] = fp8::exp2_int(e);
}

// One warp per (token, 128-element block); lane l holds elements 4l .. 4l + 3.
__global__ void __launch_bounds__(256) quantize_rows_kernel(const __nv_bfloat16* x, int64_t ldx, int m, int kbt,
                                                            uint8_t* q, int64_t ldq, float* scale, int64_t ld_scale) {
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (gw >= static_cast<int64_t>(m) * kbt) return;
  const int lane = threadIdx.x & 31;
  const int row = static_cast<int>(gw / kbt), b = static_cast<int>(gw % kbt);
  const uint2 raw = *reinterpret_cast<const uint2*>(x + static_cast<int64_t>(row) * ldx + b * 128 + lane * 4);
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __bfloat162float(e[i]);
    amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = warp_max(amax);
  const float f = fp8::act_block_factor(amax);
  *reinterpret_cast<uint32_t*>(q + static_cast<int64_t>(row) * ldq + b * 128 + lane * 4) =
      fp8::e4m3x4(v[0] * f, v[1] * f, v[2] * f, v[3] * f);
  if (lane == 0) scale[static_cast<int64_t>(b) * ld_scale + row] = __fdiv_rn(1.f, f);
}

// One 16-byte chunk per thread: chunk (tile, kb, r, c) of the packed layout.
__global__ void pack_fp8_kernel(const uint8_t* q, int64_t ldq, int n, int k, int interleave, uint8_t* out) {
  const int kbt = k / kBlockK;
  const int64_t total = static_cast<int64_t>(n / kTileN) * kbt * kTileN * 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i & 7);
    const int r = static_cast<int>((i >> 3) % kTileN);
    const int64_t tkb = (i >> 3) / kTileN;  // tile * kbt + kb
    const int kb = static_cast<int>(tkb % kbt);
    const int tile = static_cast<int>(tkb / kbt);
    int64_t src_row = static_cast<int64_t>(tile) * kTileN + r;
    if (interleave) {  // 32-row groups [gate 16 | up 16]: tile row r, group r / 32, lane r % 32
      const int grp = r >> 5, l = r & 31;
      src_row = (l < 16 ? 0 : n / 2) + tile * 64 + grp * 16 + (l & 15);
    }
    const uint4 v = *reinterpret_cast<const uint4*>(q + src_row * ldq + kb * kBlockK + c * 16);
    *reinterpret_cast<uint4*>(out + (tkb * kTileN + r) * kBlockK + ((c ^ (r & 7)) * 16)) = v;
  }
}

template <int MP, int MINB>
void set_smem_attr() {
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(gemm_fp8_kernel<MP, MINB>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
  });
}

template <int MP, int MINB>
cudaError_t launch_fp8(dim3 grid, int smem, cudaStream_t stream, const CUtensorMap& xmap, const Fp8Args& a) {
  set_smem_attr<MP, MINB>();
  return launch_pdl(gemm_fp8_kernel<MP, MINB>, grid, dim3(kThreads, 1, 1), smem, stream, xmap, a);
}

bool aligned(const void* p, uintptr_t to) { return (reinterpret_cast<uintptr_t>(p) & (to - 1)) == 0; }

// Launch shape of one call: token chunk, K split, pipeline and TMEM sizes, workspace.
struct Plan {
  int mp, chunks, tiles, kbt, S, units, group, stages, bufs, smem;
  bool pair;
  uint32_t tmem_cols;
  int64_t ticket_bytes, workspace_bytes;
};

int plan_fp8(int m, int n, int k, int split, Plan* pl) {
  if (m < 1 || n < kTileN || k < kBlockK) return NQT_ERR_ARG;
  if (n % kTileN != 0 || k % kBlockK != 0) return NQT_ERR_UNSUPPORTED;
  const int want_split = split & 0xff, want_group = (split >> 8) & 0xf;
  if (want_split > kMaxSplit || want_group > kMaxGroup || (split & ~0xfff)) return NQT_ERR_ARG;
  Plan p{};
  p.mp = m <= 32 ? 32 : (m <= 64 ? 64 : 128);
  p.chunks = (m + p.mp - 1) / p.mp;
  p.tiles = n / kTileN;
  p.kbt = k / kBlockK;
  if (p.chunks > 65535 || p.tiles > 0x7fffffff / 8) return NQT_ERR_UNSUPPORTED;
  const int64_t sms = num_sms();
  const int64_t base = static_cast<int64_t>(p.tiles) * p.chunks;
  // the K split that minimises the K blocks the busiest SM streams; a split costs one block more (the
  // partial's round trip through L2); two CTAs share an SM only at <= 64 tokens (register budget)
  int S = want_split;
  if (S == 0) {
    int64_t best = -1;
    for (int cand = 1; cand <= kMaxSplit && cand <= p.kbt; ++cand) {
      const int64_t ctas = base * cand;
      const int64_t per_sm = (ctas + sms - 1) / sms;
      if (cand > 1 && (per_sm > (p.mp <= 64 ? 2 : 1))) break;
      const int64_t cost = per_sm * ((p.kbt + cand - 1) / cand) + (cand > 1 ? 1 : 0);
      if (best < 0 || cost < best) {
        best = cost;
        S = cand;
      }
    }
  }
  if (S > p.kbt) S = p.kbt;
  p.S = S;
  p.units = (p.kbt + S - 1) / S;
  p.pair = base * S > sms && p.mp <= 64;
  // TMEM: one mp-column accumulator per K block in flight (up to 8, at least 2)
  int bufs = p.units < kMaxBufs ? p.units : kMaxBufs;
  if (bufs < 2) bufs = 2;
  p.tmem_cols = 32;
  while (p.tmem_cols < static_cast<uint32_t>(bufs * p.mp) && p.tmem_cols < (p.pair ? 256u : 512u)) p.tmem_cols <<= 1;
  p.bufs = static_cast<int>(p.tmem_cols) / p.mp < kMaxBufs ? static_cast<int>(p.tmem_cols) / p.mp : kMaxBufs;
  if (p.bufs < 1) return NQT_ERR_UNSUPPORTED;
  const int budget = p.pair ? kPairBudget : kSmemBudget;
  p.group = want_group ? want_group : (p.units > 8 ? 2 : 1);
  if (p.group > p.units) p.group = p.units;
  const int loads = (p.units + p.group - 1) / p.group;
  p.stages = loads < kMaxStages ? loads : kMaxStages;
  while (p.stages > 1 && smem_bytes(p.mp, p.group, p.stages, p.units, p.bufs) > budget) --p.stages;
  p.smem = smem_bytes(p.mp, p.group, p.stages, p.units, p.bufs);
  const int floor = tmem_smem_floor(static_cast<int>(p.tmem_cols));
  if (p.smem < floor) p.smem = floor;
  if (p.smem > budget) return NQT_ERR_UNSUPPORTED;
  p.ticket_bytes = S > 1 ? (2 * base * 4 + 255) / 256 * 256 : 0;  // tickets, then the written counters
  p.workspace_bytes = S > 1 ? p.ticket_bytes + base * S * p.mp * kTileN * 4 : 0;
  *pl = p;
  return NQT_OK;
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_fp8_quantize_weight_blocks(const void* w, int64_t ldw, int n, int k, void* q, int64_t ldq,
                                              float* scale, void* stream) {
  if (!w || !q || !scale || n < 128 || k < 128 || n % 128 || k % 128 || ldw < k || ldq < k) return NQT_ERR_ARG;
  if (!aligned(w, 16) || !aligned(q, 16) || (ldw * 2) % 16 || ldq % 16) return NQT_ERR_ARG;
  if (n / 128 > 65535) return NQT_ERR_UNSUPPORTED;
  quantize_weight_blocks_kernel<<<dim3(k / 128, n / 128), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), ldw, k / 128, static_cast<uint8_t*>(q), ldq, scale);
  return check_launch("fp8_quantize_weight_blocks");
}

extern "C" int nqt_fp8_quantize_rows(const void* x, int64_t ldx, int m, int k, void* q, int64_t ldq, float* scale,
                                     int64_t ld_scale, void* stream) {
  if (!x || !q || !scale || m < 0 || k < 128 || k % 128 || ldx < k || ldq < k || ld_scale < m) return NQT_ERR_ARG;
  if (!aligned(x, 8) || !aligned(q, 4) || ldx % 4 || ldq % 4) return NQT_ERR_ARG;
  if (m == 0) return NQT_OK;
  const int64_t warps = static_cast<int64_t>(m) * (k / 128);
  const int64_t blocks = (warps + 7) / 8;
  if (blocks > 0x7fffffff) return NQT_ERR_UNSUPPORTED;
  quantize_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, m, k / 128, static_cast<uint8_t*>(q), ldq, scale, ld_scale);
  return check_launch("fp8_quantize_rows");
}

extern "C" int nqt_gemm_fp8_pack_weight(const void* q, int64_t ldq, int n, int k, int interleave_gate_up,
                                        void* packed, void* stream) {
  if (!q || !packed || n < kTileN || k < kBlockK || n % kTileN || k % kBlockK || ldq < k) return NQT_ERR_ARG;
  if (interleave_gate_up && n % (2 * kTileN)) return NQT_ERR_ARG;
  if (!aligned(q, 16) || !aligned(packed, 16) || ldq % 16) return NQT_ERR_ARG;
  const int64_t chunks = static_cast<int64_t>(n) * k / 16;
  const int grid = static_cast<int>((chunks + 255) / 256 < 65535 ? (chunks + 255) / 256 : 65535);
  pack_fp8_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const uint8_t*>(q), ldq, n, k, interleave_gate_up,
                                                       static_cast<uint8_t*>(packed));
  return check_launch("gemm_fp8_pack_weight");
}

extern "C" int nqt_gemm_fp8_workspace_bytes(int m, int n, int k, int split, int64_t* bytes) {
  if (!bytes) return NQT_ERR_ARG;
  Plan p;
  const int rc = plan_fp8(m, n, k, split, &p);
  if (rc != NQT_OK) return rc;
  *bytes = p.workspace_bytes;
  return NQT_OK;
}

extern "C" int nqt_gemm_fp8(const void* xq, int64_t ldxq, const float* xscale, int64_t ld_xscale,
                            const void* wpacked, const float* wscale, void* y, int64_t ldy, int m, int n, int k,
                            int epilogue, int interleave_gate_up, int split, void* workspace,
                            int64_t workspace_bytes, int32_t* status, void* stream) {
  if (!xq || !xscale || !wpacked || !wscale || !y) return NQT_ERR_ARG;
  if (epilogue != kPlain && epilogue != kSiluMul) return NQT_ERR_ARG;
  if (epilogue == kSiluMul && !interleave_gate_up) return NQT_ERR_ARG;
  if (interleave_gate_up && n % (2 * kTileN)) return NQT_ERR_ARG;
  Plan p;
  const int rc = plan_fp8(m, n, k, split, &p);
  if (rc != NQT_OK) return rc;
  // TMA / bulk copies: 16-byte aligned bases and row pitches
  if (!aligned(xq, 16) || !aligned(wpacked, 16) || ldxq % 16 || ldxq < k || ld_xscale < m || !aligned(xscale, 4))
    return NQT_ERR_ARG;
  const int out_cols = epilogue == kSiluMul ? n / 2 : n;
  if (ldy < out_cols) return NQT_ERR_ARG;
  if (p.workspace_bytes > 0 && (!workspace || workspace_bytes < p.workspace_bytes || !aligned(workspace, 256)))
    return NQT_ERR_ARG;

  CUtensorMap xmap;
  if (encode_x_slabs(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xq, m, p.kbt, ldxq, p.mp, p.group) != NQT_OK) {
    set_last_message("gemm_fp8: cuTensorMapEncodeTiled failed");
    return NQT_ERR_CUDA;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  Fp8Args a{static_cast<const uint8_t*>(wpacked),
            wscale,
            xscale,
            ld_xscale,
            static_cast<__nv_bfloat16*>(y),
            ldy,
            p.S > 1 ? reinterpret_cast<float*>(ws + p.ticket_bytes) : nullptr,
            p.S > 1 ? reinterpret_cast<int32_t*>(ws) : nullptr,
            status,
            m,
            n,
            p.kbt,
            epilogue,
            interleave_gate_up ? 1 : 0,
            p.stages,
            p.group,
            p.bufs,
            p.tmem_cols,
            aligned(y, 16) && ldy % 8 == 0 ? 1 : 0};
  const dim3 grid(p.tiles, p.S, p.chunks);
  cudaError_t err;
  if (p.mp == 32)
    err = p.pair ? launch_fp8<32, 2>(grid, p.smem, as_stream(stream), xmap, a)
                 : launch_fp8<32, 1>(grid, p.smem, as_stream(stream), xmap, a);
  else if (p.mp == 64)
    err = p.pair ? launch_fp8<64, 2>(grid, p.smem, as_stream(stream), xmap, a)
                 : launch_fp8<64, 1>(grid, p.smem, as_stream(stream), xmap, a);
  else
    err = launch_fp8<128, 1>(grid, p.smem, as_stream(stream), xmap, a);
  if (err != cudaSuccess) {
    set_last_error("gemm_fp8", err);
    return NQT_ERR_CUDA;
  }
  return NQT_OK;
}
