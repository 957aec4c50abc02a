// Paged GQA decode attention for sm_100a: balanced split-KV, TMA page
// gathers, online softmax, LSE merge.
//
// Work split.  For one KV-head group the batch's KV is a flat list of
// 16-token tiles (sequence-major).  nqt_decode_plan writes the per-sequence
// tile prefix sum on the device.  The decode launch has N persistent CTAs
// per head group; CTA c streams tiles [T*c/N, T*(c+1)/N), crossing
// sequence boundaries, so every CTA moves the same number of bytes whatever
// the ragged lengths are.  A sequence covered by one CTA is written
// straight to `out`; otherwise each covering CTA leaves a normalised
// partial (O, lse) in slot 2c (its first segment) or 2c+1 (its last) and
// counts itself in on a per-(sequence, KV head) ticket; the consumer warp
// that arrives last combines the partials of its query heads and writes
// `out` (stream-K style fix-up), so no second kernel and no grid-wide wait
// stand between the last tile and the output.  No CTA waits on another.
//
// Data path.  The layer view [pages, 2, P, Hkv, D] is described by a 4-D
// tensor map {D, Hkv, P, pages*2}.  One TMA box {64, 1, 16, 2} brings
// K and V of 16 tokens x 64 dims of one KV head (4 KB) into shared memory
// with the 128-byte swizzle, so the ldmatrix reads of a head's 16 token
// rows are bank-conflict free.  A producer warp keeps STAGES tiles in
// flight through full/empty mbarriers; each consumer warp owns one KV head
// and computes S^T = K Q^T and O^T += V^T P^T with m16n8k16 tensor-core
// tiles (the GQA group's query heads are the N columns), keeping m, l and
// O in registers.
//
// Reference: BatchDecodeWithPagedKVCacheWrapper.plan/run as bound at
// executor/talker_kv.py:229-306 (FlashInfer 0.6.16): out[b, h] =
// softmax(q[b,h] . K[b, :, h/G]^T * sm_scale) V[b, :, h/G] over the
// (n_pages - 1) * P + last_page_len tokens of row b.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace nqt {
namespace {

constexpr int kTok = 16;           // tokens per TMA tile
constexpr int kBoxBytes = 4096;    // [kind 2][tok 16][64 dims] bf16
constexpr int kMaxSplitCtas = 640; // per head group
constexpr int kHeaderBytes = 256;

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct WsLayout {
  size_t tile_indptr;  // i32 [batch_cap + 1]
  size_t tickets;      // i32 [batch_cap * hq]: arrivals per (sequence, KV head), zero between launches
  size_t part_lse;     // f32 [2 * kMaxSplitCtas * hq]
  size_t part_o;       // f32 [2 * kMaxSplitCtas * hq * D]
  size_t total;
};

constexpr WsLayout ws_layout(int batch_cap, int hq, int d, int max_ctas = kMaxSplitCtas) {
  WsLayout w{};
  w.tile_indptr = kHeaderBytes;
  w.tickets = align_up(w.tile_indptr + 4 * static_cast<size_t>(batch_cap + 1), 256);
  w.part_lse = align_up(w.tickets + 4 * static_cast<size_t>(batch_cap) * hq, 256);
  w.part_o = align_up(w.part_lse + 4 * static_cast<size_t>(2 * max_ctas) * hq, 256);
  w.total = align_up(w.part_o + 4 * static_cast<size_t>(2 * max_ctas) * hq * d, 256);
  return w;
}

struct DecodeArgs {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  const int32_t* indptr;
  const int32_t* indices;
  const int32_t* last_len;
  const int32_t* tile_indptr;  // workspace
  const int32_t* header;       // workspace: [0] = total tiles
  int32_t* tickets;            // workspace: [batch][hq], entry b * hq + kv head
  float* part_lse;
  float* part_o;
  int32_t* status;
  int batch, hq, hkv, group, page_size, total_pages, n_ctas;
  int early;  // NQT_DECODE_OVERLAP_KV_WRITE: read the plan and older tiles before the dependency wait
  float scale_log2;
  uint64_t wait_ns;  // limit of the pipeline's mbarrier waits (kWaitLimitNs unless NQT_DECODE_SHORT_WAIT)
};

// ------------------------------------------------------------------ plan
// Single CTA: tiles_b = (n_pages_b - 1) * P/16 + ceil(last_len_b / 16),
// exclusive prefix sum into tile_indptr, total into header[0]; the fix-up
// tickets start at zero (the warp that completes a ticket zeroes it again
// for the next launch on this plan).
__global__ void __launch_bounds__(1024) decode_plan_kernel(const int32_t* indptr, const int32_t* last_len,
                                                           int batch, int page_size, int32_t* header,
                                                           int32_t* tile_indptr, int32_t* tickets,
                                                           int n_tickets) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry_s;
  const int tpp = page_size / kTok;
  for (int i = threadIdx.x; i < n_tickets; i += blockDim.x) tickets[i] = 0;
  if (threadIdx.x == 0) carry_s = 0;
  __syncthreads();
  for (int start = 0; start < batch; start += blockDim.x) {
    const int b = start + threadIdx.x;
    int tiles = 0;
    if (b < batch) {
      const int n = indptr[b + 1] - indptr[b];
      if (n > 0) {
        int ll = last_len[b];
        ll = ll < 1 ? 1 : (ll > page_size ? page_size : ll);
        tiles = (n - 1) * tpp + (ll + kTok - 1) / kTok;
      }
    }
    // block exclusive scan
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int v = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += y;
      }
      if (lane < nw) warp_tot[lane] = v;  // inclusive over warps
    }
    __syncthreads();
    const int carry = carry_s;
    const int excl = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + incl - tiles;
    if (b < batch) tile_indptr[b] = excl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry_s = excl + tiles;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    tile_indptr[batch] = carry_s;
    header[0] = carry_s;
  }
}

// ------------------------------------------------------------------ decode
// 4-D tiled TMA load with an L2 cache policy (the K/V stream is read once per launch: evict first, so it
// does not push q, the page table and the partials out of L2).
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}
__device__ __forceinline__ int64_t range_start(int64_t total, int c, int n) { return total * c / n; }

// Sequence that owns flat tile t: last b with tile_indptr[b] <= t.
__device__ __forceinline__ int find_seq(const int32_t* tile_indptr, int batch, int64_t t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_indptr[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// CTA owning flat tile t when `total` tiles are split over n CTAs: max c with total * c / n <= t.
__device__ __forceinline__ int owner_cta(int64_t total, int n, int64_t t) {
  return static_cast<int>(((t + 1) * n + total - 1) / total) - 1;
}

__device__ __forceinline__ int atomic_add_acq_rel_gpu(int32_t* addr, int32_t v) {
  int32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// Fix-up of one split sequence, run by the consumer warp that completed its ticket: combines the
// partials of query heads [kvh * G, kvh * G + G) from the covering CTAs c0..c1 and writes them to
// out.  Contributor i (CTA c0 + i) left its normalised O and its log2-sum-exp in slot 2(c0+i) when
// the sequence starts inside its range, else 2(c0+i)+1.  out = sum_i w_i O_i / sum_i w_i with
// w_i = 2^(lse_i - max lse), folded online so one pass over the contributors suffices.  Lane l
// owns the R float4 columns f = l + 32 r of the group's G * D/4; the partials are read from L2
// (.cg) in batches of 8 / R contributors, lse and O of a batch issued together.
template <int D, int R>
__device__ __forceinline__ void fixup_sequence(const DecodeArgs& p, int seq, int kvh, int64_t total, int n, int c0,
                                               int c1, int64_t tb0, int lane) {
  constexpr int QD = D / 4;  // float4 per head
  constexpr int kPerBatch = 8 / R;
  const int cols = p.group * QD;  // float4 columns of the group, <= 32 R
  const int head0 = kvh * p.group;
  const float NEG_INF = -__int_as_float(0x7f800000);
  float m[R], sum[R];
  float4 acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = NEG_INF;
    sum[r] = 0.f;
    acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int cb = c0; cb <= c1; cb += kPerBatch) {
    float lse[kPerBatch][R];
    float4 v[kPerBatch][R];
#pragma unroll
    for (int k = 0; k < kPerBatch; ++k) {
      const int cc = cb + k;
      const int slot = range_start(total, cc, n) >= tb0 ? 2 * cc : 2 * cc + 1;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int f = lane + 32 * r;
        if (cc <= c1 && f < cols) {
          const int64_t row = static_cast<int64_t>(slot) * p.hq + head0 + f / QD;
          lse[k][r] = __ldcg(p.part_lse + row);
          v[k][r] = __ldcg(reinterpret_cast<const float4*>(p.part_o + row * D) + f % QD);
        } else {
          lse[k][r] = NEG_INF;
          v[k][r] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kPerBatch; ++k) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (lse[k][r] == NEG_INF) continue;  // past c1 or past the group's columns
        const float nm = fmaxf(m[r], lse[k][r]);
        const float scale = exp2f(m[r] - nm);
        const float w = exp2f(lse[k][r] - nm);
        sum[r] = sum[r] * scale + w;
        acc[r].x = acc[r].x * scale + w * v[k][r].x;
        acc[r].y = acc[r].y * scale + w * v[k][r].y;
        acc[r].z = acc[r].z * scale + w * v[k][r].z;
        acc[r].w = acc[r].w * scale + w * v[k][r].w;
        m[r] = nm;
      }
    }
  }
  __nv_bfloat16* ob = p.out + seq * p.o_st;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int f = lane + 32 * r;
    if (f >= cols) continue;
    const float inv = 1.f / sum[r];
    __nv_bfloat16* dst = ob + static_cast<int64_t>(head0 + f / QD) * p.o_sh + (f % QD) * 4;
    *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(acc[r].x * inv, acc[r].y * inv);
    *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(acc[r].z * inv, acc[r].w * inv);
  }
}

// Count a split segment this warp gave up on in on its ticket (see the abandon path in decode_kernel).
__device__ __forceinline__ void abandon_ticket(const DecodeArgs& p, int64_t total, int n, int64_t t_begin,
                                               int64_t t_end, int seq, int seq_t0, int seq_t1, int kvh, int lane) {
  if (t_begin <= seq_t0 && t_end >= seq_t1) return;  // a whole sequence has no ticket
  const int c0 = owner_cta(total, n, seq_t0);
  const int c1 = owner_cta(total, n, seq_t1 - 1);
  int32_t* ticket = p.tickets + static_cast<int64_t>(seq) * p.hq + kvh;
  int arrived = 0;
  if (lane == 0) arrived = atomic_add_acq_rel_gpu(ticket, 1);
  arrived = __shfl_sync(kFull, arrived, 0);
  if (arrived == c1 - c0 && lane == 0) *ticket = 0;
}

// Last step of every warp of a decode CTA.  When a wait gave up, TMA copies of tiles that were issued
// but not consumed may still be landing in this CTA's shared memory; one thread waits for them (with
// the full limit) before the CTA exits, so no copy completes into memory the CTA has given back.
template <int STAGES>
__device__ __forceinline__ void drain_and_exit(uint64_t* full, const int& s_issued, const int* s_progress,
                                               int consumers, int n_tiles, int32_t* status) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  int lo = n_tiles;
  for (int w = 0; w < consumers; ++w) lo = s_progress[w] < lo ? s_progress[w] : lo;
  // a tile j in [lo, issued) is not consumed by every warp, so tile j + STAGES was never issued and
  // the parity of phase j / STAGES identifies tile j's copy
  for (int j = lo; j < s_issued; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1, status);
}

constexpr int kSmemPrefix = 1024;  // tile_indptr entries staged in shared memory (batch + 1 <= this)
constexpr int kSmemPages = 1024;   // page ids of one CTA's tile range staged in shared memory

template <int D, int HPC, int STAGES>
struct DecodeCfg {
  static constexpr int kHalves = D / 64;
  static constexpr int kStageBytes = HPC * kHalves * kBoxBytes;
  static constexpr int kThreads = (HPC + 1) * 32;
  static constexpr int kSmem = STAGES * kStageBytes + 1024 + 2 * STAGES * 8 + 4 * kSmemPrefix + 4 * kSmemPages;
};

template <int D, int HPC, int STAGES>
__global__ void __launch_bounds__((HPC + 1) * 32) decode_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                DecodeArgs p) {
  using Cfg = DecodeCfg<D, HPC, STAGES>;
  constexpr int kHalves = Cfg::kHalves;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::kStageBytes);
  uint64_t* empty = full + STAGES;
  int32_t* s_prefix = reinterpret_cast<int32_t*>(empty + STAGES);
  int32_t* s_pages = s_prefix + kSmemPrefix;
  // tiles the producer issued and, per consumer warp, the first tile it did not consume: after a wait
  // gave up, the CTA waits for the copies still in flight before it exits
  __shared__ int s_issued;
  __shared__ int s_progress[HPC];

  // Launched with programmatic serialization; the next kernel may be scheduled as soon as every CTA
  // here has started.  By default everything waits for the previous grid.  With `early` the caller
  // guarantees that the previous grid writes neither the plan, the page table nor any KV tile but each
  // row's last: those are read before the wait (page-id staging and the first TMA loads overlap the
  // previous kernel), while q, each row's last tile and every write here come after it.
  if (!p.early) grid_dependency_wait();
  grid_dependents_launch();
  const int c = blockIdx.x;
  const int kv0 = blockIdx.y * HPC;
  const int64_t total = p.header[0];
  // rows with no pages get a defined output of zeros (this CTA's heads of rows c, c + n_ctas, ...)
  for (int b = c; b < p.batch; b += p.n_ctas) {
    if (p.tile_indptr[b + 1] == p.tile_indptr[b]) {
      if (p.early) grid_dependency_wait();
      const int h0 = kv0 * p.group;
      for (int i = threadIdx.x; i < HPC * p.group * D; i += blockDim.x)
        p.out[b * p.o_st + static_cast<int64_t>(h0 + i / D) * p.o_sh + i % D] = __float2bfloat16_rn(0.f);
    }
  }
  // fewer tiles than CTAs: one tile each and the rest idle, so every range is non-empty and the
  // CTAs covering a sequence are exactly c0..c1 of its first and last tiles
  const int n = total < p.n_ctas ? static_cast<int>(total) : p.n_ctas;
  if (c >= n) return;  // uniform over the block
  const int64_t t_begin = range_start(total, c, n);
  const int64_t t_end = range_start(total, c + 1, n);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tpp = p.page_size / kTok;
  const int n_tiles = static_cast<int>(t_end - t_begin);

  // one parallel load of the per-sequence tile prefix instead of a chain of dependent loads
  const bool staged = p.batch + 1 <= kSmemPrefix;
  if (staged)
    for (int b = threadIdx.x; b <= p.batch; b += blockDim.x) s_prefix[b] = p.tile_indptr[b];
  const int32_t* prefix = staged ? s_prefix : p.tile_indptr;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HPC);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == HPC) {
    // ---------------------------------------------------------- producer
    // The range's tiles cover one contiguous window of kv_indices (sequences in order, pages in
    // order): load it once with all 32 lanes so the TMA issue loop never waits on a page-id load.
    const int seq_a = find_seq(prefix, p.batch, t_begin);
    const int seq_b = find_seq(prefix, p.batch, t_end - 1);
    const int win0 = p.indptr[seq_a] + static_cast<int>(t_begin - prefix[seq_a]) / tpp;
    const int win1 = p.indptr[seq_b] + static_cast<int>(t_end - 1 - prefix[seq_b]) / tpp + 1;
    const bool windowed = win1 - win0 <= kSmemPages;
    if (windowed)
      for (int i = lane; i < win1 - win0; i += 32) s_pages[i] = p.indices[win0 + i];
    __syncwarp();
    if (lane == 0) prefetch_tensormap(&tmap);
    // Lane l issues box l of each stage (KV head l / kHalves, dims half l % kHalves): one thread
    // issuing every box serialises on the per-instruction TMA issue cost.
    const int box_h = lane / kHalves, box_half = lane % kHalves;
    uint64_t evict_first;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(evict_first));
    int seq = seq_a;
    int seq_t0 = prefix[seq];
    int seq_t1 = prefix[seq + 1];
    int seq_base = p.indptr[seq];
    bool dependency_met = !p.early;
    int issued = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int64_t t = t_begin + i;
      while (t >= seq_t1) {  // advance to the owning sequence (skips empty rows)
        ++seq;
        seq_t0 = seq_t1;
        seq_t1 = prefix[seq + 1];
        seq_base = p.indptr[seq];
      }
      if (!dependency_met && t == seq_t1 - 1) {  // a row's last tile may come from the previous grid
        grid_dependency_wait();
        dependency_met = true;
      }
      const int s = i % STAGES;
      // warp-uniform decision: every lane reaches the same __syncwarp
      const bool ready = i < STAGES || mbar_wait_ns(&empty[s], ((i / STAGES) - 1) & 1, p.status, p.wait_ns);
      if (!__all_sync(kFull, ready)) break;
      const int in_seq = static_cast<int>(t - seq_t0);
      const int page_local = in_seq / tpp;
      const int tile_in_page = in_seq - page_local * tpp;
      const int pos = seq_base + page_local;
      int page = windowed ? s_pages[pos - win0] : p.indices[pos];
      if (static_cast<unsigned>(page) >= static_cast<unsigned>(p.total_pages)) {
        if (lane == 0) report(p.status, NQT_DEV_BAD_PAGE);
        page = p.total_pages;  // a box entirely outside the map: TMA fills zeros
      }
      if (lane == 0) mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
      __syncwarp();
      if (lane < HPC * kHalves)
        tma_load_4d_hint(smem + s * Cfg::kStageBytes + (box_h * kHalves + box_half) * kBoxBytes, &tmap, &full[s],
                         box_half * 64, kv0 + box_h, tile_in_page * kTok, page * 2, evict_first);
      issued = i + 1;
    }
    if (lane == 0) s_issued = issued;
    drain_and_exit<STAGES>(full, s_issued, s_progress, HPC, n_tiles, p.status);
    return;
  }

  // ------------------------------------------------------------ consumers
  const int kvh = kv0 + warp;
  const int g = lane >> 2;
  const int t4 = lane & 3;
  const int group = p.group;
  const float NEG_INF = -__int_as_float(0x7f800000);

  uint32_t qf[D / 16][2];
  float o[D / 16][4];
  float m0 = NEG_INF, m1 = NEG_INF, l0 = 0.f, l1 = 0.f;

  int seq = find_seq(prefix, p.batch, t_begin);
  int seq_t0 = prefix[seq];
  int seq_t1 = prefix[seq + 1];
  bool seg_open = false;
  int fix_a = -1, fix_b = -1;  // split sequences whose ticket this warp completed
  int stop = n_tiles;          // first tile this warp did not consume (n_tiles unless a wait gave up)

  // ldmatrix lane roles
  const int lm_j = lane >> 3;
  const int lm_r = lane & 7;

  if (p.early) grid_dependency_wait();  // q, and the partials and tickets of the previous launch
  for (int i = 0; i < n_tiles; ++i) {
    const int64_t t = t_begin + i;
    while (t >= seq_t1) {
      ++seq;
      seq_t0 = seq_t1;
      seq_t1 = prefix[seq + 1];
    }
    if (!seg_open) {
      // new segment: load this sequence's query heads of the group as B fragments
      const int qhead = kvh * group + g;
      const __nv_bfloat16* qrow = p.q + seq * p.q_st + static_cast<int64_t>(qhead) * p.q_sh;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        if (g < group) {
          qf[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t4);
          qf[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t4 + 8);
        } else {
          qf[kk][0] = 0u;
          qf[kk][1] = 0u;
        }
      }
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      m0 = m1 = NEG_INF;
      l0 = l1 = 0.f;
      seg_open = true;
    }
    const bool last_tile_of_seq = (t == seq_t1 - 1);
    int valid = kTok;
    if (last_tile_of_seq) {
      int ll = p.last_len[seq];
      ll = ll < 1 ? 1 : (ll > p.page_size ? p.page_size : ll);
      valid = ll - ((ll - 1) / kTok) * kTok;
    }

    const int s = i % STAGES;
    if (!__all_sync(kFull, mbar_wait_ns(&full[s], (i / STAGES) & 1, p.status, p.wait_ns))) {
      stop = i;
      break;
    }
    uint8_t* head_box = smem + s * Cfg::kStageBytes + warp * kHalves * kBoxBytes;

    if (valid < kTok) {
      // zero the V rows past the sequence end so 0 * stale never meets a NaN
      const int rows = kTok - valid;
      for (int idx = lane; idx < rows * 8 * kHalves; idx += 32) {
        const int half = idx / (rows * 8);
        const int rem = idx - half * rows * 8;
        const int row = valid + rem / 8;
        const int chunk = rem & 7;
        *reinterpret_cast<uint4*>(head_box + half * kBoxBytes + 2048 + row * 128 + chunk * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      __syncwarp();
    }

    // S^T[tok][n] = sum_d K[tok][d] Q[n][d]
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int half = kk >> 2;
      const int chunk = ((kk & 3) << 1) + (lm_j >> 1);
      const int tok = ((lm_j & 1) << 3) + lm_r;
      const uint32_t addr = smem_addr(head_box + half * kBoxBytes) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(a0, a1, a2, a3, addr);
      mma_bf16_16816(sc, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
    }

    // online softmax (log2 domain); lane holds heads 2*t4 (c0,c2) and 2*t4+1 (c1,c3)
    const bool lo_ok = g < valid;
    const bool hi_ok = g + 8 < valid;
    const float s0 = lo_ok ? sc[0] * p.scale_log2 : NEG_INF;
    const float s1 = lo_ok ? sc[1] * p.scale_log2 : NEG_INF;
    const float s2 = hi_ok ? sc[2] * p.scale_log2 : NEG_INF;
    const float s3 = hi_ok ? sc[3] * p.scale_log2 : NEG_INF;
    float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, off));
    }
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float al0 = exp2f(m0 - nm0), al1 = exp2f(m1 - nm1);
    const float p0 = exp2f(s0 - nm0), p1 = exp2f(s1 - nm1);
    const float p2 = exp2f(s2 - nm0), p3 = exp2f(s3 - nm1);
    l0 = l0 * al0 + p0 + p2;
    l1 = l1 * al1 + p1 + p3;
    m0 = nm0;
    m1 = nm1;
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      o[mt][0] *= al0;
      o[mt][1] *= al1;
      o[mt][2] *= al0;
      o[mt][3] *= al1;
    }

    // P^T as the B operand: lane (g, t4) needs P[head g][tok 2t4, 2t4+1, 2t4+8, 2t4+9]
    const uint32_t pack_a = pack_bf16x2(p0, p2);  // head 2*t4: tok g (lo), tok g+8 (hi)
    const uint32_t pack_b = pack_bf16x2(p1, p3);  // head 2*t4+1
    const int src1 = (2 * t4) * 4 + (g >> 1);
    const int src2 = (2 * t4 + 1) * 4 + (g >> 1);
    const uint32_t x1a = __shfl_sync(kFull, pack_a, src1);
    const uint32_t x1b = __shfl_sync(kFull, pack_b, src1);
    const uint32_t x2a = __shfl_sync(kFull, pack_a, src2);
    const uint32_t x2b = __shfl_sync(kFull, pack_b, src2);
    const uint32_t x1 = (g & 1) ? x1b : x1a;
    const uint32_t x2 = (g & 1) ? x2b : x2a;
    uint32_t pb0 = __byte_perm(x1, x2, 0x5410);
    uint32_t pb1 = __byte_perm(x1, x2, 0x7632);
    if (g >= group) pb0 = pb1 = 0u;

    // O^T[d][n] += sum_tok V[tok][d] P[n][tok]
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int half = mt >> 2;
      const int chunk = ((mt & 3) << 1) + (lm_j & 1);
      const int tok = ((lm_j >> 1) << 3) + lm_r;
      const uint32_t addr =
          smem_addr(head_box + half * kBoxBytes + 2048) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4_trans(a0, a1, a2, a3, addr);
      mma_bf16_16816(o[mt], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool seg_end = last_tile_of_seq || (i == n_tiles - 1);
    if (seg_end) {
      float lt0 = l0, lt1 = l1;
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        lt0 += __shfl_xor_sync(kFull, lt0, off);
        lt1 += __shfl_xor_sync(kFull, lt1, off);
      }
      const float inv0 = 1.f / lt0, inv1 = 1.f / lt1;
      const int ha = kvh * group + 2 * t4;  // query head of columns c0/c2
      const bool whole = (t_begin <= seq_t0) && (t_end >= seq_t1);
      if (whole) {
        __nv_bfloat16* ob = p.out + seq * p.o_st;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          const int d0 = mt * 16 + g;
          if (2 * t4 < group) {
            ob[ha * p.o_sh + d0] = __float2bfloat16_rn(o[mt][0] * inv0);
            ob[ha * p.o_sh + d0 + 8] = __float2bfloat16_rn(o[mt][2] * inv0);
          }
          if (2 * t4 + 1 < group) {
            ob[(ha + 1) * p.o_sh + d0] = __float2bfloat16_rn(o[mt][1] * inv1);
            ob[(ha + 1) * p.o_sh + d0 + 8] = __float2bfloat16_rn(o[mt][3] * inv1);
          }
        }
      } else {
        const int slot = (t_begin >= seq_t0) ? 2 * c : 2 * c + 1;
        float* po = p.part_o + static_cast<int64_t>(slot) * p.hq * D;
        float* pl = p.part_lse + static_cast<int64_t>(slot) * p.hq;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          const int d0 = mt * 16 + g;
          if (2 * t4 < group) {
            po[ha * D + d0] = o[mt][0] * inv0;
            po[ha * D + d0 + 8] = o[mt][2] * inv0;
          }
          if (2 * t4 + 1 < group) {
            po[(ha + 1) * D + d0] = o[mt][1] * inv1;
            po[(ha + 1) * D + d0 + 8] = o[mt][3] * inv1;
          }
        }
        if (g == 0) {
          if (2 * t4 < group) pl[ha] = m0 + log2f(lt0);
          if (2 * t4 + 1 < group) pl[ha + 1] = m1 + log2f(lt1);
        }
        // count this warp in on the (sequence, KV head) ticket: the warp completing it has seen every
        // covering CTA's partial (release by each arriving lane 0 after its warp's stores, acquire by
        // the completing one) and combines them once its own tiles are done
        __syncwarp();
        const int c0 = owner_cta(total, n, seq_t0);
        const int c1 = owner_cta(total, n, seq_t1 - 1);
        int32_t* ticket = p.tickets + static_cast<int64_t>(seq) * p.hq + kvh;
        int arrived = 0;
        if (lane == 0) arrived = atomic_add_acq_rel_gpu(ticket, 1);
        arrived = __shfl_sync(kFull, arrived, 0);
        if (arrived == c1 - c0) {
          if (lane == 0) *ticket = 0;  // ready for the next launch on this plan
          // only a range's first and last segments can be split: at most two fix-ups per warp
          if (fix_a < 0) fix_a = seq; else fix_b = seq;
        }
      }
      seg_open = false;
    }
  }

  if (stop < n_tiles) {
    // A wait gave up (NQT_DEV_TIMEOUT is set and this launch's output is undefined).  The split
    // segments this warp did not finish still count in on their tickets, so every ticket of the
    // launch completes and returns to zero: later launches on the same plan stay correct.  Only a
    // range's first and last segments can be split; the open one is the segment of tile `stop`.
    abandon_ticket(p, total, n, t_begin, t_end, seq, seq_t0, seq_t1, kvh, lane);
    const int last = find_seq(prefix, p.batch, t_end - 1);
    if (last != seq) abandon_ticket(p, total, n, t_begin, t_end, last, prefix[last], prefix[last + 1], kvh, lane);
  }

  // deferred fix-ups: the accumulators are dead here, so the combine does not raise the register
  // footprint of the tile loop
  __syncwarp();
  for (int f = 0; f < 2; ++f) {
    const int fs = f == 0 ? fix_a : fix_b;
    if (fs < 0) continue;
    const int f_t0 = prefix[fs], f_t1 = prefix[fs + 1];
    const int c0 = owner_cta(total, n, f_t0);
    const int c1 = owner_cta(total, n, f_t1 - 1);
    const int cols = group * (D / 4);
    if (cols <= 32)
      fixup_sequence<D, 1>(p, fs, kvh, total, n, c0, c1, f_t0, lane);
    else if (cols <= 64)
      fixup_sequence<D, 2>(p, fs, kvh, total, n, c0, c1, f_t0, lane);
    else if (cols <= 128)
      fixup_sequence<D, 4>(p, fs, kvh, total, n, c0, c1, f_t0, lane);
    else
      fixup_sequence<D, 8>(p, fs, kvh, total, n, c0, c1, f_t0, lane);
  }
  if (lane == 0) s_progress[warp] = stop;
  drain_and_exit<STAGES>(full, s_issued, s_progress, HPC, n_tiles, p.status);
}

// ------------------------------------------------------------------ host
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

int encode_layer_map(CUtensorMap* map, const void* layer, int total_pages, int page_size, int hkv, int d) {
  auto encode = get_encode();
  if (encode == nullptr) return NQT_ERR_CUDA;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(hkv),
                        static_cast<cuuint64_t>(page_size), static_cast<cuuint64_t>(total_pages) * 2};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(hkv) * d * 2,
                           static_cast<cuuint64_t>(page_size) * hkv * d * 2};
  cuuint32_t box[4] = {64, 1, kTok, 2};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(layer), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NQT_OK : NQT_ERR_CUDA;
}

template <int D, int HPC, int STAGES>
int launch_decode(const CUtensorMap& map, DecodeArgs a, int groups, int max_ctas, cudaStream_t s) {
  using Cfg = DecodeCfg<D, HPC, STAGES>;
  static int occ = -1;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(decode_kernel<D, HPC, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    int o = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_kernel<D, HPC, STAGES>, Cfg::kThreads, Cfg::kSmem);
    occ = o > 0 ? o : 1;
  });
  int n = num_sms() * occ / groups;
  if (n < 1) n = 1;
  if (n > max_ctas) n = max_ctas;
  a.n_ctas = n;
  cudaError_t err =
      launch_pdl(decode_kernel<D, HPC, STAGES>, dim3(n, groups), dim3(Cfg::kThreads), Cfg::kSmem, s, map, a);
  if (err != cudaSuccess) {
    set_last_error("decode_attention", err);
    return NQT_ERR_CUDA;
  }
  return NQT_OK;
}

// KV heads per CTA and TMA pipeline depth of the widest configuration (4 heads: 32 KB stages,
// 3 stages -> 2 CTAs per SM).
#ifndef NQT_DECODE_HPC
#define NQT_DECODE_HPC 4
#endif
#ifndef NQT_DECODE_STAGES
#define NQT_DECODE_STAGES 3
#endif

template <int D>
int dispatch_hpc(const CUtensorMap& map, const DecodeArgs& a, int max_ctas, cudaStream_t s) {
  constexpr int H = NQT_DECODE_HPC;
  if (a.hkv % H == 0) return launch_decode<D, H, NQT_DECODE_STAGES>(map, a, a.hkv / H, max_ctas, s);
  if (a.hkv % 2 == 0) return launch_decode<D, 2, 4>(map, a, a.hkv / 2, max_ctas, s);
  return launch_decode<D, 1, 4>(map, a, a.hkv, max_ctas, s);
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" size_t nqt_decode_workspace_bytes(int batch_capacity, int num_qo_heads, int head_dim) {
  if (batch_capacity < 1 || num_qo_heads < 1 || head_dim < 1) return 0;
  return ws_layout(batch_capacity, num_qo_heads, head_dim).total;
}

extern "C" int nqt_decode_plan(const int32_t* kv_indptr, const int32_t* last_page_len, int batch,
                               int batch_capacity, int page_size, int num_qo_heads, int head_dim, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!kv_indptr || !last_page_len || !workspace) return NQT_ERR_ARG;
  if (batch < 1 || batch > batch_capacity || page_size < kTok || page_size % kTok) return NQT_ERR_ARG;
  const WsLayout w = ws_layout(batch_capacity, num_qo_heads, head_dim);
  if (workspace_bytes < w.total) return NQT_ERR_CAPACITY;
  uint8_t* base = static_cast<uint8_t*>(workspace);
  decode_plan_kernel<<<1, 1024, 0, as_stream(stream)>>>(
      kv_indptr, last_page_len, batch, page_size, reinterpret_cast<int32_t*>(base),
      reinterpret_cast<int32_t*>(base + w.tile_indptr), reinterpret_cast<int32_t*>(base + w.tickets),
      batch * num_qo_heads);
  return check_launch("decode_plan");
}

namespace {

// Argument checks shared by the decode entry points.
int check_decode_args(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* layer_cache,
                      int total_pages, int page_size, const int32_t* kv_indptr, const int32_t* kv_indices,
                      const int32_t* last_page_len, const void* out, int64_t out_stride_tok, int64_t out_stride_head,
                      int batch, int num_qo_heads, int num_kv_heads, int head_dim) {
  if (!q || !layer_cache || !kv_indptr || !kv_indices || !last_page_len || !out) return NQT_ERR_ARG;
  if (batch < 1 || total_pages < 1) return NQT_ERR_ARG;
  if (num_kv_heads < 1 || num_qo_heads % num_kv_heads) return NQT_ERR_ARG;
  if (num_qo_heads / num_kv_heads > 8 || num_kv_heads > 256) return NQT_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return NQT_ERR_UNSUPPORTED;
  if (page_size < kTok || page_size % kTok || page_size > 256) return NQT_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(layer_cache) & 15) || (reinterpret_cast<uintptr_t>(q) & 3)) return NQT_ERR_ARG;
  if ((q_stride_tok & 1) || (q_stride_head & 1)) return NQT_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(out) & 3) || (out_stride_tok & 1) || (out_stride_head & 1)) return NQT_ERR_ARG;
  if (static_cast<int64_t>(total_pages) * 2 >= (int64_t(1) << 31)) return NQT_ERR_UNSUPPORTED;
  return NQT_OK;
}

// Attention launch over a plan already written at `base` with layout `w`.
int run_decode(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* layer_cache,
               int total_pages, int page_size, const int32_t* kv_indptr, const int32_t* kv_indices,
               const int32_t* last_page_len, int batch, int num_qo_heads, int num_kv_heads, int head_dim,
               float sm_scale, void* out, int64_t out_stride_tok, int64_t out_stride_head, uint8_t* base,
               const WsLayout& w, int max_ctas, int early, int short_wait, int32_t* status, cudaStream_t s) {
  CUtensorMap map;
  int rc = encode_layer_map(&map, layer_cache, total_pages, page_size, num_kv_heads, head_dim);
  if (rc != NQT_OK) return rc;
  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_stride_tok;
  a.q_sh = q_stride_head;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_st = out_stride_tok;
  a.o_sh = out_stride_head;
  a.indptr = kv_indptr;
  a.indices = kv_indices;
  a.last_len = last_page_len;
  a.tile_indptr = reinterpret_cast<const int32_t*>(base + w.tile_indptr);
  a.header = reinterpret_cast<const int32_t*>(base);
  a.tickets = reinterpret_cast<int32_t*>(base + w.tickets);
  a.part_lse = reinterpret_cast<float*>(base + w.part_lse);
  a.part_o = reinterpret_cast<float*>(base + w.part_o);
  a.status = status;
  a.batch = batch;
  a.hq = num_qo_heads;
  a.hkv = num_kv_heads;
  a.group = num_qo_heads / num_kv_heads;
  a.page_size = page_size;
  a.total_pages = total_pages;
  a.n_ctas = 1;
  a.early = early;
  a.scale_log2 = sm_scale * 1.4426950408889634f;
  a.wait_ns = short_wait ? 0 : kWaitLimitNs;
  return head_dim == 128 ? dispatch_hpc<128>(map, a, max_ctas, s) : dispatch_hpc<64>(map, a, max_ctas, s);
}

}  // namespace

extern "C" int nqt_decode_attention_ex(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                       const void* layer_cache, int total_pages, int page_size,
                                       const int32_t* kv_indptr, const int32_t* kv_indices,
                                       const int32_t* last_page_len, int batch, int batch_capacity,
                                       int num_qo_heads, int num_kv_heads, int head_dim, float sm_scale, void* out,
                                       int64_t out_stride_tok, int64_t out_stride_head, void* workspace,
                                       size_t workspace_bytes, int flags, int32_t* status, void* stream) {
  int rc = check_decode_args(q, q_stride_tok, q_stride_head, layer_cache, total_pages, page_size, kv_indptr,
                             kv_indices, last_page_len, out, out_stride_tok, out_stride_head, batch, num_qo_heads,
                             num_kv_heads, head_dim);
  if (rc != NQT_OK) return rc;
  if (!workspace || batch > batch_capacity) return NQT_ERR_ARG;
  if (flags & ~(NQT_DECODE_OVERLAP_KV_WRITE | NQT_DECODE_SHORT_WAIT)) return NQT_ERR_ARG;
  const WsLayout w = ws_layout(batch_capacity, num_qo_heads, head_dim);
  if (workspace_bytes < w.total) return NQT_ERR_CAPACITY;
  return run_decode(q, q_stride_tok, q_stride_head, layer_cache, total_pages, page_size, kv_indptr, kv_indices,
                    last_page_len, batch, num_qo_heads, num_kv_heads, head_dim, sm_scale, out, out_stride_tok,
                    out_stride_head, static_cast<uint8_t*>(workspace), w, kMaxSplitCtas,
                    (flags & NQT_DECODE_OVERLAP_KV_WRITE) ? 1 : 0, (flags & NQT_DECODE_SHORT_WAIT) ? 1 : 0,
                    status, as_stream(stream));
}

extern "C" int nqt_decode_attention(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                    const void* layer_cache, int total_pages, int page_size,
                                    const int32_t* kv_indptr, const int32_t* kv_indices,
                                    const int32_t* last_page_len, int batch, int batch_capacity, int num_qo_heads,
                                    int num_kv_heads, int head_dim, float sm_scale, void* out,
                                    int64_t out_stride_tok, int64_t out_stride_head, void* workspace,
                                    size_t workspace_bytes, int32_t* status, void* stream) {
  return nqt_decode_attention_ex(q, q_stride_tok, q_stride_head, layer_cache, total_pages, page_size, kv_indptr,
                                 kv_indices, last_page_len, batch, batch_capacity, num_qo_heads, num_kv_heads,
                                 head_dim, sm_scale, out, out_stride_tok, out_stride_head, workspace,
                                 workspace_bytes, 0, status, stream);
}

// ---------------------------------------------------------------------------
// Decode attention with library-owned scratch, for callers that cannot
// allocate device memory.
//
// Some hosts of this library must not call cudaMalloc on the serving path: a
// loader that only hands out pointers to buffers it already owns, a process
// whose allocator is held by another runtime, or code running where an
// allocation could block or fail at the wrong time.  They still need the
// split-KV plan and the per-split partial results somewhere.  This entry
// point keeps them in one fixed array compiled into the library: every GPU
// that loads libnqt holds kNoAllocScratchBytes of it until the process exits.
//
// Host code cannot use the array's name as a device address (on the host
// the name is a stand-in, not the device buffer), so the address is looked
// up once per device with cudaGetSymbolAddress, with that device current,
// on the first call made on it; make that first call before any stream
// capture.  The address stays valid for the life of the device's primary
// context: a caller that resets the device (cudaDeviceReset) must not call
// this entry point on that device again in the same process, because the
// cached address belongs to the destroyed context.  Nothing in the array has to start at zero: each call rewrites
// the plan before the attention kernels read it.  All calls share the
// array, so two calls that can overlap on the GPU (different streams, or
// different threads on one device) race on it; serialise them.
namespace {

constexpr int kNoAllocMaxBatch = 1024;     // rows per call
constexpr int kNoAllocMaxHeads = 32;       // num_qo_heads
constexpr int kNoAllocMaxHeadsDim = 2048;  // num_qo_heads * head_dim
constexpr int kNoAllocMaxCtas = 296;       // split CTAs per KV-head group (2 per SM on 148 SMs)
// the layout grows with num_qo_heads at a fixed num_qo_heads * head_dim, so the widest head count bounds
// every allowed shape (header, tile prefix, tickets, lse, partial O: about 5.1 MB)
constexpr size_t kNoAllocScratchBytes =
    ws_layout(kNoAllocMaxBatch, kNoAllocMaxHeads, kNoAllocMaxHeadsDim / kNoAllocMaxHeads, kNoAllocMaxCtas).total;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    set_last_error("nqt_decode_attention_noalloc: cudaGetDevice", err);
    return NQT_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_last_message("nqt_decode_attention_noalloc: device ordinal beyond the 64 devices this library tracks");
    return NQT_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr) {
      set_last_error("nqt_decode_attention_noalloc: cudaGetSymbolAddress", err);
      return NQT_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_noalloc_ptr[dev]);
  return NQT_OK;
}

}  // namespace

extern "C" size_t nqt_decode_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int nqt_decode_attention_noalloc(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                            const void* layer_cache, int total_pages, int page_size,
                                            const int32_t* kv_indptr, const int32_t* kv_indices,
                                            const int32_t* last_page_len, int batch, int num_qo_heads,
                                            int num_kv_heads, int head_dim, float sm_scale, void* out,
                                            int64_t out_stride_tok, int64_t out_stride_head, int32_t* status,
                                            void* stream) {
  int rc = check_decode_args(q, q_stride_tok, q_stride_head, layer_cache, total_pages, page_size, kv_indptr,
                             kv_indices, last_page_len, out, out_stride_tok, out_stride_head, batch, num_qo_heads,
                             num_kv_heads, head_dim);
  if (rc != NQT_OK) return rc;
  if (batch > kNoAllocMaxBatch || num_qo_heads > kNoAllocMaxHeads || num_qo_heads * head_dim > kNoAllocMaxHeadsDim) {
    set_last_message("nqt_decode_attention_noalloc: shape beyond the fixed scratch (batch <= 1024, "
                     "num_qo_heads <= 32, num_qo_heads * head_dim <= 2048)");
    return NQT_ERR_CAPACITY;
  }
  const WsLayout w = ws_layout(batch, num_qo_heads, head_dim, kNoAllocMaxCtas);
  if (w.total > kNoAllocScratchBytes) return NQT_ERR_CAPACITY;
  uint8_t* base = nullptr;
  rc = noalloc_scratch(&base);
  if (rc != NQT_OK) return rc;
  cudaStream_t s = as_stream(stream);
  decode_plan_kernel<<<1, 1024, 0, s>>>(kv_indptr, last_page_len, batch, page_size, reinterpret_cast<int32_t*>(base),
                                        reinterpret_cast<int32_t*>(base + w.tile_indptr),
                                        reinterpret_cast<int32_t*>(base + w.tickets), batch * num_qo_heads);
  rc = check_launch("nqt_decode_attention_noalloc: plan");
  if (rc != NQT_OK) return rc;
  return run_decode(q, q_stride_tok, q_stride_head, layer_cache, total_pages, page_size, kv_indptr, kv_indices,
                    last_page_len, batch, num_qo_heads, num_kv_heads, head_dim, sm_scale, out, out_stride_tok,
                    out_stride_head, base, w, kNoAllocMaxCtas, 0, 0, status, s);
}
