// Ragged causal prefill attention over paged KV (sm_100a).
//
// CTA = (64 query rows, one KV head).  A query row is a (token, head of the
// GQA group) pair, so one K/V tile feeds every query head that reads it.
// Rows of sequence b are the last qo_len_b positions of its KV: query token
// i sees KV positions <= kv_len_b - qo_len_b + i.
//
// A producer warp streams K/V of 64-token blocks into shared memory with the
// same 4-D tensor map as the decode kernel (one {64 dims, 1 head, 16 tokens,
// K+V} box per page tile, 128-byte swizzle); four consumer warps own 16 rows
// each and run S = Q K^T and O += P V with m16n8k16 tiles, fp32 online
// softmax in registers.
//
// Reference: BatchPrefillWithPagedKVCacheWrapper.plan/run with causal=True
// as bound at executor/talker_kv.py:140-226.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace nqt {
namespace {

constexpr int kTok = 16;
constexpr int kBoxBytes = 4096;
constexpr int kRows = 64;        // query rows per CTA
constexpr int kBlockTok = 64;    // KV tokens per pipeline stage
constexpr int kSub = kBlockTok / kTok;
constexpr int kConsumers = 4;

struct PrefillArgs {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  const int32_t* qo_indptr;
  const int32_t* kv_indptr;
  const int32_t* indices;
  const int32_t* last_len;
  int32_t* status;
  int batch, hq, hkv, group, page_size, total_pages;
  float scale_log2;
  int tma_out;  // tcgen05 path: full query tiles leave through a TMA store (out map valid)
  int out16;    // tcgen05 path: every output row chunk is 16-byte aligned (else 4-byte stores)
};

template <int D, int STAGES>
struct PrefillCfg {
  static constexpr int kHalves = D / 64;
  static constexpr int kStageBytes = kSub * kHalves * kBoxBytes;  // K+V of 64 tokens, one head
  static constexpr int kThreads = (kConsumers + 1) * 32;
  static constexpr int kSmem = STAGES * kStageBytes + 1024 + 2 * STAGES * 8 + 64;
};

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory"); }

// (sequence, query tile) of CTA `cta`, longest first (called by a whole warp; every lane gets the
// result; seq = -1: no tile).  A query tile's cost is the number of 64-key blocks up to its diagonal,
// nb = ceil(e / 64) with e = min(kv_len, shift + (i + 1) * tpt) the key end of tile i (shift = kv_len -
// qo_len), non-decreasing in i.  CTAs take tiles in decreasing nb (ties: batch order, then tile
// order), so the first wave starts the most expensive tiles of every chunk and the cheap ones fill the
// tail.  For one sequence the tiles with nb >= v are its last ge(v) tiles, ge(v) = T - #{i : e_i <=
// 64 (v - 1)}, so the CTA's level v is a binary search over sums of ge and its tile a scan over the batch.
struct SeqTiles {
  int tiles, shift, kv_len;
};

__device__ __forceinline__ SeqTiles seq_tiles(const int32_t* qo_indptr, const int32_t* kv_indptr,
                                              const int32_t* last_len, int page_size, int b, int tpt) {
  SeqTiles t{0, 0, 0};
  const int qo = qo_indptr[b + 1] - qo_indptr[b];
  const int n_pages = kv_indptr[b + 1] - kv_indptr[b];
  if (qo <= 0 || n_pages <= 0) return t;
  int ll = last_len[b];
  ll = ll < 1 ? 1 : (ll > page_size ? page_size : ll);
  t.kv_len = (n_pages - 1) * page_size + ll;
  t.shift = t.kv_len - qo;
  t.tiles = (qo + tpt - 1) / tpt;
  return t;
}

constexpr int kStagedSeqs = 512;  // sequences whose tile geometry the mapping keeps in shared memory

__device__ void longest_first_tile(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* last_len,
                                   int page_size, int batch, int tpt, int cta, int& seq, int& tile) {
  const int lane = threadIdx.x & 31;
  __shared__ SeqTiles s_seq[kStagedSeqs];
  seq = -1;
  tile = 0;
  const bool staged = batch <= kStagedSeqs;
  if (staged) {
    for (int b = lane; b < batch; b += 32) s_seq[b] = seq_tiles(qo_indptr, kv_indptr, last_len, page_size, b, tpt);
    __syncwarp();
  }
  auto geom = [&](int b) {
    return staged ? s_seq[b] : seq_tiles(qo_indptr, kv_indptr, last_len, page_size, b, tpt);
  };
  // lane-parallel over the batch: the tiles of the sequences ahead of b (longer key length first, ties
  // in batch order), then the one sequence whose tiles hold this CTA
  for (int base = 0; base < batch; base += 32) {
    const int b = base + lane;
    SeqTiles tb{0, 0, 0};
    int first = 0;
    if (b < batch) {
      tb = geom(b);
      for (int o = 0; o < batch; ++o) {
        const SeqTiles to = geom(o);
        if (to.kv_len > tb.kv_len || (to.kv_len == tb.kv_len && o < b)) first += to.tiles;
      }
    }
    const unsigned hit = __ballot_sync(kFull, tb.tiles > 0 && cta >= first && cta < first + tb.tiles);
    if (hit != 0u) {
      const int src = __ffs(hit) - 1;
      seq = base + src;
      tile = __shfl_sync(kFull, tb.tiles - 1 - (cta - first), src);  // a sequence's last (longest) tile first
      return;
    }
  }
}

template <int D, int STAGES>
__global__ void __launch_bounds__((kConsumers + 1) * 32) prefill_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                        PrefillArgs p) {
  using Cfg = PrefillCfg<D, STAGES>;
  constexpr int kHalves = Cfg::kHalves;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::kStageBytes);
  uint64_t* empty = full + STAGES;
  int* s_info = reinterpret_cast<int*>(empty + STAGES);

  // 1-D grid, KV head fastest: CTAs start in blockIdx order, so the heaviest tiles of every head go
  // out in the first wave (a (tiles, heads) grid would start all of head 0's tiles, light ones
  // included, before head 1's heaviest)
  const int kvh = blockIdx.x % p.hkv;
  const int cta = blockIdx.x / p.hkv;
  const int G = p.group;
  const int tokens_per_tile = kRows / G;
  if (threadIdx.x < 32) {
    int seq, tile;
    longest_first_tile(p.qo_indptr, p.kv_indptr, p.last_len, p.page_size, p.batch, tokens_per_tile, cta, seq,
                       tile);
    if (threadIdx.x == 0) {
      s_info[0] = seq;
      s_info[1] = tile;
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int seq = s_info[0];
  if (seq < 0) return;
  const int tile = s_info[1];
  const int q0 = p.qo_indptr[seq];
  const int qo_len = p.qo_indptr[seq + 1] - q0;
  const int n_pages = p.kv_indptr[seq + 1] - p.kv_indptr[seq];
  int ll = p.last_len[seq];
  ll = ll < 1 ? 1 : (ll > p.page_size ? p.page_size : ll);
  const int kv_len = n_pages > 0 ? (n_pages - 1) * p.page_size + ll : 0;
  const int t_first = tile * tokens_per_tile;                       // first query token of the tile
  const int t_last = min(qo_len, t_first + tokens_per_tile) - 1;    // last
  const int shift = kv_len - qo_len;                                // query i sees keys <= shift + i
  const int kv_hi = min(kv_len, shift + t_last + 1);
  const int n_blocks = kv_hi > 0 ? (kv_hi + kBlockTok - 1) / kBlockTok : 0;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == kConsumers) {
    if (lane == 0 && n_blocks > 0) {
      prefetch_tensormap(&tmap);
      const int32_t* pages = p.indices + p.kv_indptr[seq];
      for (int j = 0; j < n_blocks; ++j) {
        const int s = j % STAGES;
        if (j >= STAGES && !mbar_wait(&empty[s], ((j / STAGES) - 1) & 1, p.status)) break;
        mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
        uint8_t* dst = smem + s * Cfg::kStageBytes;
#pragma unroll
        for (int st = 0; st < kSub; ++st) {
          const int pos = j * kBlockTok + st * kTok;
          const int pi = pos / p.page_size;
          int page = p.total_pages;  // past the sequence: zero-filled box
          if (pi < n_pages) {
            page = pages[pi];
            if (static_cast<unsigned>(page) >= static_cast<unsigned>(p.total_pages)) {
              report(p.status, NQT_DEV_BAD_PAGE);
              page = p.total_pages;
            }
          }
          const int tok_in_page = pos - pi * p.page_size;
#pragma unroll
          for (int half = 0; half < kHalves; ++half)
            tma_load_4d(dst + (st * kHalves + half) * kBoxBytes, &tmap, &full[s], half * 64, kvh, tok_in_page,
                        page * 2);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int g = lane >> 2, t4 = lane & 3;
  const int row0 = warp * 16 + g;  // rows of this lane: row0 and row0 + 8
  const float NEG_INF = -__int_as_float(0x7f800000);
  int qtok[2], qhead[2];
  bool qvalid[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = row0 + 8 * h;
    qtok[h] = t_first + r / G;
    qhead[h] = kvh * G + r % G;
    qvalid[h] = qtok[h] < qo_len;
  }
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (qvalid[h]) {
        const __nv_bfloat16* qr = p.q + static_cast<int64_t>(q0 + qtok[h]) * p.q_st + static_cast<int64_t>(qhead[h]) * p.q_sh;
        qa[kk][h] = *reinterpret_cast<const uint32_t*>(qr + kk * 16 + 2 * t4);
        qa[kk][2 + h] = *reinterpret_cast<const uint32_t*>(qr + kk * 16 + 8 + 2 * t4);
      } else {
        qa[kk][h] = 0u;
        qa[kk][2 + h] = 0u;
      }
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {NEG_INF, NEG_INF}, l[2] = {0.f, 0.f};
  const int lim0 = shift + qtok[0];  // last visible key of each row
  const int lim1 = shift + qtok[1];
  const int lm_j = lane >> 3, lm_r = lane & 7;

  for (int j = 0; j < n_blocks; ++j) {
    const int s = j % STAGES;
    if (!mbar_wait(&full[s], (j / STAGES) & 1, p.status)) return;
    uint8_t* stage = smem + s * Cfg::kStageBytes;
    const int base = j * kBlockTok;
    if (base + kBlockTok > kv_len) {
      // zero V rows at or past kv_len (stale page contents never meet p = 0)
      consumer_bar();
      const int first_bad = max(0, kv_len - base);
      const int n_bad = kBlockTok - first_bad;
      for (int idx = threadIdx.x; idx < n_bad * kHalves * 8; idx += kConsumers * 32) {
        const int t = first_bad + idx / (kHalves * 8);
        const int rem = idx % (kHalves * 8);
        const int half = rem / 8, chunk = rem % 8;
        const int st = t / kTok, tr = t % kTok;
        *reinterpret_cast<uint4*>(stage + (st * kHalves + half) * kBoxBytes + 2048 + tr * 128 + chunk * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      consumer_bar();
    }
    // S = Q K^T: 8 n-tiles of 8 tokens
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int st = 0; st < kSub; ++st) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int half = kk >> 2;
        const int chunk = ((kk & 3) << 1) + (lm_j & 1);
        const int tok = ((lm_j >> 1) << 3) + lm_r;
        const uint32_t addr = smem_addr(stage + (st * kHalves + half) * kBoxBytes) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3, addr);
        // b0,b1: tokens 0-7 (k lo, k hi); b2,b3: tokens 8-15
        mma_bf16_16816(sc[2 * st], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
        mma_bf16_16816(sc[2 * st + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
      }
    }
    // mask + online softmax; lane rows: g (c0,c1) and g+8 (c2,c3); cols 2*t4, 2*t4+1
    float mx[2] = {NEG_INF, NEG_INF};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int key = base + n * 8 + 2 * t4;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kpos = key + (e & 1);
        const int lim = (e < 2) ? lim0 : lim1;
        const bool ok = (kpos <= lim) && (kpos < kv_len);
        sc[n][e] = ok ? sc[n][e] * p.scale_log2 : NEG_INF;
        mx[e >> 1] = fmaxf(mx[e >> 1], sc[n][e]);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(kFull, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(kFull, mx[h], 2));
    }
    float alpha[2], nm[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      nm[h] = fmaxf(m[h], mx[h]);
      // rows with nothing visible yet keep m = -inf; exp2(-inf - -inf) would be NaN
      const float ref = nm[h] == NEG_INF ? 0.f : nm[h];
      alpha[h] = exp2f(m[h] - ref);
      m[h] = nm[h];
      nm[h] = ref;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(sc[n][0] - nm[0]);
      const float p1 = exp2f(sc[n][1] - nm[0]);
      const float p2 = exp2f(sc[n][2] - nm[1]);
      const float p3 = exp2f(sc[n][3] - nm[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      // A fragment of P for k-step n/2: a0/a1 from even n-tile, a2/a3 from odd
      const int ks = n >> 1;
      if ((n & 1) == 0) {
        pa[ks][0] = pack_bf16x2(p0, p1);
        pa[ks][1] = pack_bf16x2(p2, p3);
      } else {
        pa[ks][2] = pack_bf16x2(p0, p1);
        pa[ks][3] = pack_bf16x2(p2, p3);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) l[h] = l[h] * alpha[h] + rs[h];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // O += P V: per k-step (16 tokens = one sub-tile), two d-chunks per ldmatrix.x4.trans
#pragma unroll
    for (int ks = 0; ks < kSub; ++ks) {
#pragma unroll
      for (int nc = 0; nc < D / 16; ++nc) {
        const int half = nc >> 2;
        const int chunk = ((nc & 3) << 1) + (lm_j >> 1);
        const int tok = ((lm_j & 1) << 3) + lm_r;
        const uint32_t addr =
            smem_addr(stage + (ks * kHalves + half) * kBoxBytes + 2048) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3, addr);
        // b0: (tok 0-7, chunk c) b1: (tok 8-15, chunk c) b2: (tok 0-7, c+1) b3: (tok 8-15, c+1)
        mma_bf16_16816(o[2 * nc], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b0, b1);
        mma_bf16_16816(o[2 * nc + 1], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // finalize
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(kFull, l[h], 1);
    l[h] += __shfl_xor_sync(kFull, l[h], 2);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (!qvalid[h]) continue;
    const float inv = l[h] > 0.f ? 1.f / l[h] : 0.f;
    __nv_bfloat16* orow = p.out + static_cast<int64_t>(q0 + qtok[h]) * p.o_st + static_cast<int64_t>(qhead[h]) * p.o_sh;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<__nv_bfloat162*>(orow + n * 8 + 2 * t4) =
          __floats2bfloat162_rn(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
  }
}

// ------------------------------------------------------------------ tcgen05 path (D = 128)
// CTA = two 128-row query tiles of one sequence and one KV head (row = token x GQA head; tile A holds
// the first 128 / G tokens, tile B the next 128 / G), over KV blocks of 64 tokens.  Both tiles read
// every K / V block from the same shared-memory stage, so a CTA moves half the K / V bytes per FLOP
// of a one-tile CTA: with one tile, the per-SM delivery of the 16-token K / V boxes (about 20 B per
// cycle), not the tensor pipe or the softmax, set the time per block.
//   warp 0       TMA producer (Q of both tiles, then K and V of each block)
//   warp 1       TMEM allocator; its lane 0 issues tile A's MMAs
//   warps 2..5   softmax of tile A, warps 6..9 softmax of tile B: thread = one query row = one TMEM lane
//   warp 10      lane 0 issues tile B's MMAs
// TMEM (512 columns): tile t has its S double buffer at [128 t, 128 t + 64) and [128 t + 64, 128 t + 128)
// and O at [256 + 128 t, 384 + 128 t), all fp32.  S = Q K^T: A = Q (K-major, 128B swizzle), B = K
// (K-major).  P (bf16, two per column) overwrites the first 32 columns of its own S buffer, and
// O += P V takes A = P from TMEM and B = V (MN-major: token rows of 64 contiguous dims).  O is
// rescaled in TMEM only when a row's running max grows by more than 2^8 (exact either way: the
// exponent base only has to be shared by P and l).
namespace tcp {
constexpr int kM = 128;                  // rows per tile
constexpr int kTiles = 2;                // tiles per CTA
constexpr int kN = 64;                   // keys per block
constexpr int kStages = 4;
constexpr int kSmemPages = 1024;         // page ids of the sequence staged in shared memory
constexpr int kQBytes = kM * 128 * 2;    // one tile: [half][128 rows][128 B]
constexpr int kKVHalf = kN * 128;        // [64 tokens][128 B]
constexpr int kKVBytes = 4 * kKVHalf;    // K h0, K h1, V h0, V h1
constexpr int kSoftmaxWarps = 4 * kTiles;
constexpr int kIssuerB = 2 + kSoftmaxWarps;  // warp of tile B's MMA-issuing thread
constexpr int kThreads = (kIssuerB + 1) * 32;
constexpr int kBarBytes = 256;
constexpr int kSmem = 1024 + kTiles * kQBytes + kStages * kKVBytes + kBarBytes + 4 * kSmemPages;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;
}  // namespace tcp

// exp2 on the special-function unit (PTX ex2.approx.ftz.f32, relative error about 2^-22): P is
// rounded to bf16 (relative step 2^-9) right after, and every argument is <= 8.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Three-input max and packed two-lane fp32 arithmetic (sm_100 FMNMX3 / FFMA2 / FADD2): half the
// instructions of the scalar forms for the softmax's row max, scale-and-shift and row sum.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ uint64_t f2(float lo, float hi) { return f2(__float_as_uint(lo), __float_as_uint(hi)); }
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// TMA store of a 3-D box from shared memory (bulk group), its commit and the wait until the
// shared-memory source has been read; a named barrier over `n` threads.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__global__ void __launch_bounds__(tcp::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kvmap,
                      const __grid_constant__ CUtensorMap omap, PrefillArgs p) {
  using namespace tcp;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;  // tile t at t * kQBytes
  uint8_t* sKV = sQ + kTiles * kQBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kStages * kKVBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kStages;  // [tile][stage]: the tile's S and PV of the stage's block are done
  uint64_t* s_full = kv_empty + kTiles * kStages;  // [tile][S buffer]
  uint64_t* p_full = s_full + 2 * kTiles;  // [tile][S buffer]
  uint64_t* o_done = p_full + 2 * kTiles;  // [tile][S buffer parity of the PV]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2 * kTiles);
  int* info = reinterpret_cast<int*>(tmem_slot + 1);
  int32_t* s_pages = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(bars) + kBarBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // 1-D grid, KV head fastest: CTAs start in blockIdx order, so the heaviest tiles of every head go
  // out in the first wave (a (tiles, heads) grid would start all of head 0's tiles, light ones
  // included, before head 1's heaviest)
  const int kvh = blockIdx.x % p.hkv;
  const int cta = blockIdx.x / p.hkv;
  const int G = p.group;
  const int tpt = kM / G;  // tokens per tile
  if (threadIdx.x < 32) {
    int seq, tile;
    longest_first_tile(p.qo_indptr, p.kv_indptr, p.last_len, p.page_size, p.batch, kTiles * tpt, cta, seq, tile);
    if (threadIdx.x == 0) {
      info[0] = seq;
      info[1] = tile;
    }
  }
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) mbar_init(&kv_full[s], 1);
    for (int s = 0; s < kTiles * kStages; ++s) mbar_init(&kv_empty[s], 1);
    for (int b = 0; b < 2 * kTiles; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&o_done[b], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int seq = info[0];

  // blocks each tile needs (0: the tile has no rows); tile B's rows come after tile A's, so nbt[1] is
  // 0 or >= nbt[0]
  int nbt[kTiles] = {0, 0};
  int q0 = 0, qo_len = 0, n_pages = 0, kv_len = 0, t_first = 0, shift = 0;
  if (seq >= 0) {
    q0 = p.qo_indptr[seq];
    qo_len = p.qo_indptr[seq + 1] - q0;
    n_pages = p.kv_indptr[seq + 1] - p.kv_indptr[seq];
    int ll = p.last_len[seq];
    ll = ll < 1 ? 1 : (ll > p.page_size ? p.page_size : ll);
    kv_len = n_pages > 0 ? (n_pages - 1) * p.page_size + ll : 0;
    t_first = info[1] * kTiles * tpt;
    shift = kv_len - qo_len;
#pragma unroll
    for (int t = 0; t < kTiles; ++t) {
      const int f = t_first + t * tpt;
      const int t_last = min(qo_len, f + tpt) - 1;
      const int kv_hi = min(kv_len, shift + t_last + 1);
      nbt[t] = (t_last >= f && kv_hi > 0) ? (kv_hi + kN - 1) / kN : 0;
    }
  }
  const int nb = max(nbt[0], nbt[1]);

  if (nb > 0) {
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      // stage the page ids this CTA reads in shared memory (one coalesced pass by the warp)
      const int32_t* pages_g = p.indices + p.kv_indptr[seq];
      const int n_used = min(n_pages, (nb * kN + p.page_size - 1) / p.page_size);
      const bool staged = n_used <= kSmemPages;
      if (staged)
        for (int i = lane; i < n_used; i += 32) s_pages[i] = pages_g[i];
      __syncwarp();
      const int32_t* pages = staged ? s_pages : pages_g;
      if (lane == 0) {
        prefetch_tensormap(&qmap);
        prefetch_tensormap(&kvmap);
        const int nq = nbt[1] > 0 ? kTiles : 1;
        mbar_arrive_expect_tx(q_full, nq * kQBytes);
        for (int t = 0; t < nq; ++t)
          for (int half = 0; half < 2; ++half)
            tma_load_3d(sQ + t * kQBytes + half * (kQBytes / 2), &qmap, q_full, half * 64, kvh * G,
                        q0 + t_first + t * tpt);
      }
      // Lane l issues box l of each block (sub-tile l/4, K or V, dims half): a single thread
      // issuing all 16 boxes serialises on the per-instruction TMA issue cost.
      const int sub = lane >> 2, kind = (lane >> 1) & 1, half = lane & 1;
      for (int j = 0; j < nb; ++j) {
        const int s = j % kStages;
        // warp-uniform decision: every lane reaches the same __syncwarp.  The stage's previous block,
        // j - kStages, is released by each tile that read it
        bool ready = true;
        if (j >= kStages) {
#pragma unroll
          for (int t = 0; t < kTiles; ++t)
            if (j - kStages < nbt[t] && !mbar_wait(&kv_empty[t * kStages + s], ((j / kStages) - 1) & 1, p.status))
              ready = false;
        }
        if (!__all_sync(kFull, ready)) break;
        if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], kKVBytes);
        __syncwarp();
        if (lane < 16) {
          const int pos = j * kN + sub * 16;
          const int pi = pos / p.page_size;
          int page = p.total_pages;  // past the sequence: zero-filled box
          if (pi < n_pages) {
            page = pages[pi];
            if (static_cast<unsigned>(page) >= static_cast<unsigned>(p.total_pages)) {
              report(p.status, NQT_DEV_BAD_PAGE);
              page = p.total_pages;
            }
          }
          const int tip = pos - pi * p.page_size;
          tma_load_4d(sKV + s * kKVBytes + (kind * 2 + half) * kKVHalf + sub * 2048, &kvmap, &kv_full[s], half * 64,
                      kvh, tip, page * 2 + kind);
        }
      }
    } else if (warp == 1 || warp == kIssuerB) {
      // ------------------------------------------------------------ MMA issuers
      // One thread per tile (warp 1: tile A, warp kIssuerB: tile B), so neither tile's MMAs queue
      // behind the other's waits.  Order per tile: S(0), S(1), then per block j: PV(j), S(j+2).
      // S(j+2) reuses the tile's S / P buffer (j & 1); the tensor pipe runs one thread's MMAs in issue
      // order, so it overwrites P(j) only after PV(j) has read it.
      const int t = warp == 1 ? 0 : 1;
      const int nbx = t == 0 ? nbt[0] : nbt[1];
      if (lane == 0 && nbx > 0) {
        constexpr uint32_t kIdescS = tc::idesc_bf16_f32(kM, kN, false, false);
        constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(kM, 128, false, true);
        bool ok = mbar_wait(q_full, 0, p.status);
        // descriptors are built once; a byte offset inside shared memory (< 256 KB) moves only the
        // 14-bit start-address field, so it is added to the descriptor as offset >> 4
        const uint64_t q_desc = tc::smem_desc_sw128(smem_addr(sQ + t * kQBytes), 16, 1024);
        const uint64_t k_desc = tc::smem_desc_sw128(smem_addr(sKV), 16, 1024);
        const uint64_t v_desc = tc::smem_desc_sw128(smem_addr(sKV + 2 * kKVHalf), kKVHalf, 1024);
        const uint32_t s_cols = tmem + t * 128, o_cols = tmem + kColO + t * 128;
        auto issue_s = [&](int j) {
          if (!mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, p.status)) {
            ok = false;
            return;
          }
          tc::fence_after_sync();
          const int sb = j & 1;
          const uint64_t kd = k_desc + static_cast<uint32_t>(((j % kStages) * kKVBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = ((kk >> 2) * (kQBytes / 2) + (kk & 3) * 32) >> 4;
            const uint32_t koff = ((kk >> 2) * kKVHalf + (kk & 3) * 32) >> 4;
            tc::mma_f16_ss(s_cols + sb * kN, q_desc + off, kd + koff, kIdescS, kk > 0 ? 1u : 0u);
          }
          tc::commit(&s_full[2 * t + sb]);
        };
        auto issue_pv = [&](int i) {
          const int sb = i & 1, s = i % kStages;
          if (!mbar_wait(&p_full[2 * t + sb], (i >> 1) & 1, p.status)) {
            ok = false;
            return;
          }
          tc::fence_after_sync();
          const uint64_t vd = v_desc + static_cast<uint32_t>((s * kKVBytes) >> 4);
#pragma unroll
          for (int ks = 0; ks < kN / 16; ++ks)
            tc::mma_f16_ts(o_cols, s_cols + sb * kN + ks * 8, vd + ((ks * 2048) >> 4), kIdescPV,
                           (i > 0 || ks > 0) ? 1u : 0u);
          tc::commit(&o_done[2 * t + sb]);
          tc::commit(&kv_empty[t * kStages + s]);  // this tile's S(i) and PV(i) have read stage s
        };
        for (int j = 0; j < 2 && j < nbx && ok; ++j) issue_s(j);
        for (int j = 0; j < nbx && ok; ++j) {
          issue_pv(j);
          if (ok && j + 2 < nbx) issue_s(j + 2);
        }
      }
    } else {
      // ------------------------------------------------------------ softmax warps (2 .. kIssuerB - 1)
      const int t = (warp - 2) >> 2;
      const int nbx = t == 0 ? nbt[0] : nbt[1];
      const int quarter = warp & 3;
      const int row = quarter * 32 + lane;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
      const uint32_t col_s = t * 128, col_o = kColO + t * 128;
      uint64_t* sfull = s_full + 2 * t;
      uint64_t* pfull = p_full + 2 * t;
      uint64_t* odone = o_done + 2 * t;
      const int qtok = t_first + t * tpt + row / G;
      const int head = kvh * G + row % G;
      const int lim = shift + qtok;
      const float NEG_INF = -__int_as_float(0x7f800000);
      float m_used = NEG_INF, l = 0.f;
      bool ok = true;
      for (int j = 0; j < nbx && ok; ++j) {
        const int sb = j & 1;
        const int s = j % kStages;
        if (!mbar_wait(&sfull[sb], (j >> 1) & 1, p.status)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        uint32_t sr[64];
        tc::ld_32x32b_x32(t_row + col_s + sb * kN, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tc::ld_32x32b_x32(t_row + col_s + sb * kN + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tc::wait_ld();
        const int base = j * kN;
        // raw scores; the causal / length mask only matters on the diagonal and the last block
        if (base + kN - 1 > lim || base + kN > kv_len) {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int key = base + c;
            if (key > lim || key >= kv_len) sr[c] = __float_as_uint(NEG_INF);
          }
        }
        float mx8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = max3f(__uint_as_float(sr[e]), __uint_as_float(sr[e + 8]), __uint_as_float(sr[e + 16]));
          const float b = max3f(a, __uint_as_float(sr[e + 24]), __uint_as_float(sr[e + 32]));
          const float c = max3f(b, __uint_as_float(sr[e + 40]), __uint_as_float(sr[e + 48]));
          mx8[e] = fmaxf(c, __uint_as_float(sr[e + 56]));
        }
        const float mx_raw = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        const float mx = mx_raw * p.scale_log2;  // log2 domain (scale > 0 keeps the order)
        const float m_new = fmaxf(m_used, mx);
        const bool need = (m_used != NEG_INF) && (m_new > m_used + 8.f);
        if (__any_sync(kFull, need)) {
          // rescale this warp's O rows once PV(j-1) has landed
          if (!mbar_wait(&odone[(j - 1) & 1], ((j - 1) >> 1) & 1, p.status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const float alpha = need ? ex2_approx(m_used - m_new) : 1.f;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t o[32];
            tc::ld_32x32b_x32(t_row + col_o + ch * 32, o);
            tc::wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tc::st_32x32b_x32(t_row + col_o + ch * 32, o);
          }
          tc::wait_st();
          if (need) {
            l *= alpha;
            m_used = m_new;
          }
        }
        if (m_used == NEG_INF) m_used = m_new;
        // P(j) goes over the first 32 columns of S(j): this thread's row, already in registers
        const uint64_t sc2 = f2(p.scale_log2, p.scale_log2);
        const uint64_t mo2 = f2(-m_used, -m_used);
        uint64_t rs2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};  // row-sum partials, two lanes each
        uint32_t pk[32];
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          uint64_t x2[4];
          float pv[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            x2[q] = f2_fma(f2(sr[c8 * 8 + 2 * q], sr[c8 * 8 + 2 * q + 1]), sc2, mo2);
            float lo, hi;
            f2_split(x2[q], lo, hi);
            pv[2 * q] = ex2_approx(lo);
            pv[2 * q + 1] = ex2_approx(hi);
            pk[c8 * 4 + q] = pack_bf16x2(pv[2 * q], pv[2 * q + 1]);
          }
          const uint64_t r = f2_add(f2_add(f2(pv[0], pv[1]), f2(pv[2], pv[3])), f2_add(f2(pv[4], pv[5]), f2(pv[6], pv[7])));
          rs2[c8 & 1] = f2_add(rs2[c8 & 1], r);
        }
        tc::st_32x32b_x32(t_row + col_s + sb * kN, pk);
        {
          float lo, hi;
          f2_split(f2_add(rs2[0], rs2[1]), lo, hi);
          l += lo + hi;
        }
        if (base + kN > kv_len) {
          // zero V rows at or past kv_len so 0 * stale never meets a NaN (both tiles may write the
          // same zeros into this block's stage; the stage holds it since kv_full(j))
          const int first_bad = max(0, kv_len - base);
          const int n_bad = kN - first_bad;
          uint8_t* v0 = sKV + s * kKVBytes + 2 * kKVHalf;
          for (int idx = row; idx < n_bad * 16; idx += kM) {
            const int tok = first_bad + (idx >> 4);
            const int hf = (idx >> 3) & 1, chunk = idx & 7;
            *reinterpret_cast<uint4*>(v0 + hf * kKVHalf + tok * 128 + chunk * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pfull[sb]);
      }
      // epilogue: O / l once the tile's last PV has completed, written as bf16 into the tile's own Q
      // buffer (free: its last reader, S(nbx - 1), completed before the last PV) in the Q box layout.
      // A full tile (every row inside the chunk) leaves through one TMA store per 64 dims; a ragged
      // one through coalesced 16-byte stores of its valid rows (a warp covers two whole rows).  Every
      // thread of the tile reaches the named barrier.
      const bool full = p.tma_out && t_first + (t + 1) * tpt <= qo_len;
      const bool have = ok && nbx > 0 && mbar_wait(&odone[(nbx - 1) & 1], ((nbx - 1) >> 1) & 1, p.status);
      uint8_t* sO = sQ + t * kQBytes;
      if (have) {
        tc::fence_after_sync();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint8_t* srow = sO + row * 128;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t o[32];
          tc::ld_32x32b_x32(t_row + col_o + ch * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
            pk.y = pack_bf16x2(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
            pk.z = pack_bf16x2(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
            pk.w = pack_bf16x2(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
            // dims 32 ch + 8 v: half ch / 2, 16-byte chunk (ch % 2) * 4 + v, 128B-swizzled by row
            const int chunk = (ch & 1) * 4 + v;
            *reinterpret_cast<uint4*>(srow + (ch >> 1) * (kQBytes / 2) + ((chunk ^ (row & 7)) << 4)) = pk;
          }
        }
      }
      if (nbx > 0) {
        if (full) fence_proxy_async_smem();
        named_bar_sync(1 + t, 4 * 32);
        if (full) {
          if (quarter == 2 && lane == 0) {  // warp 2 + 4 t
            for (int half = 0; half < 2; ++half)
              tma_store_3d(&omap, sO + half * (kQBytes / 2), half * 64, kvh * G, q0 + t_first + t * tpt);
            bulk_commit_group();
            bulk_wait_group_read0();  // the Q buffer stays valid until the store has read it
          }
        } else {
          // 128 rows x 16 chunks of 16 bytes; consecutive threads take consecutive chunks of a row
          for (int i = row; i < kM * 16; i += kM) {
            const int r = i >> 4, c = i & 15;
            const int tok = t_first + t * tpt + r / G;
            if (tok < qo_len) {
              const uint4 v = *reinterpret_cast<const uint4*>(sO + (c >> 3) * (kQBytes / 2) + r * 128 +
                                                              (((c & 7) ^ (r & 7)) << 4));
              __nv_bfloat16* dst =
                  p.out + static_cast<int64_t>(q0 + tok) * p.o_st + static_cast<int64_t>(kvh * G + r % G) * p.o_sh + c * 8;
              if (p.out16) {
                *reinterpret_cast<uint4*>(dst) = v;
              } else {  // out and its strides are only 4-byte aligned
                uint32_t* d4 = reinterpret_cast<uint32_t*>(dst);
                d4[0] = v.x;
                d4[1] = v.y;
                d4[2] = v.z;
                d4[3] = v.w;
              }
            }
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
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

int encode_map(CUtensorMap* map, const void* layer, int total_pages, int page_size, int hkv, int d) {
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

// K-only or V-only boxes {64 dims, 1 head, 16 tokens, 1 kind} for the tcgen05 path.
int encode_kv_map_single(CUtensorMap* map, const void* layer, int total_pages, int page_size, int hkv, int d) {
  auto encode = get_encode();
  if (encode == nullptr) return NQT_ERR_CUDA;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(hkv),
                        static_cast<cuuint64_t>(page_size), static_cast<cuuint64_t>(total_pages) * 2};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(hkv) * d * 2,
                           static_cast<cuuint64_t>(page_size) * hkv * d * 2};
  cuuint32_t box[4] = {64, 1, kTok, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(layer), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NQT_OK : NQT_ERR_CUDA;
}

// Q viewed as {D, heads, tokens}; one box = 64 dims x G heads x (128 / G) tokens = 128 rows of 128 B.
int encode_q_map(CUtensorMap* map, const void* q, int64_t q_st, int64_t q_sh, int tokens, int hq, int group) {
  auto encode = get_encode();
  if (encode == nullptr) return NQT_ERR_CUDA;
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(hq), static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(q_sh) * 2, static_cast<cuuint64_t>(q_st) * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(group), static_cast<cuuint32_t>(tcp::kM / group)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NQT_OK : NQT_ERR_CUDA;
}

int launch_prefill_tc(const CUtensorMap& qmap, const CUtensorMap& kvmap, const CUtensorMap& omap,
                      const PrefillArgs& a, int total_q, cudaStream_t s) {
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tcp::kSmem);
  });
  const int tokens_per_cta = tcp::kTiles * (tcp::kM / a.group);
  const int grid_x = (total_q + tokens_per_cta - 1) / tokens_per_cta + a.batch;
  prefill_tc_kernel<<<dim3(grid_x * a.hkv), tcp::kThreads, tcp::kSmem, s>>>(qmap, kvmap, omap, a);
  return check_launch("prefill_attention_tc");
}

template <int D, int STAGES>
int launch_prefill(const CUtensorMap& map, const PrefillArgs& a, int grid_x, cudaStream_t s) {
  using Cfg = PrefillCfg<D, STAGES>;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(prefill_kernel<D, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  });
  prefill_kernel<D, STAGES><<<dim3(grid_x * a.hkv), Cfg::kThreads, Cfg::kSmem, s>>>(map, a);
  return check_launch("prefill_attention");
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_prefill_attention(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                     const void* layer_cache, int total_pages, int page_size,
                                     const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_indices,
                                     const int32_t* last_page_len, int batch, int total_q_tokens, int num_qo_heads,
                                     int num_kv_heads, int head_dim, float sm_scale, void* out,
                                     int64_t out_stride_tok, int64_t out_stride_head, int32_t* status,
                                     void* stream) {
  if (!q || !layer_cache || !qo_indptr || !kv_indptr || !kv_indices || !last_page_len || !out) return NQT_ERR_ARG;
  if (batch < 1 || total_q_tokens < 0 || total_pages < 1) return NQT_ERR_ARG;
  if (num_kv_heads < 1 || num_qo_heads % num_kv_heads) return NQT_ERR_ARG;
  const int group = num_qo_heads / num_kv_heads;
  if (group > 8 || (kRows % group)) return NQT_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return NQT_ERR_UNSUPPORTED;
  if (page_size < kTok || page_size % kTok || page_size > 256) return NQT_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(layer_cache) & 15) || (reinterpret_cast<uintptr_t>(q) & 3) ||
      (reinterpret_cast<uintptr_t>(out) & 3))
    return NQT_ERR_ARG;
  if ((q_stride_tok & 1) || (q_stride_head & 1) || (out_stride_tok & 1) || (out_stride_head & 1)) return NQT_ERR_ARG;
  if (static_cast<int64_t>(total_pages) * 2 >= (int64_t(1) << 31)) return NQT_ERR_UNSUPPORTED;
  if (total_q_tokens == 0) return NQT_OK;
  PrefillArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_stride_tok;
  a.q_sh = q_stride_head;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_st = out_stride_tok;
  a.o_sh = out_stride_head;
  a.qo_indptr = qo_indptr;
  a.kv_indptr = kv_indptr;
  a.indices = kv_indices;
  a.last_len = last_page_len;
  a.status = status;
  a.batch = batch;
  a.hq = num_qo_heads;
  a.hkv = num_kv_heads;
  a.group = group;
  a.page_size = page_size;
  a.total_pages = total_pages;
  a.scale_log2 = sm_scale * 1.4426950408889634f;
  cudaStream_t s = as_stream(stream);
  if (head_dim == 128) {
    // tcgen05 path: Q rows come in by TMA, so q must be 16-byte aligned with strides in 16-byte units
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (q_stride_tok % 8) || (q_stride_head % 8)) return NQT_ERR_ARG;
    CUtensorMap qmap, kvmap;
    int rc = encode_q_map(&qmap, q, q_stride_tok, q_stride_head, total_q_tokens, num_qo_heads, group);
    if (rc != NQT_OK) return rc;
    rc = encode_kv_map_single(&kvmap, layer_cache, total_pages, page_size, num_kv_heads, head_dim);
    if (rc != NQT_OK) return rc;
    // full query tiles leave through a TMA store when out allows a tensor map (16-byte aligned base
    // and strides); otherwise every row is stored by its thread
    CUtensorMap omap{};
    a.out16 = (reinterpret_cast<uintptr_t>(out) & 15) == 0 && out_stride_tok % 8 == 0 && out_stride_head % 8 == 0;
    a.tma_out = a.out16 &&
                encode_q_map(&omap, out, out_stride_tok, out_stride_head, total_q_tokens, num_qo_heads, group) == NQT_OK;
    return launch_prefill_tc(qmap, kvmap, omap, a, total_q_tokens, s);
  }
  a.tma_out = 0;
  a.out16 = 0;
  CUtensorMap map;
  int rc = encode_map(&map, layer_cache, total_pages, page_size, num_kv_heads, head_dim);
  if (rc != NQT_OK) return rc;
  const int tokens_per_tile = kRows / group;
  const int grid_x = (total_q_tokens + tokens_per_tile - 1) / tokens_per_tile + batch;
  return launch_prefill<64, 4>(map, a, grid_x, s);
}
