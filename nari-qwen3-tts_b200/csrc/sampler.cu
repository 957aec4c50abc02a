// Fused logits sampler: repetition penalty, temperature, top-k, top-p and a
// seeded draw in one launch.
//
// Per row:
//   1. x = logits (fp32); where seen: x > 0 ? x / penalty : x * penalty.
//   2. temperature == 0: first argmax of x (greedy) -> done.
//   3. y = x / T (optionally rounded to the logits type, as torch does for a
//      half-precision row without a seen mask).
//   4. k_eff = k <= 0 ? V : min(k, V); the top-k of y ordered by (value desc,
//      token id asc), so ties go to the lowest token id.
//   5. p = softmax over the top-k values; if top_p < 1, rank r is dropped
//      when (cumsum_r - p_r) > top_p with the cumulative sum accumulated in
//      double and rounded per element (what torch's CPU cumsum does), and
//      the kept mass is renormalised.
//   6. Draw: argmax_r p_r / E_r (exponential race; first max wins), where
//      E_r = -log(U_r) and U_r comes from Philox4x32-10 keyed by the row's
//      seed with counter (rank, 0, offset) - or E_r is read from a caller
//      buffer (the parity entry).  torch.multinomial(p, 1) computes exactly
//      argmax(p / Exp(1)) on the CPU, so the same noise gives the same id.
//   7. Optionally mark the sampled token in the seen mask.
//
// Work split: a group of G = 1, 2, 4 or 8 warps takes a row (the host picks
// G so that rows x G fill the GPU); the group streams its row two or three
// times (after the first pass it is an L1 hit) and its warps meet only at a
// named barrier:
//   histogram  256 bins of t = max(0, (m - x) / w + 64), with m and the width
//           w = (m - mean) / 48 from a strided sample of the row.  y never
//           decreases as x grows and t never increases, so the bins up to the
//           one holding the k-th value hold the whole y-top-k, except for an
//           exact tie in y made by the rounding of the quotient (checked
//           below).  When that bin alone holds too many, its 256 sub-bins are
//           counted in a second pass (t - bin is exact, so the split stays
//           monotone).
//   compaction  warp ballots collect the <= 64 candidates; y is computed for
//           them only, they are bitonic-sorted in one warp's registers, and
//           the largest logit left out must not tie the k-th value after the
//           division.
// Rows the group path cannot settle (k > 64, NaN or +inf logits, a row that
// does not narrow to 64 candidates, a rounding tie) are marked, and after the
// group phase the whole CTA takes each of them through the exact general path:
// a 4-pass radix select (8 bits per pass) of the k-th key, compaction of every
// key >= it and a bitonic sort in shared memory.
//
// Reference semantics: sample_logits_stateless / _cpu_sample_row
// (model/sampling.py:55-95, 127-225).
#include <type_traits>

#include "common.cuh"

namespace nqt {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;  // rows per CTA
constexpr int kMaxVocab = 16384;
constexpr int kFastK = 64;        // largest top-k of the warp path
constexpr int kBins = 256;        // histogram bins of the warp path
constexpr float kGapBins = 48.f;    // bin width = (sample max - sample mean) / kGapBins
constexpr float kBinsAbove = 64.f;  // bins kept for the logits above the sample's max
constexpr float kFltMax = 3.402823466e38f;

struct SampleArgs {
  const void* logits;
  int64_t lstride;
  int rows, vocab, np2;
  const float* temp;
  const int32_t* top_k;
  const float* top_p;
  const int64_t* seed;
  const int64_t* offset;
  int64_t offset_stride;
  const float* noise;
  int64_t noise_stride;
  const float* penalty;
  uint8_t* seen;
  int64_t seen_stride;
  int update_seen;
  int round_scaled;
  int64_t* tokens;
  float* probs;
  int32_t* ids;
  int32_t* status;
};

// ---- Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), written from the paper.
__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint2 key) {
  const uint32_t kMul0 = 0xD2511F53u, kMul1 = 0xCD9E8D57u;
  const uint32_t kWeyl0 = 0x9E3779B9u, kWeyl1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kMul0, ctr.x), lo0 = kMul0 * ctr.x;
    const uint32_t hi1 = __umulhi(kMul1, ctr.z), lo1 = kMul1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += kWeyl0;
    key.y += kWeyl1;
  }
  return ctr;
}

__device__ __forceinline__ float exp_noise(int64_t seed, int64_t offset, int rank) {
  const uint4 ctr = make_uint4(static_cast<uint32_t>(rank), 0u, static_cast<uint32_t>(offset),
                               static_cast<uint32_t>(static_cast<uint64_t>(offset) >> 32));
  const uint2 key = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(static_cast<uint64_t>(seed) >> 32));
  const uint4 r = philox4x32_10(ctr, key);
  const float u = (static_cast<float>(r.x >> 8) + 0.5f) * 5.9604644775390625e-8f;  // (0, 1)
  return -logf(u);
}

__device__ __forceinline__ uint32_t order_key(float v) {
  if (v == 0.f) v = 0.f;  // -0 and +0 compare equal, so give them one key
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t cand_word(uint32_t key, int i) {
  return (static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(i));
}

__device__ __forceinline__ int cand_token(uint64_t c) { return static_cast<int>(~static_cast<uint32_t>(c)); }

template <typename T>
__device__ __forceinline__ T block_reduce_sum(T v, T* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  T r = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) r += scratch[w];
  return r;
}

// First maximum: larger value wins, equal values go to the lower index.
__device__ __forceinline__ void argmax_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(kFull, v, o);
    const int i2 = __shfl_xor_sync(kFull, i, o);
    argmax_merge(v, i, v2, i2);
  }
}

__device__ __forceinline__ int block_argmax(float v, int i, float* sv, int* si) {
  warp_argmax(v, i);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = i;
  }
  __syncthreads();
  float bv = sv[0];
  int bi = si[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) argmax_merge(bv, bi, sv[w], si[w]);
  return bi;
}

// Inclusive scan of one int per thread across the block.
__device__ __forceinline__ int block_incl_scan(int v, int* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) s_warp[warp] = v;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += s_warp[w];
  __syncthreads();
  return v + base;
}

__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += y;
  }
  return v;
}

// Bitonic sort (descending) of 64 keys held two per lane: rank i lives in
// lane i % 32, slot i / 32.  Pairs closer than 32 ranks are exchanged with
// shuffles; the j == 32 step is a swap between a lane's two slots.
__device__ __forceinline__ void warp_sort64_desc(uint64_t& v0, uint64_t& v1) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {
        if (v0 < v1) {
          const uint64_t t = v0;
          v0 = v1;
          v1 = t;
        }
      } else {
        const uint64_t p0 = __shfl_xor_sync(kFull, v0, j);
        const uint64_t p1 = __shfl_xor_sync(kFull, v1, j);
        const bool lower = (lane & j) == 0;
        const bool max0 = lower == ((lane & k) == 0);
        const bool max1 = lower == (((lane + 32) & k) == 0);
        v0 = max0 ? (v0 > p0 ? v0 : p0) : (v0 < p0 ? v0 : p0);
        v1 = max1 ? (v1 > p1 ? v1 : p1) : (v1 < p1 ? v1 : p1);
      }
    }
  }
}

struct RowParams {
  float temp, pen, top_p;
  int k_eff;
  int64_t seed, off;
};

__device__ __forceinline__ RowParams row_params(const SampleArgs& a, int row) {
  RowParams p;
  p.temp = a.temp[row];
  p.pen = a.penalty != nullptr ? a.penalty[row] : 1.f;
  const int kreq = a.top_k[row];
  p.top_p = a.top_p[row];
  p.seed = a.noise == nullptr ? a.seed[row] : 0;
  p.off = a.noise == nullptr ? a.offset[row * a.offset_stride] : 0;
  p.k_eff = (kreq <= 0 || kreq >= a.vocab) ? a.vocab : kreq;
  return p;
}

// Step 1: the repetition penalty on a seen logit.
__device__ __forceinline__ float penalised(float x, bool seen, float pen) {
  return seen ? (x > 0.f ? __fdiv_rn(x, pen) : __fmul_rn(x, pen)) : x;
}

// Step 3: y = x / T, rounded to the logits type when asked.
template <typename T>
__device__ __forceinline__ float scaled(const SampleArgs& a, const RowParams& p, float x) {
  const float y = __fdiv_rn(x, p.temp);
  return a.round_scaled ? to_f32(from_f32<T>(y)) : y;
}

// ---- the group path ---------------------------------------------------------
// G warps (1, 2, 4 or 8) take one row together; the host picks G so that the
// rows times G fill the GPU.  Every decision that needs the whole row is made
// by each warp of the group from the same shared data, so the warps only meet
// at the group barrier.

template <int G>
struct GroupShared {
  int hist[kBins];
  uint64_t slots[G][kFastK];
  float x_out[G];
  int count[G];
  float best_v[G];
  int best_i[G];
};

// Named barrier 1 + group over the group's G * 32 threads (immediate
// operands, so the CTA reserves only the barriers it uses).
template <int G>
__device__ __forceinline__ void group_sync(int group) {
  if constexpr (G == 1) {
    __syncwarp();
  } else if constexpr (G == 8) {
    asm volatile("bar.sync 1, 256;" ::: "memory");
  } else if constexpr (G == 4) {
    if (group == 0) {
      asm volatile("bar.sync 1, 128;" ::: "memory");
    } else {
      asm volatile("bar.sync 2, 128;" ::: "memory");
    }
  } else {
    static_assert(G == 2, "groups of 1, 2, 4 or 8 warps");
    switch (group) {
      case 0: asm volatile("bar.sync 1, 64;" ::: "memory"); break;
      case 1: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
      case 2: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
      default: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
    }
  }
}

// The group's view of its row: every pass streams the row again (16-byte
// vectors when aligned, else elements); after the first pass the row is an
// L1 hit.  for_each calls f(e, x, valid) with x penalised; every lane of a
// warp makes the same number of calls, so f may use warp collectives.
template <typename T, int G, bool SEEN>
struct GroupRow {
  static constexpr int kVec = 16 / static_cast<int>(sizeof(T));
  using SeenBits = typename std::conditional<kVec == 8, uint64_t, uint32_t>::type;
  const T* lrow;
  const uint8_t* srow;
  int V;
  float pen;
  int gl;  // lane index within the group, 0 .. G * 32 - 1
  bool vec;

  __device__ __forceinline__ GroupRow(const T* l, const uint8_t* s, int vocab, float p, int group_lane)
      : lrow(l), srow(s), V(vocab), pen(p), gl(group_lane) {
    vec = (reinterpret_cast<uintptr_t>(lrow) & 15u) == 0 && V % kVec == 0 &&
          (!SEEN || (reinterpret_cast<uintptr_t>(srow) % kVec) == 0);
  }

  __device__ __forceinline__ float pen_of(float x, bool seen) const {
    if constexpr (SEEN) return penalised(x, seen, pen);
    return x;
  }

  template <class F>
  __device__ __forceinline__ void for_each(F&& f) const {
    if (vec) {
      const int chunks = V / kVec;
      constexpr int kUnroll = sizeof(T) == 4 ? 4 : 2;
      constexpr int kStride = G * 32;
      for (int c0 = 0; c0 < chunks; c0 += kStride * kUnroll) {
        uint4 r[kUnroll];
        SeenBits b[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int c = c0 + u * kStride + gl;
          r[u] = c < chunks ? reinterpret_cast<const uint4*>(lrow)[c] : make_uint4(0u, 0u, 0u, 0u);
          b[u] = 0;
          if constexpr (SEEN) b[u] = c < chunks ? reinterpret_cast<const SeenBits*>(srow)[c] : SeenBits(0);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int c = c0 + u * kStride + gl;
          const T* t = reinterpret_cast<const T*>(&r[u]);
#pragma unroll
          for (int q = 0; q < kVec; ++q) {
            f(c * kVec + q, pen_of(to_f32(t[q]), ((b[u] >> (8 * q)) & 0xffu) != 0), c < chunks);
          }
        }
      }
    } else {
      for (int base = 0; base < V; base += G * 32) {
        const int e = base + gl;
        const bool valid = e < V;
        float x = 0.f;
        if (valid) x = pen_of(to_f32(lrow[e]), SEEN && srow[e] != 0);
        f(e, x, valid);
      }
    }
  }

  // One strided sample of the row, the same in every warp (one vector or a
  // few elements per lane, spread over the row), for the histogram's bin
  // width: max, sum and count of the finite values.
  __device__ __forceinline__ void sample(float& m, float& sum, int& n) const {
    const int lane = threadIdx.x & 31;
    m = -__builtin_huge_valf();
    sum = 0.f;
    n = 0;
    auto add = [&](float x) {
      const bool fin = x >= -kFltMax && x <= kFltMax;
      m = fin ? fmaxf(m, x) : m;
      sum += fin ? x : 0.f;
      n += fin ? 1 : 0;
    };
    if (vec) {
      const int chunks = V / kVec;
      const int c = static_cast<int>((static_cast<int64_t>(lane) * chunks) >> 5);
      const uint4 r = reinterpret_cast<const uint4*>(lrow)[c];
      const T* t = reinterpret_cast<const T*>(&r);
#pragma unroll
      for (int q = 0; q < kVec; ++q) {
        bool seen = false;
        if constexpr (SEEN) seen = srow[c * kVec + q] != 0;
        add(pen_of(to_f32(t[q]), seen));
      }
    } else {
      for (int j = 0; j < kVec; ++j) {
        const int e = static_cast<int>((static_cast<int64_t>(lane * kVec + j) * V) / (32 * kVec));
        add(pen_of(to_f32(lrow[e]), SEEN && srow[e] != 0));
      }
    }
    m = warp_max(m);
    sum = warp_sum(sum);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(kFull, n, o);
  }
};

// Bins of one histogram: lane owns bins 8 * lane .. 8 * lane + 7.  Returns
// the first bin whose count, added to `base`, reaches k (-1 if none) and the
// counts before it and through it.
__device__ __forceinline__ int warp_pick_bin(const int* hist, int k, int base, int& above, int& total) {
  const int lane = threadIdx.x & 31;
  int c[8];
  int mine = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = hist[8 * lane + i];
    mine += c[i];
  }
  int run = warp_incl_scan(mine) - mine + base;
  int found = -1, f_above = 0, f_total = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (found < 0 && run + c[i] >= k) {
      found = 8 * lane + i;
      f_above = run;
      f_total = run + c[i];
    }
    run += c[i];
  }
  const unsigned bal = __ballot_sync(kFull, found >= 0);
  if (bal == 0u) return -1;
  const int src = __ffs(bal) - 1;
  above = __shfl_sync(kFull, f_above, src);
  total = __shfl_sync(kFull, f_total, src);
  return __shfl_sync(kFull, found, src);
}

// Softmax, top-p and the draw over <= 64 ranked candidates in one warp:
// rank lane in c0, rank lane + 32 in c1, their noise in n0 / n1.  Returns
// the sampled token.
__device__ int draw_top64(const SampleArgs& a, const RowParams& p, int row, uint64_t c0, uint64_t c1, float n0,
                          float n1) {
  const int lane = threadIdx.x & 31;
  const int V = a.vocab, k_eff = p.k_eff;
  const bool in0 = lane < k_eff, in1 = lane + 32 < k_eff;
  const float vtop = __shfl_sync(kFull, key_value(static_cast<uint32_t>(c0 >> 32)), 0);
  const float e0 = in0 ? expf(key_value(static_cast<uint32_t>(c0 >> 32)) - vtop) : 0.f;
  const float e1 = in1 ? expf(key_value(static_cast<uint32_t>(c1 >> 32)) - vtop) : 0.f;
  const float esum = warp_sum(e0) + warp_sum(e1);
  float p0 = in0 ? __fdiv_rn(e0, esum) : 0.f;
  float p1 = in1 ? __fdiv_rn(e1, esum) : 0.f;
  if (p.top_p < 1.f) {
    // cumulative mass in rank order, accumulated in double
    const double d0 = p0, d1 = p1;
    double i0 = d0, i1 = d1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y0 = __shfl_up_sync(kFull, i0, o);
      const double y1 = __shfl_up_sync(kFull, i1, o);
      if (lane >= o) {
        i0 += y0;
        i1 += y1;
      }
    }
    const double total0 = __shfl_sync(kFull, i0, 31);
    const double run0 = (i0 - d0) + d0;
    const double run1 = ((i1 - d1) + total0) + d1;
    if (in0 && __fsub_rn(static_cast<float>(run0), p0) > p.top_p) p0 = 0.f;
    if (in1 && __fsub_rn(static_cast<float>(run1), p1) > p.top_p) p1 = 0.f;
    const float norm = fmaxf(warp_sum(p0) + warp_sum(p1), 1.17549435e-38f);
    p0 = __fdiv_rn(p0, norm);
    p1 = __fdiv_rn(p1, norm);
  }
  float bv = -1.f;
  int br = k_eff;
  if (in0) argmax_merge(bv, br, __fdiv_rn(p0, n0), lane);
  if (in1) argmax_merge(bv, br, __fdiv_rn(p1, n1), lane + 32);
  warp_argmax(bv, br);
  if (a.probs != nullptr) {
    const int64_t base = static_cast<int64_t>(row) * V;
    if (in0) {
      a.probs[base + lane] = p0;
      a.ids[base + lane] = cand_token(c0);
    }
    if (in1) {
      a.probs[base + lane + 32] = p1;
      a.ids[base + lane + 32] = cand_token(c1);
    }
  }
  const int rank = br < k_eff ? br : 0;
  const uint64_t w0 = __shfl_sync(kFull, c0, rank & 31);
  const uint64_t w1 = __shfl_sync(kFull, c1, rank & 31);
  return cand_token(rank < 32 ? w0 : w1);
}

__device__ __forceinline__ void finish_row(const SampleArgs& a, int row, int token) {
  a.tokens[row] = token;
  if (a.update_seen && a.seen != nullptr) a.seen[row * a.seen_stride + token] = 1;
}

// One row in a group of G warps (warp wg of the group).  Returns false when
// the row needs the general path; only the group's warp 0 reports that.
template <typename T, int G, bool SEEN>
__device__ bool group_row(const SampleArgs& a, const RowParams& p, int row, int group, int wg, GroupShared<G>& gs) {
  const int V = a.vocab, lane = threadIdx.x & 31;
  const T* lrow = static_cast<const T*>(a.logits) + row * a.lstride;
  const uint8_t* srow = SEEN ? a.seen + row * a.seen_stride : nullptr;
  const int64_t pbase = static_cast<int64_t>(row) * V;
  const GroupRow<T, G, SEEN> src(lrow, srow, V, p.pen, wg * 32 + lane);

  if (!(p.temp > 0.f)) {
    // greedy: first argmax of the penalised logits
    float bv = -__builtin_huge_valf();
    int bi = 0x7fffffff;
    src.for_each([&](int e, float x, bool valid) {
      if (valid) argmax_merge(bv, bi, x, e);
    });
    warp_argmax(bv, bi);
    if (lane == 0) {
      gs.best_v[wg] = bv;
      gs.best_i[wg] = bi;
    }
    group_sync<G>(group);
    bv = gs.best_v[0];
    bi = gs.best_i[0];
#pragma unroll
    for (int w = 1; w < G; ++w) argmax_merge(bv, bi, gs.best_v[w], gs.best_i[w]);
    const int token = bi < V ? bi : 0;
    if (a.probs != nullptr) {
      for (int r = wg * 32 + lane; r < V; r += G * 32) {
        a.probs[pbase + r] = r == 0 ? 1.f : 0.f;
        a.ids[pbase + r] = r == 0 ? token : -1;
      }
    }
    if (wg == 0 && lane == 0) finish_row(a, row, token);
    return true;
  }
  const int k_eff = p.k_eff;
  if (k_eff > kFastK) return false;

  // the draw's noise for ranks lane and lane + 32 (the group's warp 0 draws)
  float n0 = 1.f, n1 = 1.f;
  if (wg == 0) {
    if (a.noise != nullptr) {
      n0 = lane < V ? a.noise[row * a.noise_stride + lane] : 1.f;
      n1 = lane + 32 < V ? a.noise[row * a.noise_stride + lane + 32] : 1.f;
    } else {
      n0 = exp_noise(p.seed, p.off, lane);
      n1 = exp_noise(p.seed, p.off, lane + 32);
    }
  }

  // bin width from a strided sample: w = (sample max - sample mean) / kGapBins
  float m, sum;
  int n;
  src.sample(m, sum, n);
  const float gap = n > 1 ? m - sum / static_cast<float>(n) : 0.f;
  if (!(gap > 1e-30f) || !(gap <= kFltMax)) return false;
  const float inv_w = kGapBins / gap;

  // bin position t = max(0, (m - x) / w + kBinsAbove), one rounding (fma) in every pass; it never
  // increases as x grows.  The first kBinsAbove bins hold the logits above the sample's max; t >= 255
  // (and NaN) is counted nowhere.
  auto tpos = [&](float x) { return __fmaf_rn(m - x, inv_w, kBinsAbove); };
  for (int i = wg * 32 + lane; i < kBins; i += G * 32) gs.hist[i] = 0;
  group_sync<G>(group);
  src.for_each([&](int, float x, bool valid) {
    const float t = tpos(x);
    if (valid && t < 255.f) atomicAdd(&gs.hist[static_cast<int>(fmaxf(t, 0.f))], 1);
  });
  group_sync<G>(group);
  int above = 0, total = 0;
  const int b1 = warp_pick_bin(gs.hist, k_eff, 0, above, total);
  if (b1 < 0) return false;
  float t_cut = static_cast<float>(b1 + 1);
  if (total > kFastK) {
    // 256 sub-bins of bin b1: t - b1 is exact (Sterbenz), so the split is monotone in x
    const float fb1 = static_cast<float>(b1);
    group_sync<G>(group);
    for (int i = wg * 32 + lane; i < kBins; i += G * 32) gs.hist[i] = 0;
    group_sync<G>(group);
    src.for_each([&](int, float x, bool valid) {
      const float t = tpos(x);
      if (valid && t < 255.f) {
        const float tc = fmaxf(t, 0.f);
        if (tc >= fb1 && tc < t_cut) atomicAdd(&gs.hist[static_cast<int>((tc - fb1) * 256.f)], 1);
      }
    });
    group_sync<G>(group);
    int above2 = 0;
    const int s2 = warp_pick_bin(gs.hist, k_eff, above, above2, total);
    if (s2 < 0 || total > kFastK) return false;
    t_cut = fb1 + static_cast<float>(s2 + 1) * (1.f / 256.f);  // exact: at most 16 significant bits
  }

  // ballot compaction of {t < t_cut} into the warp's slots; the largest logit left out
  int count = 0;
  float x_out = -__builtin_huge_valf();
  uint64_t* slots = gs.slots[wg];
  src.for_each([&](int e, float x, bool valid) {
    const float t = tpos(x);
    const bool take = valid && t < 255.f && fmaxf(t, 0.f) < t_cut;
    const unsigned bal = __ballot_sync(kFull, take);
    if (take) {
      const int slot = count + __popc(bal & ((1u << lane) - 1u));
      if (slot < kFastK) slots[slot] = (static_cast<uint64_t>(__float_as_uint(x)) << 32) | static_cast<uint32_t>(e);
    }
    count += __popc(bal);
    x_out = fmaxf(x_out, (valid && !take) ? x : -__builtin_huge_valf());
  });
  x_out = warp_max(x_out);
  if (lane == 0) {
    gs.count[wg] = count;
    gs.x_out[wg] = x_out;
  }
  if (a.probs != nullptr) {
    for (int r = k_eff + wg * 32 + lane; r < V; r += G * 32) {
      a.probs[pbase + r] = 0.f;
      a.ids[pbase + r] = -1;
    }
  }
  group_sync<G>(group);
  if (wg != 0) return true;

  // the group's warp 0: y and keys for the candidates, ranked in registers
  int total_count = 0;
  x_out = -__builtin_huge_valf();
  int w0 = -1, off0 = 0, w1 = -1, off1 = 0;
#pragma unroll
  for (int w = 0; w < G; ++w) {
    const int cw = gs.count[w];
    if (w0 < 0 && lane < total_count + cw) {
      w0 = w;
      off0 = lane - total_count;
    }
    if (w1 < 0 && lane + 32 < total_count + cw) {
      w1 = w;
      off1 = lane + 32 - total_count;
    }
    total_count += cw;
    x_out = fmaxf(x_out, gs.x_out[w]);
  }
  if (total_count > kFastK || total_count < k_eff) return false;  // the histogram counts rule both out
  uint64_t c0 = 0ull, c1 = 0ull;
  if (lane < total_count) {
    const uint64_t sl = gs.slots[w0][off0];
    c0 = cand_word(order_key(scaled<T>(a, p, __uint_as_float(static_cast<uint32_t>(sl >> 32)))),
                   static_cast<int>(sl & 0xffffffffu));
  }
  if (lane + 32 < total_count) {
    const uint64_t sl = gs.slots[w1][off1];
    c1 = cand_word(order_key(scaled<T>(a, p, __uint_as_float(static_cast<uint32_t>(sl >> 32)))),
                   static_cast<int>(sl & 0xffffffffu));
  }
  warp_sort64_desc(c0, c1);
  // a logit outside the candidates whose quotient ties the k-th value needs the general path
  // (x_out = -inf when nothing was left out; its quotient cannot tie a finite candidate)
  const uint64_t kth = __shfl_sync(kFull, (k_eff - 1) < 32 ? c0 : c1, (k_eff - 1) & 31);
  if (x_out > -__builtin_huge_valf() && order_key(scaled<T>(a, p, x_out)) >= static_cast<uint32_t>(kth >> 32)) {
    return false;
  }
  const int token = draw_top64(a, p, row, c0, c1, n0, n1);
  if (lane == 0) finish_row(a, row, token);
  return true;
}

// ---- the general path (whole CTA, keys in shared memory) ---------------------

struct BlockShared {
  int hist[256];
  float redf[kWarps];
  int redi[kWarps];
  double redd[kWarps];
  int digit, remaining, count;
};

template <typename T>
__device__ void block_row(const SampleArgs& a, int row, BlockShared& sh, uint64_t* s_cand, uint32_t* s_key) {
  const int tid = threadIdx.x;
  const int V = a.vocab;
  const RowParams p = row_params(a, row);
  const int k_eff = p.k_eff;
  const T* lrow = static_cast<const T*>(a.logits) + row * a.lstride;
  const uint8_t* srow = a.seen != nullptr ? a.seen + row * a.seen_stride : nullptr;

  for (int e = tid; e < V; e += kThreads) {
    const float x = penalised(to_f32(lrow[e]), srow != nullptr && srow[e] != 0, p.pen);
    s_key[e] = order_key(scaled<T>(a, p, x));
  }
  __syncthreads();

  // radix select of the k_eff-th largest key
  uint32_t tau = 0u;
  int n_cand = V;
  if (k_eff < V) {
    uint32_t prefix = 0u, mask = 0u;
    int remaining = k_eff;
    int eq_count = 0;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      sh.hist[tid] = 0;  // kThreads == 256 bins
      __syncthreads();
      for (int e = tid; e < V; e += kThreads) {
        const uint32_t k = s_key[e];
        if ((k & mask) == prefix) atomicAdd(&sh.hist[(k >> shift) & 255u], 1);
      }
      __syncthreads();
      const int h = sh.hist[tid];
      // suffix counts, elements with digit >= tid: an inclusive scan over the reversed bins
      const int incl = block_incl_scan(sh.hist[255 - tid], sh.redi);
      sh.hist[255 - tid] = incl;
      __syncthreads();
      const int suffix = sh.hist[tid];
      const int above = suffix - h;  // elements with digit > tid
      if (above < remaining && remaining <= suffix) {
        sh.digit = tid;
        sh.remaining = remaining - above;
        sh.count = h;
      }
      __syncthreads();
      const int digit = sh.digit;
      remaining = sh.remaining;
      eq_count = sh.count;
      prefix |= static_cast<uint32_t>(digit) << shift;
      mask |= 255u << shift;
      __syncthreads();
    }
    tau = prefix;
    n_cand = (k_eff - remaining) + eq_count;  // every key >= tau
  }

  // compact every key >= tau, then sort (value desc, id asc)
  if (tid == 0) sh.count = 0;
  __syncthreads();
  int n_pow2 = 1;
  while (n_pow2 < n_cand) n_pow2 <<= 1;
  for (int e = tid; e < V; e += kThreads) {
    const uint32_t k = s_key[e];
    if (k >= tau) s_cand[atomicAdd(&sh.count, 1)] = cand_word(k, e);
  }
  __syncthreads();
  for (int i = n_cand + tid; i < n_pow2; i += kThreads) s_cand[i] = 0ull;
  __syncthreads();
  for (int k = 2; k <= n_pow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n_pow2; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = s_cand[i], y = s_cand[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            s_cand[i] = y;
            s_cand[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }

  // softmax over the top-k values (rank order), then top-p
  const float v0 = key_value(static_cast<uint32_t>(s_cand[0] >> 32));
  // each thread owns a contiguous run of ranks so the cumulative sum is in rank order
  const int per = (k_eff + kThreads - 1) / kThreads;
  const int r0 = tid * per;
  const int r1 = min(k_eff, r0 + per);
  float e_local = 0.f;
  for (int r = r0; r < r1; ++r) e_local += expf(key_value(static_cast<uint32_t>(s_cand[r] >> 32)) - v0);
  const float esum = block_reduce_sum<float>(e_local, sh.redf);
  float kept_local = 0.f;
  if (p.top_p < 1.f) {
    double part = 0.0;
    for (int r = r0; r < r1; ++r)
      part += static_cast<double>(__fdiv_rn(expf(key_value(static_cast<uint32_t>(s_cand[r] >> 32)) - v0), esum));
    // exclusive scan of per-thread sums (double) across the block
    const int lane = tid & 31, warp = tid >> 5;
    double incl = part;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += y;
    }
    __syncthreads();
    if (lane == 31) sh.redd[warp] = incl;
    __syncthreads();
    double run = incl - part;
    for (int w = 0; w < warp; ++w) run += sh.redd[w];
    for (int r = r0; r < r1; ++r) {
      const float pr = __fdiv_rn(expf(key_value(static_cast<uint32_t>(s_cand[r] >> 32)) - v0), esum);
      run += static_cast<double>(pr);
      const float cum = static_cast<float>(run);
      const bool drop = __fsub_rn(cum, pr) > p.top_p;
      // keep the low word (token id) and store p in the high word for the draw
      const float keep = drop ? 0.f : pr;
      kept_local += keep;
      s_cand[r] = (static_cast<uint64_t>(__float_as_uint(keep)) << 32) | (s_cand[r] & 0xffffffffull);
    }
  } else {
    for (int r = r0; r < r1; ++r) {
      const float pr = __fdiv_rn(expf(key_value(static_cast<uint32_t>(s_cand[r] >> 32)) - v0), esum);
      s_cand[r] = (static_cast<uint64_t>(__float_as_uint(pr)) << 32) | (s_cand[r] & 0xffffffffull);
    }
  }
  float norm = 1.f;
  if (p.top_p < 1.f) {
    const float kept = block_reduce_sum<float>(kept_local, sh.redf);
    norm = fmaxf(kept, 1.17549435e-38f);
  }
  __syncthreads();

  // exponential race over ranks
  float bv = -1.f;
  int br = k_eff;
  const int64_t pbase = static_cast<int64_t>(row) * V;
  for (int r = r0; r < r1; ++r) {
    float pr = __uint_as_float(static_cast<uint32_t>(s_cand[r] >> 32));
    if (p.top_p < 1.f) pr = __fdiv_rn(pr, norm);
    const float e = a.noise != nullptr ? a.noise[row * a.noise_stride + r] : exp_noise(p.seed, p.off, r);
    argmax_merge(bv, br, __fdiv_rn(pr, e), r);
    if (a.probs != nullptr) {
      a.probs[pbase + r] = pr;
      a.ids[pbase + r] = cand_token(s_cand[r]);
    }
  }
  if (a.probs != nullptr) {
    for (int r = k_eff + tid; r < V; r += kThreads) {
      a.probs[pbase + r] = 0.f;
      a.ids[pbase + r] = -1;
    }
  }
  const int rank = block_argmax(bv, br, sh.redf, sh.redi);
  if (tid == 0) finish_row(a, row, cand_token(s_cand[rank < k_eff ? rank : 0]));
  __syncthreads();  // s_cand and s_key are reused by the next row
}

// Dynamic shared memory: [np2] candidates of the general path, then one
// region that holds the groups' histograms and slots during the group phase
// and the keys of a row on the general path afterwards.
__host__ __device__ constexpr size_t region_bytes(int vocab, size_t group_bytes) {
  return static_cast<size_t>(vocab) * 4 > group_bytes ? static_cast<size_t>(vocab) * 4 : group_bytes;
}

// kWarps / G rows per CTA, G warps per row.  Four CTAs per SM (at most 64 registers per thread, no
// spills; about 45 KB of shared memory each): the passes are bound by instruction latency, so more
// resident warps help (16384 x 3072 rows: 234 -> 179 us against two CTAs per SM).
template <typename T, int G>
__global__ void __launch_bounds__(kThreads, 4) sample_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ BlockShared bs;
  __shared__ int s_rest[kWarps];
  __shared__ int s_nrest;
  constexpr int kRows = kWarps / G;
  uint64_t* s_cand = reinterpret_cast<uint64_t*>(smem);
  uint8_t* region = smem + static_cast<size_t>(a.np2) * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = warp / G, wg = warp % G;
  if (threadIdx.x == 0) s_nrest = 0;
  __syncthreads();
  const int row = blockIdx.x * kRows + group;
  if (row < a.rows) {
    const RowParams p = row_params(a, row);
    GroupShared<G>& gs = reinterpret_cast<GroupShared<G>*>(region)[group];
    const bool done = a.seen != nullptr ? group_row<T, G, true>(a, p, row, group, wg, gs)
                                        : group_row<T, G, false>(a, p, row, group, wg, gs);
    if (!done && wg == 0 && lane == 0) s_rest[atomicAdd(&s_nrest, 1)] = row;
  }
  __syncthreads();
  const int nrest = s_nrest;
  for (int i = 0; i < nrest; ++i) block_row<T>(a, s_rest[i], bs, s_cand, reinterpret_cast<uint32_t*>(region));
}

template <typename T, int G>
int launch_g(SampleArgs a, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(a.np2) * 8 + region_bytes(a.vocab, sizeof(GroupShared<G>) * (kWarps / G));
  // the static shared memory counts against the default 48 KB as well
  if (smem > 32 * 1024) {
    cudaFuncSetAttribute(sample_kernel<T, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  }
  constexpr int kRows = kWarps / G;
  sample_kernel<T, G><<<(a.rows + kRows - 1) / kRows, kThreads, smem, s>>>(a);
  return check_launch("sample_rows");
}

// Warps per row: enough that rows x G reaches eight warps per SM, at most 8.
template <typename T>
int launch(SampleArgs a, cudaStream_t s) {
  const int want = (8 * num_sms() + a.rows - 1) / a.rows;
  if (want >= 5) return launch_g<T, 8>(a, s);
  if (want >= 3) return launch_g<T, 4>(a, s);
  if (want >= 2) return launch_g<T, 2>(a, s);
  return launch_g<T, 1>(a, s);
}

int run(SampleArgs a, int dtype, void* stream) {
  if (!a.logits || !a.temp || !a.top_k || !a.top_p || !a.tokens) return NQT_ERR_ARG;
  if (a.rows < 1 || a.vocab < 1) return NQT_ERR_ARG;
  if (a.vocab > kMaxVocab) return NQT_ERR_CAPACITY;
  if ((a.probs == nullptr) != (a.ids == nullptr)) return NQT_ERR_ARG;
  if (a.update_seen && a.seen == nullptr) return NQT_ERR_ARG;
  int np2 = 1;
  while (np2 < a.vocab) np2 <<= 1;
  a.np2 = np2;
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case NQT_BF16: return launch<__nv_bfloat16>(a, s);
    case NQT_F16: return launch<__half>(a, s);
    case NQT_F32: return launch<float>(a, s);
    default: return NQT_ERR_ARG;
  }
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_sample_rows(const void* logits, int logits_dtype, int64_t logits_stride, int rows, int vocab,
                               const float* temperature, const int32_t* top_k, const float* top_p,
                               const int64_t* seed, const int64_t* offset, int64_t offset_stride,
                               const float* repetition_penalty, uint8_t* seen, int64_t seen_stride,
                               int update_seen, int round_scaled_to_input, int64_t* tokens_out, float* probs_out,
                               int32_t* ids_out, int32_t* status, void* stream) {
  if (!seed || !offset) return NQT_ERR_ARG;
  SampleArgs a{logits, logits_stride, rows, vocab, 0, temperature, top_k, top_p, seed, offset, offset_stride,
               nullptr, 0, repetition_penalty, seen, seen_stride, update_seen, round_scaled_to_input, tokens_out,
               probs_out, ids_out, status};
  return run(a, logits_dtype, stream);
}

extern "C" int nqt_sample_rows_noise(const void* logits, int logits_dtype, int64_t logits_stride, int rows,
                                     int vocab, const float* temperature, const int32_t* top_k, const float* top_p,
                                     const float* noise, int64_t noise_stride, const float* repetition_penalty,
                                     uint8_t* seen, int64_t seen_stride, int update_seen, int round_scaled_to_input,
                                     int64_t* tokens_out, float* probs_out, int32_t* ids_out, int32_t* status,
                                     void* stream) {
  if (!noise) return NQT_ERR_ARG;
  SampleArgs a{logits, logits_stride, rows, vocab, 0, temperature, top_k, top_p, nullptr, nullptr, 0,
               noise, noise_stride, repetition_penalty, seen, seen_stride, update_seen, round_scaled_to_input,
               tokens_out, probs_out, ids_out, status};
  return run(a, logits_dtype, stream);
}
