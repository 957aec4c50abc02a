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
// Work split: a group of G = 1, 2, 4 or 8 warps takes a row (the host picks G so that rows x G fill
// the GPU and the row fits the group's lanes).  The fast path (fast_row, below) reads the row once,
// cuts it to a few hundred candidates with a count-guaranteed threshold, takes the exact penalty and
// division only for those, and ranks at most 128 of them in one warp.  Rows it cannot settle (k > 64,
// a penalty below 1 with a seen mask, NaN or +inf logits, unaligned or oversized rows, a candidate
// capacity overflow, or a rounding tie at the k-th value) are marked, and after the fast phase the
// whole CTA takes each of them through the exact general path: a 4-pass radix select (8 bits per
// pass) of the k-th key, compaction of every key >= it and a bitonic sort in shared memory.
//
// Reference semantics: sample_logits_stateless / _cpu_sample_row
// (model/sampling.py:55-95, 127-225).
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace nqt {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;  // rows per CTA
constexpr int kMaxVocab = 16384;
constexpr int kFastK = 64;        // largest top-k of the fast path
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

// Exp(1) noise of draw rank r: one Philox4x32-10 block keyed by the row's seed, with counter
// (r / 128 * 32 + r % 32, 0, offset) and output word (r / 32) % 4, so one block serves ranks l, l + 32,
// l + 64 and l + 96 (a warp's lane l draws ranks l and l + 32 from one block).
__device__ __forceinline__ uint4 noise_block(int64_t seed, int64_t offset, int counter) {
  const uint4 ctr = make_uint4(static_cast<uint32_t>(counter), 0u, static_cast<uint32_t>(offset),
                               static_cast<uint32_t>(static_cast<uint64_t>(offset) >> 32));
  const uint2 key = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(static_cast<uint64_t>(seed) >> 32));
  return philox4x32_10(ctr, key);
}

__device__ __forceinline__ float exp_of_word(uint32_t w) {
  const float u = (static_cast<float>(w >> 8) + 0.5f) * 5.9604644775390625e-8f;  // (0, 1)
  return -logf(u);
}

__device__ __forceinline__ float exp_noise(int64_t seed, int64_t offset, int rank) {
  const uint4 r = noise_block(seed, offset, (rank >> 7) * 32 + (rank & 31));
  const int word = (rank >> 5) & 3;
  return exp_of_word(word == 0 ? r.x : (word == 1 ? r.y : (word == 2 ? r.z : r.w)));
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

// Bitonic sort (descending) of 64 keys held two per lane (rank i in lane i % 32, slot i / 32), in the
// flip form of warp_sort64_desc_f32 (one lower-lane predicate per step).
__device__ __forceinline__ void warp_sort64_desc(uint64_t& v0, uint64_t& v1) {
  const int lane = threadIdx.x & 31;
  auto cmp = [&](int dist, int bit) {
    const uint64_t p0 = __shfl_xor_sync(kFull, v0, dist);
    const uint64_t p1 = __shfl_xor_sync(kFull, v1, dist);
    const bool lower = (lane & bit) == 0;
    v0 = (lower == (p0 > v0)) ? p0 : v0;
    v1 = (lower == (p1 > v1)) ? p1 : v1;
  };
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
    cmp(k - 1, k >> 1);
#pragma unroll
    for (int j = k >> 2; j > 0; j >>= 1) cmp(j, j);
  }
  const uint64_t r0 = __shfl_sync(kFull, v1, 31 - lane);
  const uint64_t r1 = __shfl_sync(kFull, v0, 31 - lane);
  v0 = v0 > r0 ? v0 : r0;
  v1 = v1 < r1 ? v1 : r1;
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) cmp(j, j);
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

// ---- the fast path ----------------------------------------------------------
// A group of G warps (1, 2, 4 or 8) takes one row; its lanes hold the whole row in registers as
// 16-byte vectors (vector c in group lane c % (32 G), slot c / (32 G)), so the row crosses HBM once
// and every later pass runs on registers or on a few hundred candidates in shared memory.
//
//   cut 1   The row is split into 64 chunks (by lane and slot).  tau0 = the k-th largest chunk
//           maximum: the k chunks whose maxima reach tau0 hold at least k elements >= tau0, so the
//           raw top-k lies in C = {x >= tau0}.  A repetition penalty >= 1 only lowers a logit, so C
//           also holds the top-k of the penalised row whenever the check below passes.  The maxima
//           come from packed (x2) NaN-propagating max instructions on the raw vectors; for 2-byte
//           logits tau0 is found by bisection on their 16-bit order keys, else by a warp sort.
//   prefilter  A vector whose packed maximum is below tau0 holds no candidate; the others (about
//           a quarter) are copied to shared memory, then expanded element by element with warp
//           ballots into C (at most 256).
//   rank    2-byte logits whose y is not rounded to the logits type: all of C (at most 192) is ranked
//           with 32-bit keys in one warp sort (the ranking block in fast_row has its checks); the steps below
//           are the path of fp32 and y-rounded rows.
//   exact   Only the candidates read their seen-mask byte and take the exact penalty; when C has
//           more than 64, tau1 = the k-th largest of the 64 lane-local top-2 values narrows it to
//           F = {x_pen >= tau1} (at least k), else F = C.  y = x_pen / T for F only; F is sorted in
//           one warp's registers (value desc, token id asc).
//   check   Every element outside F has x_pen <= x_out = max(largest penalised candidate left out,
//           largest input value below tau0).  If y(x_out) does not stay strictly below the k-th
//           value, or any capacity above overflows, the row goes to the exact general path.
// Greedy rows are the k = 1 case with y = x_pen.
constexpr int kChunks = 64;    // chunk maxima behind cut 1
constexpr int kCvCap = 160;    // candidate vectors per row
constexpr int kCandCap = 256;  // candidate elements per row

// Vectors per lane of the register-resident row, per group size (V <= 32 G kVpl * elements/vector).
template <int G>
struct Vpl {
  static constexpr int value = G == 1 ? 12 : (G == 2 ? 8 : 4);
};

// Packed-vector helpers per element type: a 16-byte vector is 8 bf16 / 8 fp16 / 4 fp32.
template <typename T>
struct Lanes;

__device__ __forceinline__ uint32_t u32_of(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ uint32_t u32_of(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __nv_bfloat162 bf2_of(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ __half2 h2_of(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ float max_nan_f32(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

template <>
struct Lanes<__nv_bfloat16> {
  static constexpr int kVec = 8;
  static constexpr uint32_t kNegInf = 0xFF80FF80u;
  // two partial maxima (NaN-propagating) of the vector's 8 elements
  static __device__ __forceinline__ uint32_t vmax(const uint4& v) {
    return u32_of(__hmax2_nan(__hmax2_nan(bf2_of(v.x), bf2_of(v.y)), __hmax2_nan(bf2_of(v.z), bf2_of(v.w))));
  }
  static __device__ __forceinline__ uint32_t pmax(uint32_t a, uint32_t b) {
    return u32_of(__hmax2_nan(bf2_of(a), bf2_of(b)));
  }
  static __device__ __forceinline__ float fold(uint32_t m) {
    const __nv_bfloat162 h = bf2_of(m);
    return __bfloat162float(__hmax_nan(h.x, h.y));
  }
  static __device__ __forceinline__ uint32_t splat(float t) { return u32_of(__float2bfloat162_rn(t)); }
  static __device__ __forceinline__ bool any_ge(uint32_t m, uint32_t t2) {
    return __hge2_mask(bf2_of(m), bf2_of(t2)) != 0u;
  }
  static __device__ __forceinline__ uint32_t any_ge_mask(uint32_t m, uint32_t t2) {
    return __hge2_mask(bf2_of(m), bf2_of(t2));
  }
  static __device__ __forceinline__ float elem(const uint4& v, int e) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&v)[e]);
  }
  // element e (a runtime index) without indexing into a local array
  static __device__ __forceinline__ float elem_dyn(const uint4& v, int e) {
    const uint32_t w = (e & 4) ? ((e & 2) ? v.w : v.z) : ((e & 2) ? v.y : v.x);
    return __uint_as_float((e & 1) ? (w & 0xFFFF0000u) : (w << 16));
  }
  // largest bf16 value below t (t a finite bf16 value)
  static __device__ __forceinline__ float prev(float t) {
    if (t == 0.f) return -__bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(1)));
    const unsigned short b = __bfloat16_as_ushort(__float2bfloat16_rn(t));
    return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(t > 0.f ? b - 1 : b + 1)));
  }
  // a bf16 value is exact in the top 16 bits of its fp32 pattern: bits 12-15 are zero
  static constexpr uint32_t kExactLow = 0xFu;
  // 16-bit order key of a bf16 value held in a float (larger value, larger key) and its inverse
  static __device__ __forceinline__ uint32_t key16(float v) {
    const uint32_t b = __float_as_uint(v) >> 16;
    return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  }
  static __device__ __forceinline__ float value16(uint32_t k) {
    const uint32_t b = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return __uint_as_float(b << 16);
  }
};

template <>
struct Lanes<__half> {
  static constexpr int kVec = 8;
  static constexpr uint32_t kNegInf = 0xFC00FC00u;
  static __device__ __forceinline__ uint32_t vmax(const uint4& v) {
    return u32_of(__hmax2_nan(__hmax2_nan(h2_of(v.x), h2_of(v.y)), __hmax2_nan(h2_of(v.z), h2_of(v.w))));
  }
  static __device__ __forceinline__ uint32_t pmax(uint32_t a, uint32_t b) { return u32_of(__hmax2_nan(h2_of(a), h2_of(b))); }
  static __device__ __forceinline__ float fold(uint32_t m) {
    const __half2 h = h2_of(m);
    return __half2float(__hmax_nan(h.x, h.y));
  }
  static __device__ __forceinline__ uint32_t splat(float t) { return u32_of(__float2half2_rn(t)); }
  static __device__ __forceinline__ bool any_ge(uint32_t m, uint32_t t2) { return __hge2_mask(h2_of(m), h2_of(t2)) != 0u; }
  static __device__ __forceinline__ uint32_t any_ge_mask(uint32_t m, uint32_t t2) { return __hge2_mask(h2_of(m), h2_of(t2)); }
  static __device__ __forceinline__ float elem(const uint4& v, int e) {
    return __half2float(reinterpret_cast<const __half*>(&v)[e]);
  }
  static __device__ __forceinline__ float elem_dyn(const uint4& v, int e) {
    const uint32_t w = (e & 4) ? ((e & 2) ? v.w : v.z) : ((e & 2) ? v.y : v.x);
    return __half2float(__ushort_as_half(static_cast<unsigned short>((e & 1) ? (w >> 16) : (w & 0xFFFFu))));
  }
  static __device__ __forceinline__ float prev(float t) {
    if (t == 0.f) return -__half2float(__ushort_as_half(static_cast<unsigned short>(1)));
    const unsigned short b = __half_as_ushort(__float2half_rn(t));
    return __half2float(__ushort_as_half(static_cast<unsigned short>(t > 0.f ? b - 1 : b + 1)));
  }
  // an fp16 value converted to fp32 has its low 13 mantissa bits zero: bit 12 is zero
  static constexpr uint32_t kExactLow = 0x1u;
  // 16-bit order key of an fp16 value held in a float (larger value, larger key) and its inverse
  static __device__ __forceinline__ uint32_t key16(float v) {
    const uint32_t b = __half_as_ushort(__float2half_rn(v));
    return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  }
  static __device__ __forceinline__ float value16(uint32_t k) {
    const uint32_t b = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
  }
};

template <>
struct Lanes<float> {
  static constexpr int kVec = 4;
  static constexpr uint32_t kNegInf = 0xFF800000u;
  static __device__ __forceinline__ uint32_t vmax(const uint4& v) {
    return __float_as_uint(max_nan_f32(max_nan_f32(__uint_as_float(v.x), __uint_as_float(v.y)),
                                       max_nan_f32(__uint_as_float(v.z), __uint_as_float(v.w))));
  }
  static __device__ __forceinline__ uint32_t pmax(uint32_t a, uint32_t b) {
    return __float_as_uint(max_nan_f32(__uint_as_float(a), __uint_as_float(b)));
  }
  static __device__ __forceinline__ float fold(uint32_t m) { return __uint_as_float(m); }
  static __device__ __forceinline__ uint32_t splat(float t) { return __float_as_uint(t); }
  static __device__ __forceinline__ bool any_ge(uint32_t m, uint32_t t) { return __uint_as_float(m) >= __uint_as_float(t); }
  static __device__ __forceinline__ float elem(const uint4& v, int e) { return reinterpret_cast<const float*>(&v)[e]; }
  static __device__ __forceinline__ float elem_dyn(const uint4& v, int e) {
    return __uint_as_float((e & 2) ? ((e & 1) ? v.w : v.z) : ((e & 1) ? v.y : v.x));
  }
  static __device__ __forceinline__ float prev(float t) {
    if (t == 0.f) return -__uint_as_float(1u);
    const uint32_t b = __float_as_uint(t);
    return __uint_as_float(t > 0.f ? b - 1u : b + 1u);
  }
};

// ---- 32-bit rank keys (2-byte logits) ---------------------------------------
// A candidate's key is the top 20 bits of the order key of its penalised value, then 4095 - token
// (V <= 4096).  A bf16 or fp16 value converted to fp32 fits the 20 bits exactly, so for unpenalised
// candidates equal keys mean equal values and the token breaks the tie as the reference does; a penalised
// value that the 20 bits cut is moved one step towards its true position (it then keeps its order against
// every exact key) and is marked inexact by its low bits.
constexpr int kRankMaxVocab = 4096;
constexpr int kRankCap = 192;  // candidates ranked: 128 at once, the rest merged into the top 64

__device__ __forceinline__ uint32_t kmax(uint32_t a, uint32_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint32_t kmin(uint32_t a, uint32_t b) { return a < b ? a : b; }

// Descending bitonic sort of the 32 E keys of a warp, key i = lane * E + e in slot e.  Every comparator
// keeps the larger key at the lower index: merge kk opens with the flip comparator (i, i ^ (kk - 1)),
// then half-cleaners at kk / 4 .. 1; distances below E stay inside a lane.
template <int E>
__device__ __forceinline__ void warp_sort_desc(uint32_t (&v)[E]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 2; kk <= 32 * E; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      const bool flip = j == (kk >> 1);
      const int d = flip ? kk - 1 : j;
      if (d < E) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int f = e ^ d;
          if (f > e) {
            const uint32_t x = v[e], y = v[f];
            v[e] = kmax(x, y);
            v[f] = kmin(x, y);
          }
        }
      } else {
        // partner lane lane ^ (d / E); a flip comparator pairs slot e with the partner's slot E - 1 - e
        const bool lower = (lane & (j / E)) == 0;
        uint32_t pv[E];
#pragma unroll
        for (int e = 0; e < E; ++e) pv[e] = __shfl_xor_sync(kFull, v[flip ? E - 1 - e : e], d / E);
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = lower ? kmax(v[e], pv[e]) : kmin(v[e], pv[e]);
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ bool key_exact(uint32_t h) {  // h = 20-bit key part
  const uint32_t bits = (h & 0x80000u) ? h : (~h & 0xFFFFFu);  // the value's own top 20 bits (sign aside)
  return (bits & Lanes<T>::kExactLow) == 0u;
}

// the value whose 20-bit key part is h, exact when key_exact(h)
__device__ __forceinline__ float key20_value(uint32_t h) {
  return key_value((h << 12) | ((h & 0x80000u) ? 0u : 0xFFFu));
}

// key of a penalised value x of a 2-byte row (inexact only where `penalised`)
template <typename T>
__device__ __forceinline__ uint32_t rank_key(float x, bool pen_applied, int token) {
  const uint32_t ok32 = order_key(x);
  uint32_t h = ok32 >> 12;
  const bool pos = (ok32 & 0x80000000u) != 0u;
  if (pen_applied && key_exact<T>(h) && (ok32 & 0xFFFu) != (pos ? 0u : 0xFFFu)) h = pos ? (h | 1u) : (h & ~1u);
  return (h << 12) | (4095u - static_cast<uint32_t>(token));
}

template <int G>
struct FastShared {
  uint4 cv[kCvCap];     // candidate vectors
  int cvi[kCvCap];      // their vector index in the row
  float cx[kCandCap];   // candidate values (raw)
  int cid[kCandCap];    // candidate token ids
  float fx[2 * kFastK];  // the narrowed set F: penalised values
  int fid[2 * kFastK];   // and token ids
  float cm[kChunks];    // chunk maxima (groups of more than one warp)
  int wsum[G];          // candidate vectors per warp
  float tau0;
  int bad;
};

// Named barrier 1 + group over the group's G * 32 threads (immediate operands, so the CTA reserves only
// the barriers it uses); a single warp only needs __syncwarp.
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

// Bitonic sort (descending) of 64 floats held two per lane (rank i in lane i % 32, slot i / 32), in the
// form where every comparator keeps the larger value at the lower index: stage k opens with a flip
// comparator between i and i ^ (k - 1) inside each k-block, then half-cleaners at distances k/4 .. 1,
// so one predicate per step (the pair's lower lane) serves both slots.  Stage 64's flip pairs rank i
// with rank 63 - i across the slots.
__device__ __forceinline__ void warp_sort64_desc_f32(float& v0, float& v1) {
  const int lane = threadIdx.x & 31;
  auto cmp = [&](int dist, int bit) {
    const float p0 = __shfl_xor_sync(kFull, v0, dist);
    const float p1 = __shfl_xor_sync(kFull, v1, dist);
    const bool lower = (lane & bit) == 0;
    v0 = lower ? fmaxf(v0, p0) : fminf(v0, p0);
    v1 = lower ? fmaxf(v1, p1) : fminf(v1, p1);
  };
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
    cmp(k - 1, k >> 1);
#pragma unroll
    for (int j = k >> 2; j > 0; j >>= 1) cmp(j, j);
  }
  const float r0 = __shfl_sync(kFull, v1, 31 - lane);
  const float r1 = __shfl_sync(kFull, v0, 31 - lane);
  v0 = fmaxf(v0, r0);
  v1 = fminf(v1, r1);
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) cmp(j, j);
}

// Value of rank r of a 64-entry warp sort (held two per lane).
__device__ __forceinline__ float rank_value(float v0, float v1, int r) {
  return __shfl_sync(kFull, r < 32 ? v0 : v1, r & 31);
}

// Top 64 of two descending 64-entry warp sorts (a, b; rank i in lane i % 32, slot i / 32), sorted into a:
// max(a[i], b[63 - i]) is a bitonic sequence holding the 64 largest, then a descending bitonic merge.
__device__ __forceinline__ void warp_merge64_desc(uint64_t& a0, uint64_t& a1, uint64_t b0, uint64_t b1) {
  const int lane = threadIdx.x & 31;
  const uint64_t r0 = __shfl_sync(kFull, b1, 31 - lane);  // b[63 - lane]
  const uint64_t r1 = __shfl_sync(kFull, b0, 31 - lane);  // b[31 - lane]
  a0 = a0 > r0 ? a0 : r0;
  a1 = a1 > r1 ? a1 : r1;
  if (a0 < a1) {
    const uint64_t t = a0;
    a0 = a1;
    a1 = t;
  }
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) {
    const uint64_t p0 = __shfl_xor_sync(kFull, a0, j);
    const uint64_t p1 = __shfl_xor_sync(kFull, a1, j);
    const bool lower = (lane & j) == 0;
    a0 = lower ? (a0 > p0 ? a0 : p0) : (a0 < p0 ? a0 : p0);
    a1 = lower ? (a1 > p1 ? a1 : p1) : (a1 < p1 ? a1 : p1);
  }
}

// Candidate elements of one 16-byte vector that reach tau: bit e set for element e.
template <typename T>
__device__ __forceinline__ uint32_t vec_take_mask(const uint4& v, float tau, uint32_t tau2) {
  if constexpr (sizeof(T) == 2) {
    using L = Lanes<T>;
    (void)tau;
    uint32_t bits = 0u;
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t m = L::any_ge_mask(w[q], tau2);  // 0xFFFF in each half that reaches tau
      bits |= ((m & 1u) | ((m >> 15) & 2u)) << (2 * q);
    }
    return bits;
  } else {
    (void)tau2;
    uint32_t bits = 0u;
#pragma unroll
    for (int e = 0; e < 4; ++e) bits |= (Lanes<T>::elem(v, e) >= tau ? 1u : 0u) << e;
    return bits;
  }
}

// One row on the fast path, group of G warps (this is warp wg).  Returns false when the row needs the
// general path; every warp of the group returns the same value until the group's warp 0 works alone.
template <typename T, int G, bool SEEN>
__device__ bool fast_row(const SampleArgs& a, RowParams p, int row, int group, int wg, FastShared<G>& fs) {
  using L = Lanes<T>;
  constexpr int kVpl = Vpl<G>::value;
  constexpr int kVec = L::kVec;
  const int V = a.vocab, lane = threadIdx.x & 31;
  const int gl = wg * 32 + lane;  // lane within the group
  const T* lrow = static_cast<const T*>(a.logits) + row * a.lstride;
  const uint4* vrow = reinterpret_cast<const uint4*>(lrow);
  const int nvec = V / kVec;
  const bool greedy = !(p.temp > 0.f);
  if (greedy) p.k_eff = 1;
  // uniform per row: what the fast path cannot take
  if (p.k_eff > kFastK || (SEEN && p.pen < 1.f) || V % kVec != 0 || nvec > G * 32 * kVpl ||
      (reinterpret_cast<uintptr_t>(lrow) & 15u) != 0)
    return false;
  const int k = p.k_eff;

  // ---- stream the row once: packed maxima per vector and per chunk (the vectors are not kept)
  uint32_t vm[kVpl];
  {
    uint4 v[kVpl];
#pragma unroll
    for (int j = 0; j < kVpl; ++j) {
      const int c = gl + j * G * 32;
      v[j] = c < nvec ? vrow[c] : make_uint4(L::kNegInf, L::kNegInf, L::kNegInf, L::kNegInf);
    }
#pragma unroll
    for (int j = 0; j < kVpl; ++j) vm[j] = L::vmax(v[j]);
  }
  // the draw's noise (ranks lane and lane + 32 from one Philox block) while the loads are in flight
  float n0 = 1.f, n1 = 1.f;
  if (!greedy && wg == 0) {
    if (a.noise != nullptr) {
      n0 = lane < V ? a.noise[row * a.noise_stride + lane] : 1.f;
      n1 = lane + 32 < V ? a.noise[row * a.noise_stride + lane + 32] : 1.f;
    } else {
      const uint4 r = noise_block(p.seed, p.off, lane);
      n0 = exp_of_word(r.x);
      n1 = exp_of_word(r.y);
    }
  }
  uint32_t cm_even = L::kNegInf, cm_odd = L::kNegInf;
#pragma unroll
  for (int j = 0; j < kVpl; ++j) {
    if (j & 1) cm_odd = L::pmax(cm_odd, vm[j]); else cm_even = L::pmax(cm_even, vm[j]);
  }
  float c0, c1;  // this lane's share of the 64 chunk maxima (G == 1: two per lane)
  if constexpr (G == 1) {
    c0 = L::fold(cm_even);
    c1 = L::fold(cm_odd);
  } else {
    float m = L::fold(L::pmax(cm_even, cm_odd));
    constexpr int kLanesPerChunk = G / 2;  // 64 chunks over 32 G lanes
#pragma unroll
    for (int o = 1; o < kLanesPerChunk; o <<= 1) m = max_nan_f32(m, __shfl_xor_sync(kFull, m, o));
    if (gl % kLanesPerChunk == 0) fs.cm[gl / kLanesPerChunk] = m;
    group_sync<G>(group);
    c0 = fs.cm[lane];
    c1 = fs.cm[lane + 32];
  }

  // ---- cut 1: tau0 = k-th largest chunk maximum (every warp of the group sorts the same 64 values)
  const bool odd = (c0 != c0) || (c1 != c1) || c0 == __builtin_huge_valf() || c1 == __builtin_huge_valf();
  if (__any_sync(kFull, odd)) return false;  // NaN or +inf: the general path handles them
  float tau0;
  if constexpr (sizeof(T) == 2) {
    // the chunk maxima are exact 2-byte values: bisection on their 16-bit order keys, counting the keys at
    // or above each candidate over the warp; the result is the largest key with at least k keys >= it
    const uint32_t k0 = L::key16(c0), k1 = L::key16(c1);
    uint32_t prefix = 0u;
#pragma unroll
    for (int bit = 15; bit >= 0; --bit) {
      const uint32_t cand = prefix | (1u << bit);
      const int cnt = static_cast<int>(__reduce_add_sync(kFull, (k0 >= cand ? 1u : 0u) + (k1 >= cand ? 1u : 0u)));
      if (cnt >= k) prefix = cand;
    }
    tau0 = L::value16(prefix);
  } else {
    warp_sort64_desc_f32(c0, c1);
    tau0 = rank_value(c0, c1, k - 1);
  }
  if (!(tau0 > -__builtin_huge_valf())) return false;
  const uint32_t tau2 = L::splat(tau0);
  // the candidates' seen-mask bytes come from L2 later: start pulling the row's lines in now
  if constexpr (SEEN) {
    if (wg == 0) {
      const uint8_t* srow = a.seen + row * a.seen_stride;
      for (int off = lane * 128; off < V; off += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(srow + off));
    }
  }

  // ---- prefilter: vectors holding an element >= tau0 are read again (L1 / L2) into shared memory
  uint32_t take = 0u;
#pragma unroll
  for (int j = 0; j < kVpl; ++j) take |= (gl + j * G * 32 < nvec && L::any_ge(vm[j], tau2) ? 1u : 0u) << j;
  const int mine = __popc(take);
  const int incl = warp_incl_scan(mine);
  int base = incl - mine, total = __shfl_sync(kFull, incl, 31);
  if constexpr (G > 1) {
    if (lane == 31) fs.wsum[wg] = incl;
    group_sync<G>(group);
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < G; ++w) {
      const int t = fs.wsum[w];
      before += w < wg ? t : 0;
      all += t;
    }
    base += before;
    total = all;
  }
  if (total > kCvCap) return false;
#pragma unroll
  for (int j = 0; j < kVpl; ++j) {
    if (take & (1u << j)) {
      const int c = gl + j * G * 32;
      fs.cv[base] = vrow[c];
      fs.cvi[base] = c;
      ++base;
    }
  }
  group_sync<G>(group);
  if (wg != 0) return true;  // the group's warp 0 finishes the row

  // ---- expand the candidate vectors into C = {x >= tau0}: per-lane counts, one scan, scatter
  int n_cand = 0;
  for (int i0 = 0; i0 < total; i0 += 32) {
    const int i = i0 + lane;
    const bool ok = i < total;
    const uint4 cvv = ok ? fs.cv[i] : make_uint4(L::kNegInf, L::kNegInf, L::kNegInf, L::kNegInf);
    const int e0 = ok ? fs.cvi[i] * kVec : 0;
    uint32_t bits = vec_take_mask<T>(cvv, tau0, tau2);
    const int cnt = __popc(bits);
    const int inc = warp_incl_scan(cnt);
    int pos = n_cand + inc - cnt;
    n_cand += __shfl_sync(kFull, inc, 31);
    while (bits) {
      const int e = __ffs(bits) - 1;
      bits &= bits - 1u;
      if (pos < kCandCap) {
        fs.cx[pos] = L::elem_dyn(cvv, e);
        fs.cid[pos] = e0 + e;
      }
      ++pos;
    }
  }
  if (n_cand > kCandCap) return false;
  __syncwarp();

  if constexpr (sizeof(T) == 2) {
    if (!a.round_scaled && V <= kRankMaxVocab) {
      // ---- rank C with 32-bit keys: one 128-key sort (4 keys per lane, rank r in lane r / 4, slot
      // r % 4); candidates 128-191 replace ranks 64-127 and the top 64 is sorted again
      if (n_cand > kRankCap) return false;
      const uint8_t* srow = SEEN ? a.seen + row * a.seen_stride : nullptr;
      uint32_t key[4];
      auto load_keys = [&](int i0, int step, bool use) {
        float x[4];
        int tok[4];
        uint8_t sb[4] = {0, 0, 0, 0};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = i0 + e * step;
          const bool in = use && i < n_cand;
          x[e] = in ? fs.cx[i] : 0.f;
          tok[e] = in ? fs.cid[i] : 0;
          if constexpr (SEEN) sb[e] = in ? srow[tok[e]] : 0;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (SEEN) {
            if (__any_sync(kFull, sb[e] != 0)) x[e] = penalised(x[e], sb[e] != 0, p.pen);
          }
          if (use) key[e] = i0 + e * step < n_cand ? rank_key<T>(x[e], sb[e] != 0, tok[e]) : 0u;
        }
      };
      load_keys(lane, 32, true);
      warp_sort_desc<4>(key);
      uint32_t key64 = __shfl_sync(kFull, key[0], 16);  // rank 64: the neighbour of rank 63 when k = 64
      if (n_cand > 128) {
        load_keys(128 + (lane - 16) * 4, 1, lane >= 16);
        warp_sort_desc<4>(key);
        key64 = kmax(key64, __shfl_sync(kFull, key[0], 16));  // the largest key left out
      }
      // ranks lane and lane + 32
      uint32_t r0, r1;
      {
        uint32_t a0[4], a1[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a0[e] = __shfl_sync(kFull, key[e], lane >> 2);
          a1[e] = __shfl_sync(kFull, key[e], 8 + (lane >> 2));
        }
        const int slot = lane & 3;
        r0 = slot == 0 ? a0[0] : (slot == 1 ? a0[1] : (slot == 2 ? a0[2] : a0[3]));
        r1 = slot == 0 ? a1[0] : (slot == 1 ? a1[1] : (slot == 2 ? a1[2] : a1[3]));
      }
      // check: the k-th penalised value reaches tau0 (everything outside C lies below tau0)
      {
        const uint32_t hk = __shfl_sync(kFull, (k - 1) < 32 ? r0 : r1, (k - 1) & 31) >> 12;
        const uint32_t ht = order_key(tau0) >> 12;
        if (!(hk > ht || (hk == ht && key_exact<T>(hk)))) return false;
      }
      // y of ranks lane and lane + 32: exact from the key, or from the logit for a cut penalised value
      auto exact_y = [&](uint32_t kk, int r) {
        const uint32_t h = kk >> 12;
        float x = key20_value(h);
        if (SEEN && r <= k && kk != 0u && !key_exact<T>(h))
          x = penalised(to_f32(lrow[4095u - (kk & 4095u)]), true, p.pen);
        return greedy ? x : __fdiv_rn(x, p.temp);
      };
      const float y0 = exact_y(r0, lane), y1 = exact_y(r1, lane + 32);
      // neighbouring ranks r, r + 1 (r < k) whose keys are within two steps and not both exact may order
      // differently by (y desc, token asc), e.g. when the division by T rounds them to one value: the
      // exact values decide, and a wrong key order sends the row to the general path
      {
        const uint32_t d0 = __shfl_down_sync(kFull, r0, 1), b0 = __shfl_sync(kFull, r1, 0);
        const uint32_t d1 = __shfl_down_sync(kFull, r1, 1);
        const float e0 = __shfl_down_sync(kFull, y0, 1), f0 = __shfl_sync(kFull, y1, 0);
        const float e1 = __shfl_down_sync(kFull, y1, 1);
        auto wrong_pair = [&](uint32_t kx, float yx, uint32_t ky, float yy, bool have_y) {
          const uint32_t hx = kx >> 12, hy = ky >> 12;
          if (hx - hy > 2u || (key_exact<T>(hx) && key_exact<T>(hy))) return false;
          if (!have_y) return true;  // rank 64's exact value is not at hand
          const uint32_t tx = 4095u - (kx & 4095u), ty = 4095u - (ky & 4095u);
          return !(yx > yy || (yx == yy && tx < ty));
        };
        const bool wrong = (lane < k && wrong_pair(r0, y0, lane < 31 ? d0 : b0, lane < 31 ? e0 : f0, true)) ||
                           (lane + 32 < k && wrong_pair(r1, y1, lane < 31 ? d1 : key64, e1, lane < 31));
        if (__any_sync(kFull, wrong)) return false;
      }
      const int token = draw_top64(a, p, row, cand_word(order_key(y0), 4095 - static_cast<int>(r0 & 4095u)),
                                   cand_word(order_key(y1), 4095 - static_cast<int>(r1 & 4095u)), n0, n1);
      if (a.probs != nullptr) {
        const int64_t pbase = static_cast<int64_t>(row) * V;
        for (int r = k + lane; r < V; r += 32) {
          a.probs[pbase + r] = 0.f;
          a.ids[pbase + r] = -1;
        }
      }
      if (lane == 0) finish_row(a, row, token);
      return true;
    }
  }

  // ---- exact penalty on the candidates (slot s of lane l is candidate l + 32 s)
  constexpr int kSlots = kCandCap / 32;
  const int n_slots = (n_cand + 31) >> 5;  // warp-uniform: later slots are empty everywhere
  float cx[kSlots];
  int cid[kSlots];
#pragma unroll
  for (int s = 0; s < kSlots; ++s) {
    cx[s] = -__builtin_huge_valf();
    cid[s] = 0;
    if (s < n_slots) {
      const int i = lane + 32 * s;
      if (i < n_cand) {
        cx[s] = fs.cx[i];
        cid[s] = fs.cid[i];
      }
    }
  }
  if constexpr (SEEN) {
    uint8_t sb[kSlots];
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      sb[s] = 0;
      if (s < n_slots && lane + 32 * s < n_cand) sb[s] = a.seen[row * a.seen_stride + cid[s]];
    }
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      if (s < n_slots && __any_sync(kFull, sb[s] != 0)) cx[s] = penalised(cx[s], sb[s] != 0, p.pen);
    }
  }

  // ---- cut 2 (more than 64 candidates): tau1 = k-th largest of the 64 lane-local top-2 values
  float tau1 = -__builtin_huge_valf();
  if (n_cand > kFastK) {
    // the k-th largest of the 64 lane-local top-2 values (64 distinct candidates) is a valid floor
    float t1 = -__builtin_huge_valf(), t2 = -__builtin_huge_valf();
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      if (s < n_slots) {
        const float x = cx[s];  // absent slots hold -inf
        t2 = fmaxf(t2, fminf(t1, x));
        t1 = fmaxf(t1, x);
      }
    }
    warp_sort64_desc_f32(t1, t2);
    tau1 = rank_value(t1, t2, k - 1);
  }
  // F = {x_pen >= tau1}; x_out = the largest penalised candidate left out
  int n_f = 0;
  float x_out = -__builtin_huge_valf();
#pragma unroll
  for (int s = 0; s < kSlots; ++s) {
    if (s < n_slots) {
      const bool ok = lane + 32 * s < n_cand;
      const bool in = ok && cx[s] >= tau1;
      if (ok && !in) x_out = fmaxf(x_out, cx[s]);
      const unsigned bal = __ballot_sync(kFull, in);
      const int pos = n_f + __popc(bal & ((1u << lane) - 1u));
      if (in && pos < 2 * kFastK) {
        fs.fx[pos] = cx[s];
        fs.fid[pos] = cid[s];
      }
      n_f += __popc(bal);
    }
  }
  if (n_f > 2 * kFastK || n_f < k) return false;
  x_out = warp_max(x_out);
  __syncwarp();

  // ---- rank F by (y desc, token id asc); a second block of 64 is sorted and merged in
  auto yval = [&](float x) { return greedy ? x : scaled<T>(a, p, x); };
  auto word = [&](int i) { return i < n_f ? cand_word(order_key(yval(fs.fx[i])), fs.fid[i]) : 0ull; };
  uint64_t w0 = word(lane), w1 = word(lane + 32);
  warp_sort64_desc(w0, w1);
  if (n_f > kFastK) {
    uint64_t b0 = word(lane + 64), b1 = word(lane + 96);
    warp_sort64_desc(b0, b1);
    warp_merge64_desc(w0, w1, b0, b1);
  }
  // check: everything outside F stays strictly below the k-th value
  const uint64_t kth = __shfl_sync(kFull, (k - 1) < 32 ? w0 : w1, (k - 1) & 31);
  const float x_bound = fmaxf(x_out, L::prev(tau0));
  if (order_key(yval(x_bound)) >= static_cast<uint32_t>(kth >> 32)) return false;

  // ---- softmax, top-p and the draw over the k ranks
  const int token = draw_top64(a, p, row, w0, w1, n0, n1);
  if (a.probs != nullptr) {
    const int64_t pbase = static_cast<int64_t>(row) * V;
    for (int r = k + lane; r < V; r += 32) {
      a.probs[pbase + r] = 0.f;
      a.ids[pbase + r] = -1;
    }
  }
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
  const int64_t pbase = static_cast<int64_t>(row) * V;

  if (!(p.temp > 0.f)) {
    // greedy: first argmax of the penalised logits (model/sampling.py:183-187)
    float bv = -__builtin_huge_valf();
    int bi = 0x7fffffff;
    for (int e = tid; e < V; e += kThreads)
      argmax_merge(bv, bi, penalised(to_f32(lrow[e]), srow != nullptr && srow[e] != 0, p.pen), e);
    const int best = block_argmax(bv, bi, sh.redf, sh.redi);
    const int token = best < V ? best : 0;
    if (a.probs != nullptr) {
      for (int r = tid; r < V; r += kThreads) {
        a.probs[pbase + r] = r == 0 ? 1.f : 0.f;
        a.ids[pbase + r] = r == 0 ? token : -1;
      }
    }
    if (tid == 0) finish_row(a, row, token);
    __syncthreads();
    return;
  }

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

// Dynamic shared memory: one region that holds the groups' fast-path buffers during the fast phase and,
// afterwards, the general path's [np2] candidates followed by the keys of its row.
__host__ __device__ constexpr size_t region_bytes(int np2, int vocab, size_t group_bytes) {
  return static_cast<size_t>(np2) * 8 + static_cast<size_t>(vocab) * 4 > group_bytes
             ? static_cast<size_t>(np2) * 8 + static_cast<size_t>(vocab) * 4
             : group_bytes;
}

// kWarps / G rows per CTA, G warps per row.
template <typename T, int G>
__global__ void __launch_bounds__(kThreads, 4) sample_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ BlockShared bs;
  __shared__ int s_rest[kWarps];
  __shared__ int s_nrest;
  constexpr int kRows = kWarps / G;
  uint8_t* region = smem;
  uint64_t* s_cand = reinterpret_cast<uint64_t*>(smem);
  uint32_t* s_key = reinterpret_cast<uint32_t*>(smem + static_cast<size_t>(a.np2) * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = warp / G, wg = warp % G;
  if (threadIdx.x == 0) s_nrest = 0;
  __syncthreads();
  const int row = blockIdx.x * kRows + group;
  if (row < a.rows) {
    const RowParams p = row_params(a, row);
    FastShared<G>& fs = reinterpret_cast<FastShared<G>*>(region)[group];
    const bool done = a.seen != nullptr ? fast_row<T, G, true>(a, p, row, group, wg, fs)
                                        : fast_row<T, G, false>(a, p, row, group, wg, fs);
    if (!done && wg == 0 && lane == 0) s_rest[atomicAdd(&s_nrest, 1)] = row;
  }
  __syncthreads();
  const int nrest = s_nrest;
  for (int i = 0; i < nrest; ++i) block_row<T>(a, s_rest[i], bs, s_cand, s_key);
}

template <typename T, int G>
int launch_g(SampleArgs a, cudaStream_t s) {
  const size_t smem = region_bytes(a.np2, a.vocab, sizeof(FastShared<G>) * (kWarps / G));
  // the static shared memory counts against the default 48 KB as well; raised once per instantiation
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(sample_kernel<T, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  constexpr int kRows = kWarps / G;
  sample_kernel<T, G><<<(a.rows + kRows - 1) / kRows, kThreads, smem, s>>>(a);
  return check_launch("sample_rows");
}

// Warps per row: enough that rows x G reaches eight warps per SM, at most 8, and enough that the
// row fits the group's registers (larger rows take the general path).
template <typename T>
int launch(SampleArgs a, cudaStream_t s) {
  const int want = (8 * num_sms() + a.rows - 1) / a.rows;
  const int nvec = a.vocab / Lanes<T>::kVec;
  int g = want >= 5 ? 8 : (want >= 3 ? 4 : (want >= 2 ? 2 : 1));
  while (g < 8 && nvec > g * 32 * (g == 1 ? Vpl<1>::value : (g == 2 ? Vpl<2>::value : Vpl<4>::value))) g *= 2;
  switch (g) {
    case 1: return launch_g<T, 1>(a, s);
    case 2: return launch_g<T, 2>(a, s);
    case 4: return launch_g<T, 4>(a, s);
    default: return launch_g<T, 8>(a, s);
  }
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
