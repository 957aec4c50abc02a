// Fused logits sampler: repetition penalty, temperature, top-k, top-p and a
// seeded draw in one launch, one CTA per row.
//
// Per row:
//   1. x = logits (fp32); where seen: x > 0 ? x / penalty : x * penalty.
//   2. temperature == 0: first argmax of x (greedy) -> done.
//   3. y = x / T (optionally rounded to the logits type, as torch does for a
//      half-precision row without a seen mask); keys = order-preserving u32.
//   4. k_eff = k <= 0 ? V : min(k, V).  A 4-pass radix select (8 bits per
//      pass, shared-memory histograms) finds the k_eff-th largest key tau.
//   5. Every element with key >= tau is compacted and bitonic-sorted by
//      (value desc, token id asc); the first k_eff are the top-k, ties going
//      to the lowest token id.
//   6. p = softmax over the top-k values; if top_p < 1, rank r is dropped
//      when (cumsum_r - p_r) > top_p with the cumulative sum accumulated in
//      double and rounded per element (what torch's CPU cumsum does), and
//      the kept mass is renormalised.
//   7. Draw: argmax_r p_r / E_r (exponential race; first max wins), where
//      E_r = -log(U_r) and U_r comes from Philox4x32-10 keyed by the row's
//      seed with counter (rank, 0, offset) - or E_r is read from a caller
//      buffer (the parity entry).  torch.multinomial(p, 1) computes exactly
//      argmax(p / Exp(1)) on the CPU, so the same noise gives the same id.
//   8. Optionally mark the sampled token in the seen mask.
//
// Reference semantics: sample_logits_stateless / _cpu_sample_row
// (model/sampling.py:55-95, 127-225).
#include "common.cuh"

namespace nqt {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxVocab = 16384;
constexpr int kFastK = 64;      // largest top-k the one-warp ranking path takes
constexpr int kBins = 256;      // bins of the small-k histogram (== kThreads)
constexpr float kGapBins = 48.f;  // bin width = (row max - row mean) / kGapBins

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

__device__ __forceinline__ int block_argmax(float v, int i, float* sv, int* si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(kFull, v, o);
    const int i2 = __shfl_xor_sync(kFull, i, o);
    argmax_merge(v, i, v2, i2);
  }
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

template <typename T>
__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int V = a.vocab;
  uint64_t* s_cand = reinterpret_cast<uint64_t*>(smem);                                // [np2]
  uint32_t* s_key = reinterpret_cast<uint32_t*>(smem + static_cast<size_t>(a.np2) * 8);  // [V]
  __shared__ int s_hist[256];
  __shared__ int s_whist[kWarps][kBins];  // per-warp histograms of the small-k path
  __shared__ float s_redf[kWarps];
  __shared__ int s_redi[kWarps];
  __shared__ double s_redd[kWarps];
  __shared__ float s_stat_max[kWarps], s_stat_sum[kWarps];
  __shared__ int s_stat_n[kWarps], s_stat_bad[kWarps];
  __shared__ int s_digit, s_remaining, s_count, s_sel, s_above, s_total;

  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const T* lrow = static_cast<const T*>(a.logits) + row * a.lstride;
  const uint8_t* srow = a.seen != nullptr ? a.seen + row * a.seen_stride : nullptr;
  const float pen = a.penalty != nullptr ? a.penalty[row] : 1.f;
  const float temp = a.temp[row];
  const bool greedy = !(temp > 0.f);

  for (int i = tid; i < kWarps * kBins; i += kThreads) (&s_whist[0][0])[i] = 0;

  // 1-3. penalty, greedy argmax or scaled keys; the scaled row's max, sum and finite count
  float best_v = -__int_as_float(0x7f800000);
  int best_i = V;
  float ymax = -__int_as_float(0x7f800000), ysum = 0.f;
  int nfin = 0, bad = 0;
  auto consume = [&](int i, float x) {
    if (srow != nullptr && srow[i] != 0) x = x > 0.f ? __fdiv_rn(x, pen) : __fmul_rn(x, pen);
    if (greedy) {
      argmax_merge(best_v, best_i, x, i);
    } else {
      float y = __fdiv_rn(x, temp);
      if (a.round_scaled) y = to_f32(from_f32<T>(y));
      s_key[i] = order_key(y);
      ymax = fmaxf(ymax, y);
      if (!(y <= 3.402823466e38f)) {
        bad = 1;  // NaN or +inf: the radix path ranks it
      } else if (y >= -3.402823466e38f) {  // -inf is neither counted nor summed
        ysum += y;
        ++nfin;
      }
    }
  };
  constexpr int kVec = 16 / static_cast<int>(sizeof(T));
  if ((reinterpret_cast<uintptr_t>(lrow) & 15u) == 0 && V % kVec == 0) {
    const uint4* vrow = reinterpret_cast<const uint4*>(lrow);
    for (int vi = tid; vi < V / kVec; vi += kThreads) {
      const uint4 raw = vrow[vi];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < kVec; ++u) consume(vi * kVec + u, to_f32(e[u]));
    }
  } else {
    for (int i = tid; i < V; i += kThreads) consume(i, to_f32(lrow[i]));
  }
  int token;
  int k_eff = 0;
  if (greedy) {
    token = block_argmax(best_v, best_i, s_redf, s_redi);
    if (token >= V) token = 0;
    if (a.probs != nullptr) {
      for (int r = tid; r < V; r += kThreads) {
        a.probs[static_cast<int64_t>(row) * V + r] = r == 0 ? 1.f : 0.f;
        a.ids[static_cast<int64_t>(row) * V + r] = r == 0 ? token : -1;
      }
    }
  } else {
    const int kreq = a.top_k[row];
    k_eff = (kreq <= 0 || kreq >= V) ? V : kreq;

    // ---- small-k path: bins of the distance below the row max, width (max - mean) / kGapBins.
    // The bin index is a monotone function of the value, so the bins up to the one holding the
    // k-th value contain every member of the top-k; that bin is split once more into 256 sub-bins
    // when it alone holds too many.  At most kFastK candidates go to one warp for the exact
    // (value desc, id asc) ranking; rows that do not narrow down take the radix path below.
    bool fast = false;
    int b1 = -1, s2 = kBins;
    float m = 0.f, inv_w = 0.f;
    if (k_eff <= kFastK) {
      float wmax = ymax, wsum = ysum;
      int wn = nfin, wbad = bad;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        wmax = fmaxf(wmax, __shfl_xor_sync(kFull, wmax, o));
        wsum += __shfl_xor_sync(kFull, wsum, o);
        wn += __shfl_xor_sync(kFull, wn, o);
        wbad |= __shfl_xor_sync(kFull, wbad, o);
      }
      if (lane == 0) {
        s_stat_max[warp] = wmax;
        s_stat_sum[warp] = wsum;
        s_stat_n[warp] = wn;
        s_stat_bad[warp] = wbad;
      }
      if (tid == 0) {
        s_sel = -1;
        s_count = 0;
      }
      __syncthreads();
      m = s_stat_max[0];
      float sum = s_stat_sum[0];
      int n = s_stat_n[0], any_bad = s_stat_bad[0];
      for (int w = 1; w < kWarps; ++w) {
        m = fmaxf(m, s_stat_max[w]);
        sum += s_stat_sum[w];
        n += s_stat_n[w];
        any_bad |= s_stat_bad[w];
      }
      const float gap = n > 0 ? m - sum / static_cast<float>(n) : 0.f;
      if (!any_bad && n >= k_eff && gap > 1e-30f && gap <= 3.402823466e38f && m <= 3.402823466e38f) {
        inv_w = kGapBins / gap;
        for (int i = tid; i < V; i += kThreads) {
          const float t = (m - key_value(s_key[i])) * inv_w;
          if (t < 255.f) atomicAdd(&s_whist[warp][static_cast<int>(t)], 1);
        }
        __syncthreads();
        int c = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) c += s_whist[w][tid];
        const int incl = block_incl_scan(c, s_redi);
        if (incl >= k_eff && incl - c < k_eff) {
          s_sel = tid;
          s_above = incl - c;
          s_total = incl;
        }
        __syncthreads();
        b1 = s_sel;
        if (b1 >= 0) {
          if (s_total <= kFastK) {
            fast = true;
          } else {
            const int above = s_above;
            for (int w = 0; w < kWarps; ++w) s_whist[w][tid] = 0;
            if (tid == 0) s_sel = -1;
            __syncthreads();
            for (int i = tid; i < V; i += kThreads) {
              const float t = (m - key_value(s_key[i])) * inv_w;
              if (t < 255.f && static_cast<int>(t) == b1) {
                const int sub = min(static_cast<int>((t - static_cast<float>(b1)) * 256.f), kBins - 1);
                atomicAdd(&s_whist[warp][sub], 1);
              }
            }
            __syncthreads();
            int c2 = 0;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) c2 += s_whist[w][tid];
            const int incl2 = block_incl_scan(c2, s_redi) + above;
            if (incl2 >= k_eff && incl2 - c2 < k_eff) {
              s_sel = tid;
              s_total = incl2;
            }
            __syncthreads();
            s2 = s_sel;
            fast = s2 >= 0 && s_total <= kFastK;
          }
        }
      }
    }

    if (fast) {
      // compact the candidates (every key in bins < b1, and in bin b1 up to sub-bin s2)
      for (int i = tid; i < V; i += kThreads) {
        const uint32_t k = s_key[i];
        const float t = (m - key_value(k)) * inv_w;
        bool take = false;
        if (t < 255.f) {
          const int b = static_cast<int>(t);
          take = b < b1 ||
                 (b == b1 && (s2 >= kBins ||
                              min(static_cast<int>((t - static_cast<float>(b1)) * 256.f), kBins - 1) <= s2));
        }
        if (take) {
          const int pos = atomicAdd(&s_count, 1);
          s_cand[pos] = (static_cast<uint64_t>(k) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(i));
        }
      }
      __syncthreads();
      const int n_cand = s_count;
      if (a.probs != nullptr) {
        for (int r = k_eff + tid; r < V; r += kThreads) {
          a.probs[static_cast<int64_t>(row) * V + r] = 0.f;
          a.ids[static_cast<int64_t>(row) * V + r] = -1;
        }
      }
      if (warp == 0) {
        uint64_t c0 = lane < n_cand ? s_cand[lane] : 0ull;
        uint64_t c1 = lane + 32 < n_cand ? s_cand[lane + 32] : 0ull;
        warp_sort64_desc(c0, c1);
        const bool in0 = lane < k_eff, in1 = lane + 32 < k_eff;
        const float vtop = __shfl_sync(kFull, key_value(static_cast<uint32_t>(c0 >> 32)), 0);
        const float e0 = in0 ? expf(key_value(static_cast<uint32_t>(c0 >> 32)) - vtop) : 0.f;
        const float e1 = in1 ? expf(key_value(static_cast<uint32_t>(c1 >> 32)) - vtop) : 0.f;
        const float esum = warp_sum(e0) + warp_sum(e1);
        float p0 = in0 ? __fdiv_rn(e0, esum) : 0.f;
        float p1 = in1 ? __fdiv_rn(e1, esum) : 0.f;
        const float top_p = a.top_p[row];
        if (top_p < 1.f) {
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
          if (in0 && __fsub_rn(static_cast<float>(run0), p0) > top_p) p0 = 0.f;
          if (in1 && __fsub_rn(static_cast<float>(run1), p1) > top_p) p1 = 0.f;
          const float norm = fmaxf(warp_sum(p0) + warp_sum(p1), 1.17549435e-38f);
          p0 = __fdiv_rn(p0, norm);
          p1 = __fdiv_rn(p1, norm);
        }
        // 7. exponential race over ranks
        const int64_t seed = a.noise == nullptr ? a.seed[row] : 0;
        const int64_t off = a.noise == nullptr ? a.offset[row * a.offset_stride] : 0;
        float bv = -1.f;
        int br = k_eff;
        if (in0) {
          const float e = a.noise != nullptr ? a.noise[row * a.noise_stride + lane] : exp_noise(seed, off, lane);
          argmax_merge(bv, br, __fdiv_rn(p0, e), lane);
        }
        if (in1) {
          const int r = lane + 32;
          const float e = a.noise != nullptr ? a.noise[row * a.noise_stride + r] : exp_noise(seed, off, r);
          argmax_merge(bv, br, __fdiv_rn(p1, e), r);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float v2 = __shfl_xor_sync(kFull, bv, o);
          const int i2 = __shfl_xor_sync(kFull, br, o);
          argmax_merge(bv, br, v2, i2);
        }
        if (a.probs != nullptr) {
          if (in0) {
            a.probs[static_cast<int64_t>(row) * V + lane] = p0;
            a.ids[static_cast<int64_t>(row) * V + lane] = static_cast<int32_t>(~static_cast<uint32_t>(c0));
          }
          if (in1) {
            a.probs[static_cast<int64_t>(row) * V + lane + 32] = p1;
            a.ids[static_cast<int64_t>(row) * V + lane + 32] = static_cast<int32_t>(~static_cast<uint32_t>(c1));
          }
        }
        const int rank = br < k_eff ? br : 0;
        const uint64_t w0 = __shfl_sync(kFull, c0, rank & 31);
        const uint64_t w1 = __shfl_sync(kFull, c1, rank & 31);
        token = static_cast<int>(~static_cast<uint32_t>(rank < 32 ? w0 : w1));
        if (lane == 0) {
          a.tokens[row] = token;
          if (a.update_seen && a.seen != nullptr) a.seen[row * a.seen_stride + token] = 1;
        }
      }
      return;
    }
    __syncthreads();

    // 4. radix select of the k_eff-th largest key
    uint32_t tau = 0u;
    int n_cand = V;
    if (k_eff < V) {
      uint32_t prefix = 0u, mask = 0u;
      int remaining = k_eff;
      int eq_count = 0;
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        s_hist[tid] = 0;  // kThreads == 256 bins
        __syncthreads();
        for (int i = tid; i < V; i += kThreads) {
          const uint32_t k = s_key[i];
          if ((k & mask) == prefix) atomicAdd(&s_hist[(k >> shift) & 255u], 1);
        }
        __syncthreads();
        // suffix count at bin tid: elements with digit >= tid (block scan from the top)
        const int h = s_hist[tid];
        int suffix = h;
        {
          // inclusive scan over reversed bins
          const int lane = tid & 31, warp = tid >> 5;
          const int rev = s_hist[255 - tid];
          int incl = rev;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += y;
          }
          if (lane == 31) s_redi[warp] = incl;
          __syncthreads();
          int base = 0;
          for (int w = 0; w < warp; ++w) base += s_redi[w];
          incl += base;
          // incl = #elements with digit >= 255 - tid; publish back in bin order
          __syncthreads();
          s_hist[255 - tid] = incl;  // overwrite: now suffix counts
          __syncthreads();
          suffix = s_hist[tid];
          __syncthreads();
        }
        const int above = suffix - h;  // elements with digit > tid
        if (above < remaining && remaining <= suffix) {
          s_digit = tid;
          s_remaining = remaining - above;
          s_count = h;
        }
        __syncthreads();
        const int digit = s_digit;
        remaining = s_remaining;
        eq_count = s_count;
        prefix |= static_cast<uint32_t>(digit) << shift;
        mask |= 255u << shift;
        __syncthreads();
      }
      tau = prefix;
      n_cand = (k_eff - remaining) + eq_count;  // every key >= tau
    }

    // 5. compact keys >= tau, then sort (value desc, id asc)
    if (tid == 0) s_count = 0;
    __syncthreads();
    int n_pow2 = 1;
    while (n_pow2 < n_cand) n_pow2 <<= 1;
    for (int i = tid; i < V; i += kThreads) {
      const uint32_t k = s_key[i];
      if (k >= tau) {
        const int pos = atomicAdd(&s_count, 1);
        s_cand[pos] = (static_cast<uint64_t>(k) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(i));
      }
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

    // 6. softmax over the top-k values (rank order), then top-p
    const float v0 = key_value(static_cast<uint32_t>(s_cand[0] >> 32));
    // Each thread owns a contiguous run of ranks so the cumulative sum is in rank order.
    const int per = (k_eff + kThreads - 1) / kThreads;
    const int r0 = tid * per;
    const int r1 = min(k_eff, r0 + per);
    float e_local = 0.f;
    for (int r = r0; r < r1; ++r) e_local += expf(key_value(static_cast<uint32_t>(s_cand[r] >> 32)) - v0);
    const float esum = block_reduce_sum<float>(e_local, s_redf);
    const float top_p = a.top_p[row];
    float kept_local = 0.f;
    if (top_p < 1.f) {
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
      if (lane == 31) s_redd[warp] = incl;
      __syncthreads();
      double run = incl - part;
      for (int w = 0; w < warp; ++w) run += s_redd[w];
      for (int r = r0; r < r1; ++r) {
        const float pr = __fdiv_rn(expf(key_value(static_cast<uint32_t>(s_cand[r] >> 32)) - v0), esum);
        run += static_cast<double>(pr);
        const float cum = static_cast<float>(run);
        const bool drop = __fsub_rn(cum, pr) > top_p;
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
    if (top_p < 1.f) {
      const float kept = block_reduce_sum<float>(kept_local, s_redf);
      norm = fmaxf(kept, 1.17549435e-38f);
    }
    __syncthreads();

    // 7. exponential race over ranks
    const int64_t seed = a.noise == nullptr ? a.seed[row] : 0;
    const int64_t off = a.noise == nullptr ? a.offset[row * a.offset_stride] : 0;
    float bv = -1.f;
    int br = k_eff;
    for (int r = r0; r < r1; ++r) {
      float pr = __uint_as_float(static_cast<uint32_t>(s_cand[r] >> 32));
      if (top_p < 1.f) pr = __fdiv_rn(pr, norm);
      const float e = a.noise != nullptr ? a.noise[row * a.noise_stride + r] : exp_noise(seed, off, r);
      argmax_merge(bv, br, __fdiv_rn(pr, e), r);
      if (a.probs != nullptr) {
        a.probs[static_cast<int64_t>(row) * V + r] = pr;
        a.ids[static_cast<int64_t>(row) * V + r] = static_cast<int32_t>(~static_cast<uint32_t>(s_cand[r]));
      }
    }
    if (a.probs != nullptr) {
      for (int r = k_eff + tid; r < V; r += kThreads) {
        a.probs[static_cast<int64_t>(row) * V + r] = 0.f;
        a.ids[static_cast<int64_t>(row) * V + r] = -1;
      }
    }
    const int rank = block_argmax(bv, br, s_redf, s_redi);
    token = static_cast<int>(~static_cast<uint32_t>(s_cand[rank < k_eff ? rank : 0]));
  }
  if (tid == 0) {
    a.tokens[row] = token;
    if (a.update_seen && a.seen != nullptr) a.seen[row * a.seen_stride + token] = 1;
  }
}

template <typename T>
int launch(SampleArgs a, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(a.np2) * 8 + static_cast<size_t>(a.vocab) * 4;
  // static shared memory (histograms, reductions) counts against the default 48 KB too
  if (smem > 32 * 1024) {
    static int configured = 0;
    if (!configured) {
      cudaFuncSetAttribute(sample_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      configured = 1;
    }
  }
  sample_kernel<T><<<a.rows, kThreads, smem, s>>>(a);
  return check_launch("sample_rows");
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
