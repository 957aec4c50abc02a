// Paired QK RMSNorm + RoPE with the K/V cache write (paged and dense).
//
// One warp per (token, head); q heads and k heads share the launch.  A lane
// owns the RoPE pairs (i, i + D/2) for i = lane + 32j, so the rotation needs
// no shuffles and the only cross-lane step is the sum of squares.
//
// Reference semantics: model/kernels.py:15-91 (paged, rounds the normalised
// value to the element type before RoPE) and :163-248 (dense; rounding only
// when round_to_input, i.e. paired_qk_norm_rope_; the dense-cache variant
// does not round).
#include "common.cuh"

namespace nqt {
namespace {

struct QkArgs {
  void* q;
  int64_t q_st, q_sh;
  void* k;
  int64_t k_st, k_sh;
  const void* v;
  int64_t v_st, v_sh;
  const void* qw;
  const void* kw;
  const int64_t* pos;
  int64_t pos_stride;
  int tokens, hq, hkv;
  float eps, theta;
  int32_t* status;
  float inv_freq[128];  // RoPE theta^(-2i/D), i < D / 2, evaluated on the host
};

// Normalise + rotate one head vector in place.  Returns nothing; the rotated
// values are left in first[]/second[] (fp32, before the final rounding).
template <typename T, int D>
__device__ __forceinline__ void norm_rope_head(T* base, const T* weight, float pos, float eps, const float* inv_freq,
                                               bool round_norm, float (&first)[D / 64], float (&second)[D / 64]) {
  constexpr int J = D / 64;
  constexpr int H = D / 2;
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int i = lane + 32 * j;
    first[j] = to_f32(base[i]);
    second[j] = to_f32(base[i + H]);
    ss += first[j] * first[j] + second[j] * second[j];
  }
  ss = warp_sum(ss);
  const float inv_rms = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int i = lane + 32 * j;
    float a = first[j] * inv_rms * to_f32(weight[i]);
    float b = second[j] * inv_rms * to_f32(weight[i + H]);
    if (round_norm) {
      a = to_f32(from_f32<T>(a));
      b = to_f32(from_f32<T>(b));
    }
    const float angle = pos * inv_freq[i];
    float s, c;
    sincosf(angle, &s, &c);
    first[j] = a * c - b * s;
    second[j] = b * c + a * s;
    base[i] = from_f32<T>(first[j]);
    base[i + H] = from_f32<T>(second[j]);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(256) qk_norm_rope_paged_kernel(const __grid_constant__ QkArgs a, T* cache, int total_pages,
                                                                 int page_size, const int64_t* write_pages,
                                                                 const int64_t* write_offsets) {
  // a decode launch queued behind this one with NQT_DECODE_OVERLAP_KV_WRITE may start its page-id
  // staging and older-tile loads now; it waits for this grid before touching q or a row's last tile
  grid_dependents_launch();
  const int token = blockIdx.x;
  const int ph = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (ph >= a.hq + a.hkv) return;
  const int lane = threadIdx.x & 31;
  const bool is_q = ph < a.hq;
  const int head = is_q ? ph : ph - a.hq;
  T* base = is_q ? static_cast<T*>(a.q) + token * a.q_st + head * a.q_sh
                 : static_cast<T*>(a.k) + token * a.k_st + head * a.k_sh;
  const T* w = static_cast<const T*>(is_q ? a.qw : a.kw);
  const float pos = static_cast<float>(a.pos[token * a.pos_stride]);
  float first[D / 64], second[D / 64];
  norm_rope_head<T, D>(base, w, pos, a.eps, a.inv_freq, true, first, second);
  if (is_q) return;
  const int64_t page = write_pages[token];
  const int64_t off = write_offsets[token];
  if (page < 0 || page >= total_pages || off < 0 || off >= page_size) {
    if (lane == 0) report(a.status, NQT_DEV_BAD_PAGE);
    return;
  }
  constexpr int H = D / 2;
  // [page, kind, token, head, d]
  const int64_t row = static_cast<int64_t>(a.hkv) * D;
  T* kdst = cache + (page * 2 * page_size + off) * row + head * D;
  T* vdst = kdst + page_size * row;
  const T* vsrc = static_cast<const T*>(a.v) + token * a.v_st + head * a.v_sh;
#pragma unroll
  for (int j = 0; j < D / 64; ++j) {
    const int i = lane + 32 * j;
    kdst[i] = from_f32<T>(first[j]);
    kdst[i + H] = from_f32<T>(second[j]);
    vdst[i] = vsrc[i];
    vdst[i + H] = vsrc[i + H];
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(256) qk_norm_rope_dense_kernel(const __grid_constant__ QkArgs a, T* k_cache, T* v_cache,
                                                                 int64_t c_row, int64_t c_pos, int64_t c_head,
                                                                 int cache_position, int round_norm) {
  const int token = blockIdx.x;
  const int ph = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (ph >= a.hq + a.hkv) return;
  const int lane = threadIdx.x & 31;
  const bool is_q = ph < a.hq;
  const int head = is_q ? ph : ph - a.hq;
  T* base = is_q ? static_cast<T*>(a.q) + token * a.q_st + head * a.q_sh
                 : static_cast<T*>(a.k) + token * a.k_st + head * a.k_sh;
  const T* w = static_cast<const T*>(is_q ? a.qw : a.kw);
  const float pos = static_cast<float>(a.pos[token * a.pos_stride]);
  float first[D / 64], second[D / 64];
  norm_rope_head<T, D>(base, w, pos, a.eps, a.inv_freq, round_norm != 0, first, second);
  if (is_q || k_cache == nullptr) return;
  constexpr int H = D / 2;
  T* kdst = k_cache + token * c_row + static_cast<int64_t>(cache_position) * c_pos + head * c_head;
  T* vdst = v_cache + token * c_row + static_cast<int64_t>(cache_position) * c_pos + head * c_head;
  const T* vsrc = static_cast<const T*>(a.v) + token * a.v_st + head * a.v_sh;
#pragma unroll
  for (int j = 0; j < D / 64; ++j) {
    const int i = lane + 32 * j;
    kdst[i] = from_f32<T>(first[j]);
    kdst[i + H] = from_f32<T>(second[j]);
    vdst[i] = vsrc[i];
    vdst[i + H] = vsrc[i + H];
  }
}

bool supported_dim(int d) { return d == 64 || d == 128 || d == 256; }

template <typename T>
int launch_paged(const QkArgs& a, void* cache, int total_pages, int page_size, const int64_t* wp,
                 const int64_t* wo, int head_dim, cudaStream_t s) {
  dim3 grid(a.tokens, (a.hq + a.hkv + 7) / 8);
  switch (head_dim) {
    case 64:
      qk_norm_rope_paged_kernel<T, 64><<<grid, 256, 0, s>>>(a, static_cast<T*>(cache), total_pages, page_size, wp, wo);
      break;
    case 128:
      qk_norm_rope_paged_kernel<T, 128><<<grid, 256, 0, s>>>(a, static_cast<T*>(cache), total_pages, page_size, wp, wo);
      break;
    default:
      qk_norm_rope_paged_kernel<T, 256><<<grid, 256, 0, s>>>(a, static_cast<T*>(cache), total_pages, page_size, wp, wo);
  }
  return check_launch("qk_norm_rope_paged");
}

template <typename T>
int launch_dense(const QkArgs& a, void* kc, void* vc, int64_t cr, int64_t cp, int64_t ch, int cpos, int round,
                 int head_dim, cudaStream_t s) {
  dim3 grid(a.tokens, (a.hq + a.hkv + 7) / 8);
  T* k = static_cast<T*>(kc);
  T* v = static_cast<T*>(vc);
  switch (head_dim) {
    case 64:
      qk_norm_rope_dense_kernel<T, 64><<<grid, 256, 0, s>>>(a, k, v, cr, cp, ch, cpos, round);
      break;
    case 128:
      qk_norm_rope_dense_kernel<T, 128><<<grid, 256, 0, s>>>(a, k, v, cr, cp, ch, cpos, round);
      break;
    default:
      qk_norm_rope_dense_kernel<T, 256><<<grid, 256, 0, s>>>(a, k, v, cr, cp, ch, cpos, round);
  }
  return check_launch("qk_norm_rope_dense");
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_qk_norm_rope_paged_kv_write(
    void* q, int64_t q_stride_tok, int64_t q_stride_head, void* k, int64_t k_stride_tok, int64_t k_stride_head,
    const void* v, int64_t v_stride_tok, int64_t v_stride_head, const void* q_weight, const void* k_weight,
    const int64_t* position_ids, const int64_t* write_pages, const int64_t* write_offsets, void* layer_cache,
    int total_pages, int page_size, int tokens, int num_qo_heads, int num_kv_heads, int head_dim, float eps,
    float rope_theta, int dtype, int32_t* status, void* stream) {
  if (!q || !k || !v || !q_weight || !k_weight || !position_ids || !write_pages || !write_offsets || !layer_cache)
    return NQT_ERR_ARG;
  if (tokens < 0 || num_qo_heads < 1 || num_kv_heads < 1 || total_pages < 1 || page_size < 1) return NQT_ERR_ARG;
  if (!supported_dim(head_dim)) return NQT_ERR_UNSUPPORTED;
  if (tokens == 0) return NQT_OK;
  if ((num_qo_heads + num_kv_heads + 7) / 8 > 65535) return NQT_ERR_UNSUPPORTED;
  QkArgs a{q, q_stride_tok, q_stride_head, k, k_stride_tok, k_stride_head, v, v_stride_tok, v_stride_head,
           q_weight, k_weight, position_ids, 1, tokens, num_qo_heads, num_kv_heads, eps, rope_theta, status, {}};
  rope_inv_freq_table(a.inv_freq, head_dim, rope_theta);
  cudaStream_t s = as_stream(stream);
  if (dtype == NQT_BF16)
    return launch_paged<__nv_bfloat16>(a, layer_cache, total_pages, page_size, write_pages, write_offsets, head_dim, s);
  if (dtype == NQT_F16)
    return launch_paged<__half>(a, layer_cache, total_pages, page_size, write_pages, write_offsets, head_dim, s);
  return NQT_ERR_UNSUPPORTED;
}

extern "C" int nqt_qk_norm_rope_dense(
    void* q, int64_t q_stride_tok, int64_t q_stride_head, void* k, int64_t k_stride_tok, int64_t k_stride_head,
    const void* v, int64_t v_stride_tok, int64_t v_stride_head, const void* q_weight, const void* k_weight,
    const int64_t* positions, int64_t positions_stride, void* k_cache, void* v_cache, int64_t cache_stride_row,
    int64_t cache_stride_pos, int64_t cache_stride_head, int cache_position, int tokens, int num_qo_heads,
    int num_kv_heads, int head_dim, float eps, float rope_theta, int round_to_input, int dtype, int32_t* status,
    void* stream) {
  if (!q || !k || !q_weight || !k_weight || !positions) return NQT_ERR_ARG;
  if ((k_cache == nullptr) != (v_cache == nullptr)) return NQT_ERR_ARG;
  if (k_cache != nullptr && (v == nullptr || cache_position < 0)) return NQT_ERR_ARG;
  if (tokens < 0 || num_qo_heads < 1 || num_kv_heads < 1) return NQT_ERR_ARG;
  if (!supported_dim(head_dim)) return NQT_ERR_UNSUPPORTED;
  if (tokens == 0) return NQT_OK;
  QkArgs a{q, q_stride_tok, q_stride_head, k, k_stride_tok, k_stride_head, v, v_stride_tok, v_stride_head,
           q_weight, k_weight, positions, positions_stride, tokens, num_qo_heads, num_kv_heads, eps, rope_theta,
           status, {}};
  rope_inv_freq_table(a.inv_freq, head_dim, rope_theta);
  cudaStream_t s = as_stream(stream);
  if (dtype == NQT_BF16)
    return launch_dense<__nv_bfloat16>(a, k_cache, v_cache, cache_stride_row, cache_stride_pos, cache_stride_head,
                                       cache_position, round_to_input, head_dim, s);
  if (dtype == NQT_F16)
    return launch_dense<__half>(a, k_cache, v_cache, cache_stride_row, cache_stride_pos, cache_stride_head,
                                cache_position, round_to_input, head_dim, s);
  return NQT_ERR_UNSUPPORTED;
}
