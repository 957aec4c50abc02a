// Code-predictor attention: one query token per row over a short dense
// cache [rows, capacity, Hkv, D] (capacity <= 32, 16 in Qwen3-TTS).
//
// The fused decode step runs, in one CTA per row:
//   phase 1  one warp per query head and per KV head: fp32 RMSNorm over D,
//            times the norm weight, RoPE (no rounding before RoPE, like the
//            dense-cache kernel, model/kernels.py:335-405), stores q/k back in
//            place as bf16, K/V of the new token into the cache at
//            cache_position;
//   phase 2  one warp per query head: lane j scores cache position j,
//            warp-shuffle softmax (fp32, scale 1/sqrt(D)), then lanes split
//            the head dimension for P.V (model/kernels.py:408-463).
// The whole step stays inside the CTA, so the K/V write and the attention
// read need no cross-CTA ordering.
#include "common.cuh"

namespace nqt {
namespace {

struct CpArgs {
  __nv_bfloat16* q;
  int64_t q_st, q_sh;
  __nv_bfloat16* k;
  int64_t k_st, k_sh;
  const __nv_bfloat16* v;
  int64_t v_st, v_sh;
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  const int64_t* pos;
  int64_t pos_stride;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  int64_t c_row, c_pos, c_head;
  int capacity, cache_position, length;
  int rows, hq, hkv, group;
  float eps, theta, scale;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  int32_t* status;
};

template <int D>
__device__ __forceinline__ void norm_rope_store(__nv_bfloat16* base, const __nv_bfloat16* w, float pos, float eps,
                                                float theta, float (&f)[D / 64], float (&s)[D / 64]) {
  constexpr int J = D / 64, H = D / 2;
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    f[j] = __bfloat162float(base[lane + 32 * j]);
    s[j] = __bfloat162float(base[lane + 32 * j + H]);
    ss += f[j] * f[j] + s[j] * s[j];
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int i = lane + 32 * j;
    const float a = f[j] * inv * __bfloat162float(w[i]);
    const float b = s[j] * inv * __bfloat162float(w[i + H]);
    float sn, cs;
    sincosf(pos * rope_inv_freq(i, D, theta), &sn, &cs);
    f[j] = a * cs - b * sn;
    s[j] = b * cs + a * sn;
    base[i] = __float2bfloat16_rn(f[j]);
    base[i + H] = __float2bfloat16_rn(s[j]);
  }
}

// Phase 2 for one query head: attention of q (bf16 in global) over `len`
// cache positions.  Lane j (< len) scores position j.
template <int D>
__device__ __forceinline__ void short_attend(const CpArgs& a, int row, int head, const __nv_bfloat16* qrow,
                                             int len) {
  const int lane = threadIdx.x & 31;
  const int kvh = head / a.group;
  float score = -__int_as_float(0x7f800000);
  if (lane < len) {
    const __nv_bfloat16* krow = a.kc + row * a.c_row + lane * a.c_pos + kvh * a.c_head;
    float acc = 0.f;
#pragma unroll
    for (int d = 0; d < D; d += 8) {
      const uint4 kv = *reinterpret_cast<const uint4*>(krow + d);
      const uint4 qv = *reinterpret_cast<const uint4*>(qrow + d);
      const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv);
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 kf = __bfloat1622float2(k2[e]);
        const float2 qf = __bfloat1622float2(q2[e]);
        acc = fmaf(qf.x, kf.x, acc);
        acc = fmaf(qf.y, kf.y, acc);
      }
    }
    score = acc * a.scale;
  }
  const float mx = warp_max(score);
  const float p = lane < len ? __expf(score - mx) : 0.f;
  const float denom = warp_sum(p);
  // P.V: lane owns dims (2*lane, 2*lane+1) [+64 for D=128]
  constexpr int J = D / 64;
  float acc[J][2];
#pragma unroll
  for (int j = 0; j < J; ++j) acc[j][0] = acc[j][1] = 0.f;
  for (int pos = 0; pos < len; ++pos) {
    const float pp = __shfl_sync(kFull, p, pos);
    const __nv_bfloat16* vrow = a.vc + row * a.c_row + pos * a.c_pos + kvh * a.c_head;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float2 vf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vrow + 64 * j + 2 * lane));
      acc[j][0] = fmaf(pp, vf.x, acc[j][0]);
      acc[j][1] = fmaf(pp, vf.y, acc[j][1]);
    }
  }
  const float inv = 1.f / denom;
  __nv_bfloat16* orow = a.out + row * a.o_st + head * a.o_sh;
#pragma unroll
  for (int j = 0; j < J; ++j)
    *reinterpret_cast<__nv_bfloat162*>(orow + 64 * j + 2 * lane) =
        __floats2bfloat162_rn(acc[j][0] * inv, acc[j][1] * inv);
}

template <int D>
__global__ void __launch_bounds__(1024) cp_decode_kernel(CpArgs a) {
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const float pos = static_cast<float>(a.pos[row * a.pos_stride]);
  constexpr int H = D / 2;
  // phase 1: q heads are warps [0, hq), k heads are warps [hq, hq + hkv)
  if (warp < a.hq + a.hkv) {
    float f[D / 64], s[D / 64];
    if (warp < a.hq) {
      norm_rope_store<D>(a.q + row * a.q_st + warp * a.q_sh, a.qw, pos, a.eps, a.theta, f, s);
    } else {
      const int h = warp - a.hq;
      norm_rope_store<D>(a.k + row * a.k_st + h * a.k_sh, a.kw, pos, a.eps, a.theta, f, s);
      __nv_bfloat16* kd = a.kc + row * a.c_row + static_cast<int64_t>(a.cache_position) * a.c_pos + h * a.c_head;
      __nv_bfloat16* vd = a.vc + row * a.c_row + static_cast<int64_t>(a.cache_position) * a.c_pos + h * a.c_head;
      const __nv_bfloat16* vs = a.v + row * a.v_st + h * a.v_sh;
#pragma unroll
      for (int j = 0; j < D / 64; ++j) {
        const int i = lane + 32 * j;
        kd[i] = __float2bfloat16_rn(f[j]);
        kd[i + H] = __float2bfloat16_rn(s[j]);
        vd[i] = vs[i];
        vd[i + H] = vs[i + H];
      }
    }
  }
  __syncthreads();
  if (warp < a.hq) short_attend<D>(a, row, warp, a.q + row * a.q_st + warp * a.q_sh, a.length);
}

template <int D>
__global__ void __launch_bounds__(1024) cp_short_kernel(CpArgs a) {
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  if (warp < a.hq) short_attend<D>(a, row, warp, a.q + row * a.q_st + warp * a.q_sh, a.length);
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_cp_decode_attention(
    void* q, int64_t q_stride_tok, int64_t q_stride_head, void* k, int64_t k_stride_tok, int64_t k_stride_head,
    const void* v, int64_t v_stride_tok, int64_t v_stride_head, const void* q_weight, const void* k_weight,
    const int64_t* positions, int64_t positions_stride, void* k_cache, void* v_cache, int64_t cache_stride_row,
    int64_t cache_stride_pos, int64_t cache_stride_head, int cache_capacity, int cache_position, int rows,
    int num_qo_heads, int num_kv_heads, int head_dim, float eps, float rope_theta, float sm_scale, void* out,
    int64_t out_stride_tok, int64_t out_stride_head, int32_t* status, void* stream) {
  if (!q || !k || !v || !q_weight || !k_weight || !positions || !k_cache || !v_cache || !out) return NQT_ERR_ARG;
  if (rows < 1 || num_kv_heads < 1 || num_qo_heads % num_kv_heads) return NQT_ERR_ARG;
  if (cache_position < 0 || cache_position >= cache_capacity) return NQT_ERR_ARG;
  if (head_dim != 64 && head_dim != 128) return NQT_ERR_UNSUPPORTED;
  if (num_qo_heads + num_kv_heads > 32 || cache_capacity > 32) return NQT_ERR_UNSUPPORTED;
  // 16-byte row loads of q and K
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache)) & 15) return NQT_ERR_ARG;
  if ((q_stride_tok | q_stride_head | cache_stride_row | cache_stride_pos | cache_stride_head) & 7) return NQT_ERR_ARG;
  if (((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(v_cache)) & 3) ||
      ((out_stride_tok | out_stride_head) & 1))
    return NQT_ERR_ARG;
  CpArgs a{static_cast<__nv_bfloat16*>(q), q_stride_tok, q_stride_head, static_cast<__nv_bfloat16*>(k),
           k_stride_tok, k_stride_head, static_cast<const __nv_bfloat16*>(v), v_stride_tok, v_stride_head,
           static_cast<const __nv_bfloat16*>(q_weight), static_cast<const __nv_bfloat16*>(k_weight), positions,
           positions_stride, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
           cache_stride_row, cache_stride_pos, cache_stride_head, cache_capacity, cache_position,
           cache_position + 1, rows, num_qo_heads, num_kv_heads, num_qo_heads / num_kv_heads, eps, rope_theta,
           sm_scale, static_cast<__nv_bfloat16*>(out), out_stride_tok, out_stride_head, status};
  const int threads = 32 * (num_qo_heads + num_kv_heads);
  cudaStream_t s = as_stream(stream);
  if (head_dim == 64)
    cp_decode_kernel<64><<<rows, threads, 0, s>>>(a);
  else
    cp_decode_kernel<128><<<rows, threads, 0, s>>>(a);
  return check_launch("cp_decode_attention");
}

extern "C" int nqt_cp_short_attention(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                      const void* k_cache, const void* v_cache, int64_t cache_stride_row,
                                      int64_t cache_stride_pos, int64_t cache_stride_head, int cache_length,
                                      int rows, int num_qo_heads, int num_kv_heads, int head_dim, float sm_scale,
                                      void* out, int64_t out_stride_tok, int64_t out_stride_head, int32_t* status,
                                      void* stream) {
  if (!q || !k_cache || !v_cache || !out) return NQT_ERR_ARG;
  if (rows < 1 || num_kv_heads < 1 || num_qo_heads % num_kv_heads) return NQT_ERR_ARG;
  if (cache_length < 1 || cache_length > 32) return NQT_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return NQT_ERR_UNSUPPORTED;
  if (num_qo_heads > 32) return NQT_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache)) & 15) return NQT_ERR_ARG;
  if ((q_stride_tok | q_stride_head | cache_stride_row | cache_stride_pos | cache_stride_head) & 7) return NQT_ERR_ARG;
  if (((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(v_cache)) & 3) ||
      ((out_stride_tok | out_stride_head) & 1))
    return NQT_ERR_ARG;
  CpArgs a{};
  a.q = static_cast<__nv_bfloat16*>(const_cast<void*>(q));
  a.q_st = q_stride_tok;
  a.q_sh = q_stride_head;
  a.kc = static_cast<__nv_bfloat16*>(const_cast<void*>(k_cache));
  a.vc = static_cast<__nv_bfloat16*>(const_cast<void*>(v_cache));
  a.c_row = cache_stride_row;
  a.c_pos = cache_stride_pos;
  a.c_head = cache_stride_head;
  a.length = cache_length;
  a.rows = rows;
  a.hq = num_qo_heads;
  a.hkv = num_kv_heads;
  a.group = num_qo_heads / num_kv_heads;
  a.scale = sm_scale;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_st = out_stride_tok;
  a.o_sh = out_stride_head;
  a.status = status;
  cudaStream_t s = as_stream(stream);
  if (head_dim == 64)
    cp_short_kernel<64><<<rows, 32 * num_qo_heads, 0, s>>>(a);
  else
    cp_short_kernel<128><<<rows, 32 * num_qo_heads, 0, s>>>(a);
  return check_launch("cp_short_attention");
}
