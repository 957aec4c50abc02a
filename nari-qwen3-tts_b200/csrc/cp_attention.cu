// Code-predictor attention: one query token per row over a short dense
// cache [rows, capacity, Hkv, D] (capacity <= 32, 16 in Qwen3-TTS).
//
// The fused decode step (nqt_cp_decode_attention) runs one CTA per row and
// one warp per KV head (cp_decode_group_kernel below); the attention-only
// entry (nqt_cp_short_attention) one warp per query head.  The math:
//   phase 1  per query head and per KV head: fp32 RMSNorm over D,
//            times the norm weight, RoPE (no rounding before RoPE, like the
//            dense-cache kernel, model/kernels.py:335-405), stores q/k back in
//            place as bf16, K/V of the new token into the cache at
//            cache_position;
//   phase 2  per query head: lane j scores cache position j,
//            warp-shuffle softmax (fp32, scale 1/sqrt(D)), then lanes split
//            the head dimension for P.V, the V rows of 16 positions loaded
//            before the first is used (model/kernels.py:408-463).
// The RoPE inverse frequencies theta^(-2i/D) come in the launch arguments,
// evaluated once on the host in double and rounded to float.
// The whole step stays inside the warp that wrote the K/V row, so the write
// and the attention read need no cross-warp ordering.
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
  float inv_freq[64];  // RoPE theta^(-2i/D), i < D / 2
};

constexpr int kPvBatch = 16;  // cache positions whose V rows are in flight together

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
  // P.V: lane owns dims (2*lane, 2*lane+1) [+64 for D=128]; the V rows of a batch of positions
  // are all in flight before the first is used
  constexpr int J = D / 64;
  float acc[J][2];
#pragma unroll
  for (int j = 0; j < J; ++j) acc[j][0] = acc[j][1] = 0.f;
  const __nv_bfloat16* vbase = a.vc + row * a.c_row + kvh * a.c_head + 2 * lane;
  for (int p0 = 0; p0 < len; p0 += kPvBatch) {
    __nv_bfloat162 vv[kPvBatch][J];
#pragma unroll
    for (int b = 0; b < kPvBatch; ++b) {
#pragma unroll
      for (int j = 0; j < J; ++j) {
        vv[b][j] = p0 + b < len
                       ? *reinterpret_cast<const __nv_bfloat162*>(vbase + (p0 + b) * a.c_pos + 64 * j)
                       : __floats2bfloat162_rn(0.f, 0.f);
      }
    }
#pragma unroll
    for (int b = 0; b < kPvBatch; ++b) {
      const float pp = __shfl_sync(kFull, p, (p0 + b) & 31);
      if (p0 + b < len) {
#pragma unroll
        for (int j = 0; j < J; ++j) {
          const float2 vf = __bfloat1622float2(vv[b][j]);
          acc[j][0] = fmaf(pp, vf.x, acc[j][0]);
          acc[j][1] = fmaf(pp, vf.y, acc[j][1]);
        }
      }
    }
  }
  const float inv = 1.f / denom;
  __nv_bfloat16* orow = a.out + row * a.o_st + head * a.o_sh;
#pragma unroll
  for (int j = 0; j < J; ++j)
    *reinterpret_cast<__nv_bfloat162*>(orow + 64 * j + 2 * lane) =
        __floats2bfloat162_rn(acc[j][0] * inv, acc[j][1] * inv);
}

// The fused step, one warp per KV head: the warp normalises and rotates its
// G query heads and its K head (one sincos per lane serves all of them: the
// angle depends on the dimension and the position only), writes K and V of the
// new token into the cache, then attends for its G query heads over the
// cache, loading each K and V row once for the whole group.  Everything a warp
// reads it wrote itself or was written before the launch, so warps never wait
// on one another; a CTA is one row.
template <int D, int G>
__global__ void __launch_bounds__(256) cp_decode_group_kernel(const __grid_constant__ CpArgs a) {
  constexpr int J = D / 64, H = D / 2;
  __shared__ __align__(16) __nv_bfloat16 s_q[8][G][D];  // rotated q of each warp's heads
  const int row = blockIdx.x;
  const int kvh = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (kvh >= a.hkv) return;
  const float pos = static_cast<float>(a.pos[row * a.pos_stride]);

  // ---- load q heads, k, v of this group (all in flight together)
  float qf[G][J], qs[G][J], kf[J], ks[J];
  __nv_bfloat16 vf[J], vs[J];
  const __nv_bfloat16* kbase = a.k + row * a.k_st + kvh * a.k_sh;
  const __nv_bfloat16* vbase = a.v + row * a.v_st + kvh * a.v_sh;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int i = lane + 32 * j;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const __nv_bfloat16* qb = a.q + row * a.q_st + (kvh * G + g) * a.q_sh;
      qf[g][j] = __bfloat162float(qb[i]);
      qs[g][j] = __bfloat162float(qb[i + H]);
    }
    kf[j] = __bfloat162float(kbase[i]);
    ks[j] = __bfloat162float(kbase[i + H]);
    vf[j] = vbase[i];
    vs[j] = vbase[i + H];
  }
  float cs[J], sn[J];
#pragma unroll
  for (int j = 0; j < J; ++j) sincosf(pos * a.inv_freq[lane + 32 * j], &sn[j], &cs[j]);

  // ---- RMSNorm x weight, RoPE; q back in place and to shared memory, k in place and to the cache, v to the cache
  auto rotate = [&](float (&f)[J], float (&s)[J], const __nv_bfloat16* w) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) ss += f[j] * f[j] + s[j] * s[j];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + a.eps);
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = lane + 32 * j;
      const float x = f[j] * inv * __bfloat162float(w[i]);
      const float y = s[j] * inv * __bfloat162float(w[i + H]);
      f[j] = x * cs[j] - y * sn[j];
      s[j] = y * cs[j] + x * sn[j];
    }
  };
#pragma unroll
  for (int g = 0; g < G; ++g) {
    rotate(qf[g], qs[g], a.qw);
    __nv_bfloat16* qb = a.q + row * a.q_st + (kvh * G + g) * a.q_sh;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = lane + 32 * j;
      const __nv_bfloat16 x = __float2bfloat16_rn(qf[g][j]), y = __float2bfloat16_rn(qs[g][j]);
      qb[i] = x;
      qb[i + H] = y;
      s_q[kvh][g][i] = x;
      s_q[kvh][g][i + H] = y;
    }
  }
  rotate(kf, ks, a.kw);
  {
    __nv_bfloat16* kb = a.k + row * a.k_st + kvh * a.k_sh;
    __nv_bfloat16* kd = a.kc + row * a.c_row + static_cast<int64_t>(a.cache_position) * a.c_pos + kvh * a.c_head;
    __nv_bfloat16* vd = a.vc + row * a.c_row + static_cast<int64_t>(a.cache_position) * a.c_pos + kvh * a.c_head;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = lane + 32 * j;
      const __nv_bfloat16 x = __float2bfloat16_rn(kf[j]), y = __float2bfloat16_rn(ks[j]);
      kb[i] = x;
      kb[i + H] = y;
      kd[i] = x;
      kd[i + H] = y;
      vd[i] = vf[j];
      vd[i + H] = vs[j];
    }
  }
  __syncwarp();  // the cache row and s_q written above are read by other lanes below

  // ---- scores: lane p < len scores cache position p for every head of the group
  const int len = a.length;
  float score[G];
#pragma unroll
  for (int g = 0; g < G; ++g) score[g] = -__int_as_float(0x7f800000);
  if (lane < len) {
    const __nv_bfloat16* krow = a.kc + row * a.c_row + lane * a.c_pos + kvh * a.c_head;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
#pragma unroll
    for (int d = 0; d < D; d += 8) {
      const uint4 kv = *reinterpret_cast<const uint4*>(krow + d);
      const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint4 qv = *reinterpret_cast<const uint4*>(&s_q[kvh][g][d]);
        const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kk = __bfloat1622float2(k2[e]);
          const float2 qq = __bfloat1622float2(q2[e]);
          acc[g] = fmaf(qq.x, kk.x, acc[g]);
          acc[g] = fmaf(qq.y, kk.y, acc[g]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) score[g] = acc[g] * a.scale;
  }
  float p[G], inv[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float mx = warp_max(score[g]);
    p[g] = lane < len ? __expf(score[g] - mx) : 0.f;
    inv[g] = 1.f / warp_sum(p[g]);
  }

  // ---- P.V: lane owns dims (2 lane, 2 lane + 1) [+ 64 j]; a batch of V rows in flight together
  float o[G][J][2];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < J; ++j) o[g][j][0] = o[g][j][1] = 0.f;
  const __nv_bfloat16* vrow0 = a.vc + row * a.c_row + kvh * a.c_head + 2 * lane;
  for (int p0 = 0; p0 < len; p0 += kPvBatch) {
    __nv_bfloat162 vv[kPvBatch][J];
#pragma unroll
    for (int b = 0; b < kPvBatch; ++b)
#pragma unroll
      for (int j = 0; j < J; ++j)
        vv[b][j] = p0 + b < len ? *reinterpret_cast<const __nv_bfloat162*>(vrow0 + (p0 + b) * a.c_pos + 64 * j)
                                : __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
    for (int b = 0; b < kPvBatch; ++b) {
      if (p0 + b < len) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pp = __shfl_sync(kFull, p[g], (p0 + b) & 31);
#pragma unroll
          for (int j = 0; j < J; ++j) {
            const float2 vfl = __bfloat1622float2(vv[b][j]);
            o[g][j][0] = fmaf(pp, vfl.x, o[g][j][0]);
            o[g][j][1] = fmaf(pp, vfl.y, o[g][j][1]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    __nv_bfloat16* orow = a.out + row * a.o_st + (kvh * G + g) * a.o_sh;
#pragma unroll
    for (int j = 0; j < J; ++j)
      *reinterpret_cast<__nv_bfloat162*>(orow + 64 * j + 2 * lane) =
          __floats2bfloat162_rn(o[g][j][0] * inv[g], o[g][j][1] * inv[g]);
  }
}

template <int D>
__global__ void __launch_bounds__(1024) cp_short_kernel(const __grid_constant__ CpArgs a) {
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
           sm_scale, static_cast<__nv_bfloat16*>(out), out_stride_tok, out_stride_head, status, {}};
  rope_inv_freq_table(a.inv_freq, head_dim, rope_theta);
  const int group = num_qo_heads / num_kv_heads;
  if (num_kv_heads > 8 || (group != 1 && group != 2 && group != 4)) return NQT_ERR_UNSUPPORTED;
  if (cache_capacity > 32) return NQT_ERR_UNSUPPORTED;
  const int threads = 32 * num_kv_heads;
  cudaStream_t s = as_stream(stream);
  if (head_dim == 64) {
    if (group == 1) cp_decode_group_kernel<64, 1><<<rows, threads, 0, s>>>(a);
    if (group == 2) cp_decode_group_kernel<64, 2><<<rows, threads, 0, s>>>(a);
    if (group == 4) cp_decode_group_kernel<64, 4><<<rows, threads, 0, s>>>(a);
  } else {
    if (group == 1) cp_decode_group_kernel<128, 1><<<rows, threads, 0, s>>>(a);
    if (group == 2) cp_decode_group_kernel<128, 2><<<rows, threads, 0, s>>>(a);
    if (group == 4) cp_decode_group_kernel<128, 4><<<rows, threads, 0, s>>>(a);
  }
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
