// Code-predictor frame glue between two depth steps, one launch instead of
// six (executor/code_predictor.py:160-235, the whole-frame loop, with
// model/components.py:254-258 for the next step's input norm).
//
// After codebook g's token is sampled, per row:
//   frames[row, g]  = token
//   codec_sum[row]  = bf16(codec_sum[row] + codec_emb[token])      (accumulate; = codec_emb[token] for g = 0)
//   residual[row]   = proj_emb[token]                               (the next depth step's input)
//   h[row]          = bf16(rmsnorm(residual[row]) * ln)             (its first layer's input norm)
// The additions and the norm round exactly as the unfused torch / nqt ops do
// (bf16(fp32 a + fp32 b); fp32 sum of squares, rsqrt, x * inv * w rounded once).
// One CTA of 256 threads per row; 16-byte vectors.  A token outside
// [0, vocab) is reported as NQT_DEV_BAD_TOKEN and its row is left unchanged.
#include "common.cuh"

namespace nqt {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxVec = 2;  // widths up to 256 * 8 * 2 = 4096 elements

struct CodecStepArgs {
  const int64_t* tokens;
  int64_t* frames;  // frames[row * frames_stride] (the codebook's column)
  int64_t frames_stride;
  const __nv_bfloat16* codec_emb;  // [vocab, talker_hidden]
  __nv_bfloat16* codec_sum;        // [rows, talker_hidden]
  const __nv_bfloat16* proj_emb;   // [vocab, hidden] or null (last codebook)
  const __nv_bfloat16* ln;         // [hidden]
  __nv_bfloat16* residual;         // [rows, hidden]
  __nv_bfloat16* h;                // [rows, hidden]
  int32_t* status;
  int vocab, talker_hidden, hidden, accumulate;
  float eps;
};

__device__ __forceinline__ float bf(const uint4& v, int e) {
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&v)[e]);
}
__device__ __forceinline__ void set_bf(uint4& v, int e, float x) {
  reinterpret_cast<__nv_bfloat16*>(&v)[e] = __float2bfloat16_rn(x);
}

__global__ void __launch_bounds__(kThreads) codec_step_kernel(CodecStepArgs a) {
  __shared__ float s_red[kThreads / 32];
  const int row = blockIdx.x;
  const int64_t token = a.tokens[row];
  if (token < 0 || token >= a.vocab) {
    if (threadIdx.x == 0) report(a.status, NQT_DEV_BAD_TOKEN);
    return;
  }
  if (threadIdx.x == 0) a.frames[row * a.frames_stride] = token;
  // codec embedding sum (talker width)
  const uint4* src = reinterpret_cast<const uint4*>(a.codec_emb + token * a.talker_hidden);
  uint4* sum = reinterpret_cast<uint4*>(a.codec_sum + static_cast<int64_t>(row) * a.talker_hidden);
  for (int i = threadIdx.x; i < a.talker_hidden / 8; i += kThreads) {
    const uint4 e = src[i];
    if (a.accumulate) {
      uint4 s = sum[i];
#pragma unroll
      for (int j = 0; j < 8; ++j) set_bf(s, j, bf(s, j) + bf(e, j));
      sum[i] = s;
    } else {
      sum[i] = e;
    }
  }
  if (a.proj_emb == nullptr) return;
  // next depth step's input and its first input norm
  const uint4* p = reinterpret_cast<const uint4*>(a.proj_emb + token * a.hidden);
  uint4* res = reinterpret_cast<uint4*>(a.residual + static_cast<int64_t>(row) * a.hidden);
  const int nvec = a.hidden / 8;
  uint4 x[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      x[j] = p[i];
      res[i] = x[j];
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += bf(x[j], e) * bf(x[j], e);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) tot += s_red[w];
  const float inv = rsqrtf(tot / a.hidden + a.eps);
  const uint4* lw = reinterpret_cast<const uint4*>(a.ln);
  uint4* hv = reinterpret_cast<uint4*>(a.h + static_cast<int64_t>(row) * a.hidden);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      const uint4 w = lw[i];
      uint4 o;
#pragma unroll
      for (int e = 0; e < 8; ++e) set_bf(o, e, bf(x[j], e) * inv * bf(w, e));
      hv[i] = o;
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_cp_codec_step(const int64_t* tokens, int rows, int64_t* frames, int64_t frames_stride,
                                 const void* codec_emb, int vocab, int talker_hidden, void* codec_sum, int accumulate,
                                 const void* proj_emb, const void* ln, int hidden, float eps, void* residual, void* h,
                                 int dtype, int32_t* status, void* stream) {
  if (!tokens || !frames || !codec_emb || !codec_sum || rows < 0 || vocab < 1 || talker_hidden < 8 ||
      talker_hidden % 8 || frames_stride < 1)
    return NQT_ERR_ARG;
  if (dtype != NQT_BF16) return NQT_ERR_UNSUPPORTED;
  if (!aligned16(codec_emb) || !aligned16(codec_sum)) return NQT_ERR_ARG;
  if (proj_emb != nullptr) {
    if (!ln || !residual || !h || hidden < 8 || hidden % 8) return NQT_ERR_ARG;
    if (hidden > kThreads * 8 * kMaxVec) return NQT_ERR_UNSUPPORTED;
    if (!aligned16(proj_emb) || !aligned16(ln) || !aligned16(residual) || !aligned16(h)) return NQT_ERR_ARG;
  }
  if (rows == 0) return NQT_OK;
  CodecStepArgs a{tokens,
                  frames,
                  frames_stride,
                  static_cast<const __nv_bfloat16*>(codec_emb),
                  static_cast<__nv_bfloat16*>(codec_sum),
                  static_cast<const __nv_bfloat16*>(proj_emb),
                  static_cast<const __nv_bfloat16*>(ln),
                  static_cast<__nv_bfloat16*>(residual),
                  static_cast<__nv_bfloat16*>(h),
                  status,
                  vocab,
                  talker_hidden,
                  hidden,
                  accumulate ? 1 : 0,
                  eps};
  codec_step_kernel<<<rows, kThreads, 0, as_stream(stream)>>>(a);
  return check_launch("cp_codec_step");
}
