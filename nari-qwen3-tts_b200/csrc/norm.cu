// Talker layer glue: RMSNorm, fused residual add + RMSNorm, SwiGLU.
//
// One CTA per token row, 16-byte vector loads, fp32 math, one launch each.
// Semantics of the reference's CUDA boundary (model/layers.py:28-100):
//   rmsnorm:            out = x * rsqrt(mean(x^2) + eps) * w           (flashinfer.norm.rmsnorm)
//   fused_add_rmsnorm:  r = x + residual (fp32); residual <- r;
//                       x <- r * rsqrt(mean(r^2) + eps) * w             (flashinfer.norm.fused_add_rmsnorm)
//   silu_and_mul:       out = silu(g) * u for gate_up = [g | u]          (flashinfer.activation.silu_and_mul)
//   fused_add_rmsnorm_fp8: fused_add_rmsnorm whose bf16 output is quantised to e4m3 per 128-element block
//                       (the activation rule of the reference's FP8 gate/up GEMM, fp8.cuh) for the FP8
//                       gate/up GEMM that follows; it lets that GEMM be scheduled at once (PDL) so the
//                       weight stream starts while the norm runs.
#include "common.cuh"
#include "fp8.cuh"

namespace nqt {
namespace {

constexpr int kNormThreads = 256;

template <typename T>
struct Vec8 {
  uint4 raw;
  __device__ __forceinline__ float get(int i) const {
    const T* p = reinterpret_cast<const T*>(&raw);
    return to_f32(p[i]);
  }
  __device__ __forceinline__ void set(int i, float v) {
    T* p = reinterpret_cast<T*>(&raw);
    p[i] = from_f32<T>(v);
  }
};

__device__ __forceinline__ float block_sum(float v) {
  __shared__ float s[kNormThreads / 32];
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s[warp] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) r += s[w];
  return r;
}

// hidden <= kNormThreads * 8 * kMaxVec
constexpr int kMaxVec = 4;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const T* x, int64_t xs, const T* w, T* out,
                                                               int64_t os, int hidden, float eps) {
  const int row = blockIdx.x;
  const int nvec = hidden / 8;
  Vec8<T> v[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < nvec) {
      v[j].raw = reinterpret_cast<const uint4*>(x + row * xs)[i];
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[j].get(e) * v[j].get(e);
    }
  }
  const float inv = rsqrtf(block_sum(ss) / hidden + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < nvec) {
      Vec8<T> wv;
      wv.raw = reinterpret_cast<const uint4*>(w)[i];
      Vec8<T> o;
#pragma unroll
      for (int e = 0; e < 8; ++e) o.set(e, v[j].get(e) * inv * wv.get(e));
      reinterpret_cast<uint4*>(out + row * os)[i] = o.raw;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(T* x, T* residual, const T* w, int hidden,
                                                                   float eps) {
  const int row = blockIdx.x;
  const int nvec = hidden / 8;
  float r[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < nvec) {
      Vec8<T> a, b, o;
      a.raw = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * hidden)[i];
      b.raw = reinterpret_cast<const uint4*>(residual + static_cast<int64_t>(row) * hidden)[i];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        r[j][e] = a.get(e) + b.get(e);
        ss += r[j][e] * r[j][e];
        o.set(e, r[j][e]);
      }
      reinterpret_cast<uint4*>(residual + static_cast<int64_t>(row) * hidden)[i] = o.raw;
    }
  }
  const float inv = rsqrtf(block_sum(ss) / hidden + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < nvec) {
      Vec8<T> wv, o;
      wv.raw = reinterpret_cast<const uint4*>(w)[i];
#pragma unroll
      for (int e = 0; e < 8; ++e) o.set(e, r[j][e] * inv * wv.get(e));
      reinterpret_cast<uint4*>(x + static_cast<int64_t>(row) * hidden)[i] = o.raw;
    }
  }
}

// add_rmsnorm for bf16 rows with hidden % 128 == 0; the normed row is rounded to bf16, then each
// 128-element block (16 vectors = 16 consecutive lanes) is quantised to e4m3 with its own scale.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_fp8_kernel(__nv_bfloat16* x, __nv_bfloat16* residual,
                                                                       const __nv_bfloat16* w, int hidden, float eps,
                                                                       uint8_t* q, int64_t ldq, float* scale,
                                                                       int64_t ld_scale, int write_x) {
  grid_dependents_launch();  // the FP8 GEMM after this kernel may start streaming its weights
  const int row = blockIdx.x;
  const int nvec = hidden / 8;
  float r[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < nvec) {
      Vec8<__nv_bfloat16> a, b, o;
      a.raw = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * hidden)[i];
      b.raw = reinterpret_cast<const uint4*>(residual + static_cast<int64_t>(row) * hidden)[i];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        r[j][e] = a.get(e) + b.get(e);
        ss += r[j][e] * r[j][e];
        o.set(e, r[j][e]);
      }
      reinterpret_cast<uint4*>(residual + static_cast<int64_t>(row) * hidden)[i] = o.raw;
    }
  }
  const float inv = rsqrtf(block_sum(ss) / hidden + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    if (j * kNormThreads >= nvec) break;  // uniform over the CTA
    const int i = threadIdx.x + j * kNormThreads;
    Vec8<__nv_bfloat16> o;
    float v[8];
    float amax = 0.f;
    if (i < nvec) {
      Vec8<__nv_bfloat16> wv;
      wv.raw = reinterpret_cast<const uint4*>(w)[i];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o.set(e, r[j][e] * inv * wv.get(e));
        v[e] = o.get(e);
        amax = fmaxf(amax, fabsf(v[e]));
      }
    }
    // whole 16-lane groups are valid or not (nvec % 16 == 0)
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, off));
    if (i < nvec) {
      const float f = fp8::act_block_factor(amax);
      uint2 pk;
      pk.x = fp8::e4m3x4(v[0] * f, v[1] * f, v[2] * f, v[3] * f);
      pk.y = fp8::e4m3x4(v[4] * f, v[5] * f, v[6] * f, v[7] * f);
      *reinterpret_cast<uint2*>(q + static_cast<int64_t>(row) * ldq + i * 8) = pk;
      if ((i & 15) == 0) scale[static_cast<int64_t>(i >> 4) * ld_scale + row] = __fdiv_rn(1.f, f);
      if (write_x) reinterpret_cast<uint4*>(x + static_cast<int64_t>(row) * hidden)[i] = o.raw;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) silu_mul_kernel(const T* gu, int64_t gs, T* out, int64_t os, int d) {
  const int row = blockIdx.y;
  const int i = blockIdx.x * kNormThreads + threadIdx.x;  // vector index
  if (i >= d / 8) return;
  Vec8<T> g, u, o;
  g.raw = reinterpret_cast<const uint4*>(gu + row * gs)[i];
  u.raw = reinterpret_cast<const uint4*>(gu + row * gs + d)[i];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float gv = g.get(e);
    o.set(e, gv / (1.f + __expf(-gv)) * u.get(e));
  }
  reinterpret_cast<uint4*>(out + row * os)[i] = o.raw;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_rmsnorm(const void* x, int64_t x_stride, const void* weight, void* out, int64_t out_stride,
                           int rows, int hidden, float eps, int dtype, void* stream) {
  if (!x || !weight || !out || rows < 0 || hidden < 8 || hidden % 8) return NQT_ERR_ARG;
  if (hidden > kNormThreads * 8 * kMaxVec) return NQT_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || (x_stride % 8) || (out_stride % 8)) return NQT_ERR_ARG;
  if (rows == 0) return NQT_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype == NQT_BF16)
    rmsnorm_kernel<__nv_bfloat16><<<rows, kNormThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), x_stride, static_cast<const __nv_bfloat16*>(weight),
        static_cast<__nv_bfloat16*>(out), out_stride, hidden, eps);
  else if (dtype == NQT_F16)
    rmsnorm_kernel<__half><<<rows, kNormThreads, 0, s>>>(static_cast<const __half*>(x), x_stride,
                                                         static_cast<const __half*>(weight), static_cast<__half*>(out),
                                                         out_stride, hidden, eps);
  else
    return NQT_ERR_UNSUPPORTED;
  return check_launch("rmsnorm");
}

extern "C" int nqt_fused_add_rmsnorm(void* x, void* residual, const void* weight, int rows, int hidden, float eps,
                                     int dtype, void* stream) {
  if (!x || !residual || !weight || rows < 0 || hidden < 8 || hidden % 8 || x == residual) return NQT_ERR_ARG;
  if (hidden > kNormThreads * 8 * kMaxVec) return NQT_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(residual) || !aligned16(weight)) return NQT_ERR_ARG;
  if (rows == 0) return NQT_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype == NQT_BF16)
    add_rmsnorm_kernel<__nv_bfloat16><<<rows, kNormThreads, 0, s>>>(
        static_cast<__nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(residual),
        static_cast<const __nv_bfloat16*>(weight), hidden, eps);
  else if (dtype == NQT_F16)
    add_rmsnorm_kernel<__half><<<rows, kNormThreads, 0, s>>>(static_cast<__half*>(x), static_cast<__half*>(residual),
                                                             static_cast<const __half*>(weight), hidden, eps);
  else
    return NQT_ERR_UNSUPPORTED;
  return check_launch("fused_add_rmsnorm");
}

extern "C" int nqt_fused_add_rmsnorm_fp8(void* x, void* residual, const void* weight, int rows, int hidden, float eps,
                                         void* q, int64_t ldq, float* scale, int64_t ld_scale, int write_x, int dtype,
                                         void* stream) {
  if (!x || !residual || !weight || !q || !scale || rows < 0 || hidden < 128 || hidden % 128 || x == residual)
    return NQT_ERR_ARG;
  if (dtype != NQT_BF16) return NQT_ERR_UNSUPPORTED;
  if (hidden > kNormThreads * 8 * kMaxVec) return NQT_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(residual) || !aligned16(weight)) return NQT_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(q) & 7) || ldq % 8 || ldq < hidden || ld_scale < rows ||
      (reinterpret_cast<uintptr_t>(scale) & 3))
    return NQT_ERR_ARG;
  if (rows == 0) return NQT_OK;
  add_rmsnorm_fp8_kernel<<<rows, kNormThreads, 0, as_stream(stream)>>>(
      static_cast<__nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(residual),
      static_cast<const __nv_bfloat16*>(weight), hidden, eps, static_cast<uint8_t*>(q), ldq, scale, ld_scale,
      write_x ? 1 : 0);
  return check_launch("fused_add_rmsnorm_fp8");
}

extern "C" int nqt_silu_and_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride, int rows,
                                int d, int dtype, void* stream) {
  if (!gate_up || !out || rows < 0 || d < 8 || d % 8) return NQT_ERR_ARG;
  if (!aligned16(gate_up) || !aligned16(out) || (gate_up_stride % 8) || (out_stride % 8)) return NQT_ERR_ARG;
  if (rows == 0) return NQT_OK;
  if (rows > 65535) return NQT_ERR_UNSUPPORTED;
  cudaStream_t s = as_stream(stream);
  dim3 grid((d / 8 + kNormThreads - 1) / kNormThreads, rows);
  if (dtype == NQT_BF16)
    silu_mul_kernel<__nv_bfloat16><<<grid, kNormThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(gate_up),
                                                                 gate_up_stride, static_cast<__nv_bfloat16*>(out),
                                                                 out_stride, d);
  else if (dtype == NQT_F16)
    silu_mul_kernel<__half><<<grid, kNormThreads, 0, s>>>(static_cast<const __half*>(gate_up), gate_up_stride,
                                                          static_cast<__half*>(out), out_stride, d);
  else
    return NQT_ERR_UNSUPPORTED;
  return check_launch("silu_and_mul");
}
