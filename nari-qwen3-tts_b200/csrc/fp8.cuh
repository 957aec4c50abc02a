// FP8 (e4m3) quantisation rules shared by the gate/up quantisers
// (gemm_fp8.cu) and the fused add + RMSNorm that feeds the FP8 GEMM
// (norm.cu).
//
// Weight blocks (model/layers.py:11-25): per 128 x 128 block,
//   s = 2^ceil(log2(max(amax, 1e-4) / 448)),  q = e4m3(w / s).
// Activation blocks (the bf16-input path of the reference's FP8 GEMM,
// flashinfer fp8_blockscale_gemm_sm90: one scale per token per 128 K):
//   f = 448 / amax (1 when amax = 0),  q = e4m3(x * f),  scale = 1 / f.
// All arithmetic is fp32 with IEEE rounding; e4m3 conversion rounds to
// nearest even and saturates at +-448 (no value exceeds it by construction).
#pragma once

#include <cuda_fp8.h>

#include "common.cuh"

namespace nqt {
namespace fp8 {

constexpr float kE4m3Max = 448.f;

// ceil(log2(x)) for a normal positive float, exact: the exponent, plus one unless x is a power of two.
__device__ __forceinline__ int ceil_log2(float x) {
  const uint32_t bits = __float_as_uint(x);
  const int e = static_cast<int>((bits >> 23) & 0xffu) - 127;
  return (bits & 0x7fffffu) != 0u ? e + 1 : e;
}

// 2^e as a float, for -126 <= e <= 127.
__device__ __forceinline__ float exp2_int(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

// Power-of-two scale exponent of a weight block with absolute maximum `amax` (finite).
__device__ __forceinline__ int weight_block_exponent(float amax) {
  return ceil_log2(__fdiv_rn(fmaxf(amax, 1e-4f), kE4m3Max));
}

// Quantisation factor of an activation block: q = e4m3(x * f), dequantisation scale 1 / f.
__device__ __forceinline__ float act_block_factor(float amax) {
  return amax != 0.f ? __fdiv_rn(kE4m3Max, amax) : 1.f;
}

// Four values -> four e4m3 bytes (little-endian: a in the lowest byte).
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

}  // namespace fp8
}  // namespace nqt
