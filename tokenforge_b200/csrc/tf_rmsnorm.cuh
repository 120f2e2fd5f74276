// Per-row RMSNorm + FP8 e4m3 arithmetic shared by the standalone quantizer (rmsnorm_fp8.cu) and
// the decode GEMV's fused RMSNorm prologue (w4a16_gemv.cu), so both round identically. The rule
// (reference tokenforge/kernels/reference.py:35-56, triton/rmsnorm_fp8.py:44-73):
//   rstd  = 1 / sqrt_rn(fp32(sum x^2) / H + eps), y = fp16(x * rstd) * weight (fp16 product),
//   scale = max(amax|y| / 448, 1 / (448 * 512)), q = e4m3_rne(clamp(y / scale, -448, 448)).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace tfb {

constexpr float kFp8Max = 448.0f;
constexpr float kMinScale = 1.0f / (448.0f * 512.0f);

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The sum of squares is accumulated in fp64: every fp16 square is exact in fp32 and the fp64 sum
// of up to ~1e6 of them is exact or within 2^-53, so its fp32 rounding does not depend on the
// summation order (threads, warps, the CPU oracle all obtain the same fp32 sum).
__device__ __forceinline__ float rstd_of(double sumsq, int64_t H, float eps) {
  const float var = __fdiv_rn(__double2float_rn(sumsq), static_cast<float>(H));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

__device__ __forceinline__ float dyn_scale(float amax) {
  return fmaxf(__fdiv_rn(amax, kFp8Max), kMinScale);
}

// SiLU-gated product in fp32 (before its fp16 rounding): silu(g) * u = g / (1 + exp(-g)) * u,
// shared by the standalone kernel and the GEMV's fused staging so both round identically.
__device__ __forceinline__ float silu_mul_f32(float g, float u) {
  return g / (1.0f + expf(-g)) * u;
}

}  // namespace tfb
