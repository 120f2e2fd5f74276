// Per-row RMSNorm + FP8 e4m3 arithmetic shared by the standalone quantizer (rmsnorm_fp8.cu) and
// the decode GEMV's fused RMSNorm prologue (w4a16_gemv.cu), so both round identically. The rule
// (reference tokenforge/kernels/reference.py:35-56, triton/rmsnorm_fp8.py:44-73):
//   rstd  = 1 / sqrt_rn(fp32(sum x^2) / H + eps), y = fp16(x * rstd) * weight (fp16 product),
//   scale = max(amax|y| / 448, 1 / (448 * 512)), q = e4m3_rne(clamp(y / scale, -448, 448)).
//
// These row kernels are bound by instruction issue unless every element costs only a few
// instructions, so the helpers work on 16-byte vectors (8 fp16 values) with packed instructions:
// fp16x2 products and maxima, the sm_100 packed fp32 multiply / FMA (.f32x2), and a division by
// the row's scale built from FMAs (quant_pair_fma) instead of one IEEE division per element.
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

// The sum of squares is accumulated in fp64: every fp16 square is exact (22 significant bits)
// and the fp64 sum of up to ~1e6 of them is exact or within 2^-53, so its fp32 rounding does
// not depend on the summation order (threads, warps, the CPU oracle all obtain the same fp32
// sum). One conversion and one fp64 FMA per element: fma(d, d, s) rounds d * d + s once and
// d * d is exact, so it equals the fp64 sum of the exact square.
__device__ __forceinline__ void acc_sumsq(const uint4& v, double& s) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    double d;
    asm("cvt.f64.f16 %0, %1;" : "=d"(d) : "h"(h[e]));
    s = __fma_rn(d, d, s);
  }
}

__device__ __forceinline__ float rstd_of(double sumsq, int64_t H, float eps) {
  const float var = __fdiv_rn(__double2float_rn(sumsq), static_cast<float>(H));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

__device__ __forceinline__ float dyn_scale(float amax) {
  return fmaxf(__fdiv_rn(amax, kFp8Max), kMinScale);
}

// Packed fp32 pairs (sm_100 .f32x2 instructions; low half = first element).
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t h2_to_f32x2(__half2 h) {
  const float2 f = __half22float2(h);
  return f32x2(f.x, f.y);
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ float2 split_f32x2(uint64_t v) {
  float2 f;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(v));
  return f;
}

// -w for a vector of 8 fp16 weights (sign flips; exact).
__device__ __forceinline__ uint4 neg_weight(uint4 w) {
  w.x ^= 0x80008000u;
  w.y ^= 0x80008000u;
  w.z ^= 0x80008000u;
  w.w ^= 0x80008000u;
  return w;
}

// y = fp16(fp16(x * rstd) * w) for one vector of 8 values, returned NEGATED (-y), which is the
// form quant_pair divides: nw holds -w (neg_weight), and RN(n * -w) = -RN(n * w) exactly. |y| is
// folded into amax2 (fp16 maxima ignore NaN as fmaxf does, so a NaN element never becomes the
// row's maximum). rstd2 = (rstd, rstd).
__device__ __forceinline__ uint4 norm_vec_neg(const uint4& x, const uint4& nw, uint64_t rstd2,
                                              __half2& amax2) {
  uint4 out;
  const __half2* x2 = reinterpret_cast<const __half2*>(&x);
  const __half2* w2 = reinterpret_cast<const __half2*>(&nw);
  __half2* o2 = reinterpret_cast<__half2*>(&out);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 n = split_f32x2(mul_f32x2(h2_to_f32x2(x2[e]), rstd2));
    const __half2 ny = __hmul2(__floats2half2_rn(n.x, n.y), w2[e]);
    amax2 = __hmax2(amax2, __habs2(ny));
    o2[e] = ny;
  }
  return out;
}

// A row's divisor for the e4m3 step. Dynamic scales always lie in [1 / (448 * 512), 65504 / 448];
// a static scale outside [2^-60, 2^60], or Inf / NaN, takes the IEEE division path.
struct Fp8Div {
  float scale;
  uint64_t b2;   // (scale, scale)
  uint64_t nr2;  // (-r, -r), r = 1 / scale rounded to nearest
  bool fma_ok;
};
__device__ __forceinline__ Fp8Div fp8_div(float scale) {
  Fp8Div d;
  d.scale = scale;
  d.fma_ok = scale >= 0x1p-60f && scale <= 0x1p60f;
  const float nr = -__frcp_rn(scale);
  d.b2 = f32x2(scale, scale);
  d.nr2 = f32x2(nr, nr);
  return d;
}

// Division paths of the e4m3 step (one per row or per thread, chosen by quant_path).
enum QuantPath : int { kIeee = 0, kFma2 = 1, kFma1 = 2 };

// Two e4m3 codes (low byte: first element) of e4m3_rne(clamp(y / scale, -448, 448)) for the
// pair ny = (-y0, -y1), |y| finite, d.fma_ok. The quotient is y / scale rounded to nearest fp32
// exactly as an IEEE division rounds it, from the reciprocal r = RN(1 / b) by residual
// corrections (P. Markstein, "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990; the theorem as stated in Muller et al., Handbook of
// Floating-Point Arithmetic, 2nd ed., section 4.7): q0 = RN(a r) is within 1.5 ulp of a / b;
// q1 = RN(q0 + RN(a - b q0) r) is within half an ulp plus 2^-22 ulp; its residual a - b q1 is
// exact in fp32 (an fp16 a and |a / b| in [2^-84, 2^76] keep every step normal), and with r
// correctly rounded and q1 within one ulp, q2 = RN(q1 + (a - b q1) r) = RN(a / b) (kFma2, any
// scale in range). q1 alone differs from RN(a / b) only when a / b lies within 2^-22 ulp of an
// fp32 midpoint, and changes the e4m3 code only when that midpoint is next to an e4m3 rounding
// boundary; for the scales the dynamic rule produces (max(h / 448, 1 / (448 * 512)), h a
// positive fp16) and every fp16 a with |a| <= h no such pair exists, which the exhaustive GPU
// test over all of them establishes (kFma1, dynamic scales only). Working on -a keeps the sign
// of zero: the residual of +-0 is +0, and q + (+0) * (-r) = q for q = -0 as well.
template <int kSteps>
__device__ __forceinline__ uint16_t quant_pair_fma(__half2 ny, const Fp8Div& d) {
  const uint64_t na = h2_to_f32x2(ny);
  uint64_t q = mul_f32x2(na, d.nr2);
#pragma unroll
  for (int i = 0; i < kSteps; ++i) q = fma_f32x2(fma_f32x2(q, d.b2, na), d.nr2, q);
  const float2 f = split_f32x2(q);
  uint16_t code;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(code) : "f"(f.y), "f"(f.x));
  return code;
}

// The same codes by IEEE division (Inf y, static scales outside the FMA path's range).
__device__ __forceinline__ uint16_t quant_pair_ieee(__half2 ny, const Fp8Div& d) {
  const float2 f = __half22float2(ny);
  const float lo = __fdiv_rn(-f.x, d.scale), hi = __fdiv_rn(-f.y, d.scale);
  uint16_t code;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(code) : "f"(hi), "f"(lo));
  return code;
}

template <int kPath>
__device__ __forceinline__ uint16_t quant_pair(__half2 ny, const Fp8Div& d) {
  if constexpr (kPath == kFma1) return quant_pair_fma<1>(ny, d);
  else if constexpr (kPath == kFma2) return quant_pair_fma<2>(ny, d);
  else return quant_pair_ieee(ny, d);
}

// The path of a row (or of a thread's part of it): IEEE division unless the scale is in the
// FMA path's range and the |y| are finite; one correction step for a dynamic scale.
__device__ __forceinline__ int quant_path(const Fp8Div& d, bool finite, bool dynamic) {
  return !(d.fma_ok && finite) ? kIeee : dynamic ? kFma1 : kFma2;
}

// Eight codes (one 8-byte word) of a vector of -y values. Callers branch on the path once per
// row (quant_row), not per pair: with the branch inside the vector loop every side is issued.
template <int kPath>
__device__ __forceinline__ uint2 quant_vec(const uint4& ny, const Fp8Div& d) {
  const __half2* h = reinterpret_cast<const __half2*>(&ny);
  uint32_t c[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) c[e] = quant_pair<kPath>(h[e], d);
  return make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
}

// Writes the codes of a thread's N vectors of -y (v[i] is column vector col(i) of the row, valid
// while col(i) < nvec) to qr, on one path for all of them.
template <int N, typename Col>
__device__ __forceinline__ void quant_row(const uint4 (&v)[N], int64_t nvec, Col col,
                                          const Fp8Div& d, int path, uint2* qr) {
  if (path == kFma1) {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (col(i) < nvec) qr[col(i)] = quant_vec<kFma1>(v[i], d);
  } else if (path == kFma2) {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (col(i) < nvec) qr[col(i)] = quant_vec<kFma2>(v[i], d);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (col(i) < nvec) qr[col(i)] = quant_vec<kIeee>(v[i], d);
  }
}

// True when both halves of a thread's |y| maximum are finite (no Inf among its elements).
__device__ __forceinline__ bool amax_finite(__half2 amax2) {
  const uint32_t b = *reinterpret_cast<const uint32_t*>(&amax2);
  return (b & 0x7FFFu) < 0x7C00u && ((b >> 16) & 0x7FFFu) < 0x7C00u;
}

__device__ __forceinline__ float amax_of(__half2 amax2) {
  return fmaxf(__low2float(amax2), __high2float(amax2));
}

// SiLU-gated product in fp32 (before its fp16 rounding): silu(g) * u = g / (1 + exp(-g)) * u,
// shared by the standalone kernel and the GEMV's fused staging so both round identically.
__device__ __forceinline__ float silu_mul_f32(float g, float u) {
  return g / (1.0f + expf(-g)) * u;
}

}  // namespace tfb
