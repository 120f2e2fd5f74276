/*
 * tf_oracle.c — CPU restatement of the reference's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load this code, and only as the checker (or as the timed CPU baseline); the product
 * path (tokenforge_b200/) never calls it. Each function cites the reference file:line it
 * restates (paths inside saransh-debugs/TokenForge). The restatement is pinned against golden
 * vectors produced by running the reference itself (tests/golden/make_golden.py).
 *
 * fp16 arithmetic uses the compiler's IEEE binary16 type (_Float16): conversions round to
 * nearest even and a binary16 product is computed exactly in binary32 and rounded once, which
 * is what torch's CPU Half arithmetic does.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

typedef _Float16 f16;

static const int kOrder[8] = {0, 2, 4, 6, 1, 3, 5, 7};   /* AWQ_ORDER, pack.py:32 */
static const int kReverse[8] = {0, 4, 1, 5, 2, 6, 3, 7}; /* AWQ_REVERSE_ORDER, pack.py:35 */

static inline f16 h_from_bits(uint16_t b) {
  f16 h;
  memcpy(&h, &b, 2);
  return h;
}
static inline uint16_t h_to_bits(f16 h) {
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}

/* unpack_int4, pack.py:57-67: value j of word w = (w >> 4 * AWQ_REVERSE_ORDER[j]) & 0xF. */
void oracle_unpack_int4(const int32_t* packed, int64_t n_words, int32_t* values) {
  for (int64_t w = 0; w < n_words; ++w) {
    const uint32_t v = (uint32_t)packed[w];
    for (int j = 0; j < 8; ++j) values[8 * w + j] = (int32_t)((v >> (4 * kReverse[j])) & 0xFu);
  }
}

/* pack_int4, pack.py:42-54: word |= value[AWQ_ORDER[i]] << 4i (values assumed in [0, 15]). */
void oracle_pack_int4(const int32_t* values, int64_t n_words, int32_t* packed) {
  for (int64_t w = 0; w < n_words; ++w) {
    uint32_t word = 0;
    for (int i = 0; i < 8; ++i) word |= ((uint32_t)values[8 * w + kOrder[i]] & 0xFu) << (4 * i);
    packed[w] = (int32_t)word;
  }
}

/* Logical int4 value (row k, column n) of an AWQ-packed [K, N/8] matrix (awq_unpack,
 * pack.py:78-80). */
static inline uint32_t awq_value(const int32_t* q, int64_t n8, int64_t k, int64_t n) {
  return ((uint32_t)q[k * n8 + n / 8] >> (4 * kReverse[n % 8])) & 0xFu;
}

/* repack_awq_to_tf, pack.py:141-143: pack_int4(awq_unpack(qweight).t()).
 * qweight [K, N/8] -> qweight_t [N, K/8]. */
void oracle_repack_awq_to_tf(const int32_t* qweight, int64_t K, int64_t N, int32_t* qweight_t) {
  const int64_t n8 = N / 8, k8 = K / 8;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t kw = 0; kw < k8; ++kw) {
      uint32_t word = 0;
      for (int i = 0; i < 8; ++i) word |= awq_value(qweight, n8, 8 * kw + kOrder[i], n) << (4 * i);
      qweight_t[n * k8 + kw] = (int32_t)word;
    }
}

/* Dequantized weight (n, k) in the kernel layout: fp16(q - z) * s with one rounding
 * (dequantize_tf, pack.py:189-194). */
static inline f16 tf_weight(const int32_t* qweight_t, const uint16_t* scales,
                            const int32_t* qzeros, int64_t N, int64_t K, int64_t G, int64_t n,
                            int64_t k) {
  const uint32_t q = ((uint32_t)qweight_t[n * (K / 8) + k / 8] >> (4 * kReverse[k % 8])) & 0xFu;
  const int64_t g = k / G;
  const uint32_t z = awq_value(qzeros, N / 8, g, n);
  const f16 d = (f16)((int32_t)q - (int32_t)z);
  return d * h_from_bits(scales[g * N + n]);
}

/* dequantize_tf, pack.py:189-194: kernel layout -> fp16 [N, K]. */
void oracle_dequantize_tf(const int32_t* qweight_t, const uint16_t* scales,
                          const int32_t* qzeros, int64_t N, int64_t K, int64_t G, uint16_t* out) {
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k)
      out[n * K + k] = h_to_bits(tf_weight(qweight_t, scales, qzeros, N, K, G, n, k));
}

/* w4a16_reference, reference.py:13-21: fp64 x @ dequant(W)^T (+ bias) on the fp16-rounded
 * weights. x fp16 [M, K], out fp64 [M, N]. */
void oracle_w4a16_ref_f64(const uint16_t* x, int64_t M, int64_t K, const int32_t* qweight_t,
                          const uint16_t* scales, const int32_t* qzeros, const uint16_t* bias,
                          int64_t N, int64_t G, double* out) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t m = 0; m < M; ++m) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k)
        acc += (double)h_from_bits(x[m * K + k]) *
               (double)tf_weight(qweight_t, scales, qzeros, N, K, G, n, k);
      if (bias) acc += (double)h_from_bits(bias[n]);
      out[m * N + n] = acc;
    }
  }
}

/* w4a16_torch, reference.py:24-32 — the reference's CPU path: dequantize to fp16, fp32
 * matmul, fp32 bias, cast to fp16. Used as the timed CPU baseline (OpenMP over N; each
 * thread dequantizes one weight row into `wrow`, K floats of scratch). The fp32 sum runs in
 * K order. y fp16 [M, N]. */
void oracle_w4a16_cpu_f32(const uint16_t* x, int64_t M, int64_t K, const int32_t* qweight_t,
                          const uint16_t* scales, const int32_t* qzeros, const uint16_t* bias,
                          int64_t N, int64_t G, uint16_t* y, float* scratch, int64_t nthreads) {
#pragma omp parallel num_threads((int)nthreads)
  {
    float* wrow = scratch + (int64_t)omp_get_thread_num() * K;
#pragma omp for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      for (int64_t k = 0; k < K; ++k)
        wrow[k] = (float)tf_weight(qweight_t, scales, qzeros, N, K, G, n, k);
      for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * K;
        float acc = 0.0f;
        for (int64_t k = 0; k < K; ++k) acc += (float)h_from_bits(xr[k]) * wrow[k];
        if (bias) acc += (float)h_from_bits(bias[n]);
        y[m * N + n] = h_to_bits((f16)acc);
      }
    }
  }
}

/* Round an fp32 value to the nearest e4m3fn code, ties to even, saturating to +-448, NaN ->
 * 0x7F with the sign kept: the cast `.clamp(-448, 448).to(torch.float8_e4m3fn)` of
 * reference.py:49 and the explicit grid rounding of triton/rmsnorm_fp8.py:29-41.
 * e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; subnormal quantum 2^-9; no infinities. */
uint8_t oracle_e4m3(float v) {
  uint32_t bits;
  memcpy(&bits, &v, 4);
  const uint8_t sign = (uint8_t)((bits >> 24) & 0x80u);
  if (isnan(v)) return (uint8_t)(sign | 0x7Fu);
  float a = fabsf(v);
  if (a >= 448.0f) return (uint8_t)(sign | 0x7Eu);
  /* Scale so that one e4m3 quantum at |a|'s binade becomes 1, round to nearest even. */
  int e;
  frexpf(a, &e); /* a = f * 2^e, f in [0.5, 1) */
  int exp2 = e - 1; /* a in [2^exp2, 2^(exp2+1)) */
  if (exp2 < -6) exp2 = -6; /* subnormal range shares the 2^-6 binade's quantum */
  const float quantum = ldexpf(1.0f, exp2 - 3);
  const float r = nearbyintf(a / quantum) * quantum; /* default rounding mode: ties to even */
  if (r >= 448.0f) return (uint8_t)(sign | 0x7Eu);
  if (r == 0.0f) return sign;
  int re;
  frexpf(r, &re);
  int rexp = re - 1;
  if (rexp < -6) { /* subnormal: mantissa = r / 2^-9 */
    const int mant = (int)(r / ldexpf(1.0f, -9));
    return (uint8_t)(sign | mant);
  }
  const int biased = rexp + 7;
  const int mant = (int)(r / ldexpf(1.0f, rexp - 3)) - 8;
  return (uint8_t)(sign | (biased << 3) | mant);
}

/* Value of an e4m3fn code (the inverse of oracle_e4m3 on its range): 1 sign bit, 4 exponent
 * bits with bias 7, 3 mantissa bits; exponent 0 is subnormal (mantissa * 2^-9); code 0x7F /
 * 0xFF is NaN; there are no infinities. This is the format torch.float8_e4m3fn decodes. */
double oracle_e4m3_value(uint8_t c) {
  const int sign = c >> 7, e = (c >> 3) & 0xF, mant = c & 0x7;
  if (e == 0xF && mant == 0x7) return NAN;
  const double mag = e == 0 ? ldexp((double)mant, -9) : ldexp(1.0 + mant / 8.0, e - 7);
  return sign ? -mag : mag;
}

/* The FP8-activation linear (the consumer of rmsnorm_fp8_quant's (q, scale) that the reference
 * lacks): y[m, n] = sum_k e4m3(xq[m, k]) * x_scale[m * stride] * w[n, k] + bias[n] in fp64,
 * w the reference dequant (pack.py:189-194). xq [M, K] codes, row stride K. */
void oracle_w4a16_ref_fp8_f64(const uint8_t* xq, const float* x_scale, int64_t stride, int64_t M,
                              int64_t K, const int32_t* qweight_t, const uint16_t* scales,
                              const int32_t* qzeros, const uint16_t* bias, int64_t N, int64_t G,
                              double* out) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t m = 0; m < M; ++m) {
      const double s = (double)x_scale[m * stride];
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k)
        acc += oracle_e4m3_value(xq[m * K + k]) * s *
               (double)tf_weight(qweight_t, scales, qzeros, N, K, G, n, k);
      if (bias) acc += (double)h_from_bits(bias[n]);
      out[m * N + n] = acc;
    }
  }
}

/* RMSNorm + e4m3 quantization (reference.py:35-56 for the rule; triton/rmsnorm_fp8.py:57-73
 * for the exact fp32 operations: IEEE sqrt and divisions). The sum of squares is accumulated
 * in fp64 and rounded once to fp32, so it does not depend on the summation order.
 * scale_out[t] receives the dynamic per-token scale when static_scale is NULL. */
void oracle_rmsnorm_fp8(const uint16_t* x, int64_t T, int64_t H, const uint16_t* weight,
                        float eps, const float* static_scale, uint8_t* q, float* scale_out) {
  const float kMax = 448.0f, kMinScale = 1.0f / (448.0f * 512.0f);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    const uint16_t* xr = x + t * H;
    /* fp16 squares are exact in fp32; their fp64 sum rounded once to fp32 is the sum of
     * squares independent of summation order (the CUDA kernel accumulates the same way). */
    double ss = 0.0;
    for (int64_t i = 0; i < H; ++i) {
      const float f = (float)h_from_bits(xr[i]);
      ss += (double)(f * f);
    }
    const float var = (float)ss / (float)H;
    const float rstd = 1.0f / sqrtf(var + eps);
    float amax = 0.0f;
    for (int64_t i = 0; i < H; ++i) {
      const f16 y = (f16)((float)h_from_bits(xr[i]) * rstd) * h_from_bits(weight[i]);
      const float a = fabsf((float)y);
      if (a > amax) amax = a;
    }
    float scale;
    if (static_scale) {
      scale = *static_scale;
    } else {
      scale = amax / kMax;
      if (scale < kMinScale) scale = kMinScale;
      scale_out[t] = scale;
    }
    for (int64_t i = 0; i < H; ++i) {
      const f16 y = (f16)((float)h_from_bits(xr[i]) * rstd) * h_from_bits(weight[i]);
      float v = (float)y / scale;
      if (v > kMax) v = kMax;
      if (v < -kMax) v = -kMax;
      q[t * H + i] = oracle_e4m3(v);
    }
  }
}
