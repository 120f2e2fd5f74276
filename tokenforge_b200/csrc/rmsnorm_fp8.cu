// Fused RMSNorm + FP8 e4m3 activation quantization, one pass over HBM.
//
// Per row (reference tokenforge/kernels/triton/rmsnorm_fp8.py:44-73; torch rule
// tokenforge/kernels/reference.py:35-56):
//   var   = fp32(sum(x^2)) / H                  (sum accumulated in fp64, then fp32)
//   rstd  = 1 / sqrt_rn(var + eps)              (IEEE sqrt, IEEE division)
//   y     = fp16(x * rstd) * weight             (round to fp16, then an fp16 product)
//   scale = max(amax|y| / 448, 1 / (448 * 512)) (dynamic, per token) or the static scale
//   q     = e4m3_rne(clamp(y / scale, -448, 448)) with an IEEE division
// The clamp and the cast are one hardware conversion: cvt.rn.satfinite.e4m3x2.f32 saturates
// finite and infinite values to +-448, keeps NaN, and rounds to nearest even including the
// subnormal range and the sign of zero (so -0.0 becomes code 0x80).
//
// Fast paths hold the row in registers as fp16 (x is read from HBM once, q written once): one
// warp per row for H <= 1024 (warp-shuffle reductions), one CTA per row up to H = 8192 (warp
// shuffles + a shared-memory step). Generic path (any H, any alignment): one CTA per row, three
// sweeps over the row (the second and third hit L2).
#include "tf_common.cuh"
#include "tf_plan.h"
#include "tf_rmsnorm.cuh"

namespace tfb {
namespace {


// VPL = 16-byte vectors per lane; rows of H <= 256 * VPL elements, H % 8 == 0, aligned.
template <int VPL>
__global__ void __launch_bounds__(128) rmsnorm_fp8_warp_kernel(
    const uint4* __restrict__ x, int64_t T, int64_t H, int64_t ldx_vec,
    const uint4* __restrict__ weight, float eps, const float* __restrict__ static_scale,
    uint2* __restrict__ q, float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= T) return;
  const int64_t nvec = H / 8;
  const uint4* xr = x + row * ldx_vec;

  uint4 v[VPL];
  double sumsq = 0.0;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int64_t j = lane + 32 * i;
    v[i] = (j < nvec) ? ldg_stream_v4(xr + j) : make_uint4(0, 0, 0, 0);
    const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      sumsq += static_cast<double>(__fmul_rn(f.x, f.x)) + static_cast<double>(__fmul_rn(f.y, f.y));
    }
  }
  const float rstd = rstd_of(warp_sum(sumsq), H, eps);

  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int64_t j = lane + 32 * i;
    if (j >= nvec) continue;
    const uint4 wv = __ldg(weight + j);
    __half2* h = reinterpret_cast<__half2*>(&v[i]);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      const __half2 n2 = __halves2half2(__float2half_rn(__fmul_rn(f.x, rstd)),
                                        __float2half_rn(__fmul_rn(f.y, rstd)));
      h[e] = __hmul2(n2, w2[e]);
      const float2 y = __half22float2(h[e]);
      amax = fmaxf(amax, fmaxf(fabsf(y.x), fabsf(y.y)));
    }
  }
  float scale;
  if (static_scale != nullptr) {
    scale = __ldg(static_scale);
  } else {
    scale = dyn_scale(warp_max(amax));
    if (lane == 0) scale_out[row] = scale;
  }
  uint2* qr = q + row * nvec;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int64_t j = lane + 32 * i;
    if (j >= nvec) continue;
    const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
    uint32_t packed[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float2 a = __half22float2(h[2 * e]);
      const float2 b = __half22float2(h[2 * e + 1]);
      const uint32_t lo = cvt_e4m3x2(__fdiv_rn(a.x, scale), __fdiv_rn(a.y, scale));
      const uint32_t hi = cvt_e4m3x2(__fdiv_rn(b.x, scale), __fdiv_rn(b.y, scale));
      packed[e] = lo | (hi << 16);
    }
    qr[j] = make_uint2(packed[0], packed[1]);
  }
}

// One CTA of NT threads per row (rows of H <= NT * VPT * 8, H % 8 == 0, aligned): each thread
// holds VPT 16-byte vectors of the row in registers, so x is read once and q written once,
// and a row's latency is that of two block reductions instead of a whole row per warp.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_fp8_cta_kernel(
    const uint4* __restrict__ x, int64_t T, int64_t H, int64_t ldx_vec,
    const uint4* __restrict__ weight, float eps, const float* __restrict__ static_scale,
    uint2* __restrict__ q, float* __restrict__ scale_out) {
  __shared__ double sh_sum[NT / 32];
  __shared__ float sh_max[NT / 32];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nvec = H / 8;
  const uint4* xr = x + row * ldx_vec;
  uint4 v[VPT];
  double sumsq = 0.0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t j = tid + static_cast<int64_t>(NT) * i;
    v[i] = (j < nvec) ? ldg_stream_v4(xr + j) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      sumsq += static_cast<double>(__fmul_rn(f.x, f.x)) + static_cast<double>(__fmul_rn(f.y, f.y));
    }
  }
  sumsq = warp_sum(sumsq);
  if (lane == 0) sh_sum[warp] = sumsq;
  __syncthreads();
  double total = 0.0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) total += sh_sum[w];
  const float rstd = rstd_of(total, H, eps);

  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t j = tid + static_cast<int64_t>(NT) * i;
    if (j >= nvec) continue;
    const uint4 wv = __ldg(weight + j);
    __half2* h = reinterpret_cast<__half2*>(&v[i]);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      const __half2 n2 = __halves2half2(__float2half_rn(__fmul_rn(f.x, rstd)),
                                        __float2half_rn(__fmul_rn(f.y, rstd)));
      h[e] = __hmul2(n2, w2[e]);
      const float2 y = __half22float2(h[e]);
      amax = fmaxf(amax, fmaxf(fabsf(y.x), fabsf(y.y)));
    }
  }
  float scale;
  if (static_scale != nullptr) {
    scale = __ldg(static_scale);
  } else {
    amax = warp_max(amax);
    if (lane == 0) sh_max[warp] = amax;
    __syncthreads();
    float m = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) m = fmaxf(m, sh_max[w]);
    scale = dyn_scale(m);
    if (tid == 0) scale_out[row] = scale;
  }
  uint2* qr = q + row * nvec;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t j = tid + static_cast<int64_t>(NT) * i;
    if (j >= nvec) continue;
    const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
    uint32_t packed[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float2 a = __half22float2(h[2 * e]);
      const float2 b = __half22float2(h[2 * e + 1]);
      const uint32_t lo = cvt_e4m3x2(__fdiv_rn(a.x, scale), __fdiv_rn(a.y, scale));
      const uint32_t hi = cvt_e4m3x2(__fdiv_rn(b.x, scale), __fdiv_rn(b.y, scale));
      packed[e] = lo | (hi << 16);
    }
    qr[j] = make_uint2(packed[0], packed[1]);
  }
}

__device__ __forceinline__ float block_max(float v, float* sh) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) r = fmaxf(r, sh[w]);
  return r;
}

__device__ __forceinline__ double block_sum(double v, double* sh) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double r = 0.0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) r += sh[w];
  return r;
}

__device__ __forceinline__ __half norm_elem(const __half* xr, const __half* w, int64_t i,
                                            float rstd) {
  const float f = __half2float(xr[i]);
  return __hmul(__float2half_rn(__fmul_rn(f, rstd)), w[i]);
}

__global__ void __launch_bounds__(256) rmsnorm_fp8_generic_kernel(
    const __half* __restrict__ x, int64_t T, int64_t H, int64_t ldx,
    const __half* __restrict__ weight, float eps, const float* __restrict__ static_scale,
    uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  __shared__ float sh[32];
  __shared__ double shd[32];
  const int64_t row = blockIdx.x;
  const __half* xr = x + row * ldx;
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
    const float f = __half2float(xr[i]);
    s += static_cast<double>(__fmul_rn(f, f));
  }
  const float rstd = rstd_of(block_sum(s, shd), H, eps);
  float scale;
  if (static_scale != nullptr) {
    scale = *static_scale;
  } else {
    float amax = 0.f;
    for (int64_t i = threadIdx.x; i < H; i += blockDim.x)
      amax = fmaxf(amax, fabsf(__half2float(norm_elem(xr, weight, i, rstd))));
    scale = dyn_scale(block_max(amax, sh));
    if (threadIdx.x == 0) scale_out[row] = scale;
  }
  for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
    const float y = __half2float(norm_elem(xr, weight, i, rstd));
    q[row * H + i] = static_cast<uint8_t>(cvt_e4m3x2(__fdiv_rn(y, scale), 0.f) & 0xFFu);
  }
}

__global__ void cast_e4m3_kernel(const float* __restrict__ in, int64_t n, uint8_t* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = static_cast<uint8_t>(cvt_e4m3x2(in[i], 0.f) & 0xFFu);
}

// x16[m, k] = fp16(e4m3(q[m, k]) * scale[m * stride]): the e4m3 value is exact in fp32, the
// product is rounded once to fp16. One thread per 8 codes.
__global__ void fp8_to_fp16_kernel(const uint8_t* __restrict__ q, int64_t M, int64_t K,
                                   int64_t ldq, const float* __restrict__ scale, int64_t stride,
                                   __half* __restrict__ x16, int64_t ldx16) {
  const int64_t per_row = (K + 7) / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M * per_row) return;
  const int64_t m = i / per_row, k0 = (i - m * per_row) * 8;
  const float s = scale[m * stride];
  const uint8_t* src = q + m * ldq + k0;
  __half* dst = x16 + m * ldx16 + k0;
  for (int e = 0; e < 8 && k0 + e < K; e += 2) {
    const uint16_t pair = (k0 + e + 1 < K) ? static_cast<uint16_t>(src[e] | (src[e + 1] << 8))
                                           : static_cast<uint16_t>(src[e]);
    uint32_t h;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(pair));
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
    dst[e] = __float2half_rn(__fmul_rn(f.x, s));
    if (k0 + e + 1 < K) dst[e + 1] = __float2half_rn(__fmul_rn(f.y, s));
  }
}

// out[m, i] = fp16(silu(g) * u) with g = gu[m, i], u = gu[m, I + i] (the fused gate_up
// projection's two halves), silu(g) = g / (1 + e^-g) in fp32. Eight outputs per thread.
__global__ void silu_mul_kernel(const __half* __restrict__ gu, int64_t M, int64_t I, int64_t ld,
                                __half* __restrict__ out, int64_t ldo) {
  const int64_t per_row = (I + 7) / 8;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= M * per_row) return;
  const int64_t m = t / per_row, i0 = (t - m * per_row) * 8;
  const __half* g = gu + m * ld + i0;
  const __half* u = g + I;
  __half* o = out + m * ldo + i0;
  const bool vec = i0 + 8 <= I && ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u) |
                                     reinterpret_cast<uintptr_t>(o)) & 15u) == 0;
  if (vec) {
    const uint4 gv = *reinterpret_cast<const uint4*>(g), uv = *reinterpret_cast<const uint4*>(u);
    const __half2* g2 = reinterpret_cast<const __half2*>(&gv);
    const __half2* u2 = reinterpret_cast<const __half2*>(&uv);
    uint4 ov;
    __half2* o2 = reinterpret_cast<__half2*>(&ov);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 gf = __half22float2(g2[e]), uf = __half22float2(u2[e]);
      o2[e] = __floats2half2_rn(silu_mul_f32(gf.x, uf.x), silu_mul_f32(gf.y, uf.y));
    }
    *reinterpret_cast<uint4*>(o) = ov;
  } else {
    for (int e = 0; e < 8 && i0 + e < I; ++e) {
      const float gf = __half2float(g[e]), uf = __half2float(u[e]);
      o[e] = __float2half_rn(silu_mul_f32(gf, uf));
    }
  }
}

}  // namespace

int launch_fp8_to_fp16(const uint8_t* xq, int64_t M, int64_t K, int64_t ldq, const float* scale,
                       int64_t stride, uint16_t* x16, int64_t ldx16, cudaStream_t stream) {
  const int64_t n = M * ((K + 7) / 8);
  if (n == 0) return TF_OK;
  fp8_to_fp16_kernel<<<static_cast<unsigned>(cdiv(n, 256)), 256, 0, stream>>>(
      xq, M, K, ldq, scale, stride, reinterpret_cast<__half*>(x16), ldx16);
  return check_launch();
}

}  // namespace tfb

extern "C" int tf_rmsnorm_fp8_quant(const uint16_t* x, int64_t T, int64_t H, int64_t ldx,
                                    const uint16_t* weight, float eps, const float* static_scale,
                                    uint8_t* q, float* scale_out, void* stream_) {
  using namespace tfb;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (T < 0 || H <= 0 || ldx < H) return TF_ERR_INVALID_ARG;
  if (T == 0) return TF_OK;
  if (!x || !weight || !q || (!static_scale && !scale_out)) return TF_ERR_INVALID_ARG;
  const bool vec_ok = (H % 8 == 0) && (ldx % 8 == 0) && aligned16(x) && aligned16(weight) &&
                      (reinterpret_cast<uintptr_t>(q) % 8 == 0);
  const int64_t nvec = H / 8;
  const int rows_per_cta = 4;
  const unsigned grid = static_cast<unsigned>(cdiv(T, rows_per_cta));
  auto xv = reinterpret_cast<const uint4*>(x);
  auto wv = reinterpret_cast<const uint4*>(weight);
  auto qv = reinterpret_cast<uint2*>(q);
  // Rows up to 1024 elements: a warp per row (four rows per CTA). Longer rows: a CTA per row
  // (128 threads up to 4096 elements, 256 up to 8192), so that each row is short work.
  if (vec_ok && nvec <= 32 * 4) {
    rmsnorm_fp8_warp_kernel<4><<<grid, 128, 0, stream>>>(xv, T, H, ldx / 8, wv, eps, static_scale, qv, scale_out);
  } else if (vec_ok && nvec <= 128 * 4 && T <= 0x7fffffffLL) {
    rmsnorm_fp8_cta_kernel<128, 4><<<static_cast<unsigned>(T), 128, 0, stream>>>(
        xv, T, H, ldx / 8, wv, eps, static_scale, qv, scale_out);
  } else if (vec_ok && nvec <= 256 * 4 && T <= 0x7fffffffLL) {
    rmsnorm_fp8_cta_kernel<256, 4><<<static_cast<unsigned>(T), 256, 0, stream>>>(
        xv, T, H, ldx / 8, wv, eps, static_scale, qv, scale_out);
  } else {
    if (T > 0x7fffffffLL) return TF_ERR_UNSUPPORTED;
    rmsnorm_fp8_generic_kernel<<<static_cast<unsigned>(T), 256, 0, stream>>>(
        reinterpret_cast<const __half*>(x), T, H, ldx, reinterpret_cast<const __half*>(weight),
        eps, static_scale, q, scale_out);
  }
  return check_launch();
}

extern "C" int tf_cast_e4m3(const float* in, int64_t n, uint8_t* out, void* stream) {
  using namespace tfb;
  if (n < 0) return TF_ERR_INVALID_ARG;
  if (n == 0) return TF_OK;
  if (!in || !out) return TF_ERR_INVALID_ARG;
  cast_e4m3_kernel<<<static_cast<unsigned>(cdiv(n, 256)), 256, 0,
                     static_cast<cudaStream_t>(stream)>>>(in, n, out);
  return check_launch();
}

extern "C" int tf_silu_mul(const uint16_t* gate_up, int64_t M, int64_t I, int64_t ld, uint16_t* out,
                           int64_t ldo, void* stream) {
  using namespace tfb;
  if (M < 0 || I < 1 || ld < 2 * I || ldo < I) return TF_ERR_INVALID_ARG;
  if (M == 0) return TF_OK;
  if (!gate_up || !out) return TF_ERR_INVALID_ARG;
  const int64_t n = M * ((I + 7) / 8);
  silu_mul_kernel<<<static_cast<unsigned>(cdiv(n, 256)), 256, 0,
                    static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __half*>(gate_up), M, I, ld, reinterpret_cast<__half*>(out), ldo);
  return check_launch();
}
