// Fused RMSNorm + FP8 e4m3 activation quantization, one pass over HBM.
//
// Per row (reference tokenforge/kernels/triton/rmsnorm_fp8.py:44-73; torch rule
// tokenforge/kernels/reference.py:35-56):
//   var   = fp32(sum(x^2)) / H                  (sum accumulated in fp64, then fp32)
//   rstd  = 1 / sqrt_rn(var + eps)              (IEEE sqrt, IEEE division)
//   y     = fp16(x * rstd) * weight             (round to fp16, then an fp16 product)
//   scale = max(amax|y| / 448, 1 / (448 * 512)) (dynamic, per token) or the static scale
//   q     = e4m3_rne(clamp(y / scale, -448, 448)) with the IEEE division's rounding
// The clamp and the cast are one hardware conversion: cvt.rn.satfinite.e4m3x2.f32 saturates
// finite and infinite values to +-448, keeps NaN, and rounds to nearest even including the
// subnormal range and the sign of zero (so -0.0 becomes code 0x80). The division is built from
// FMAs on the row's reciprocal (tf_rmsnorm.cuh, quant_pair_fma), bit-identical to IEEE division.
//
// Fast paths hold each row in registers as fp16 (x is read from HBM once, q written once):
//   H <= 1024: a warp per row (warp-shuffle reductions);
//   1024 < H <= 4096 and many rows: a persistent CTA per SM streams rows into per-warp
//     shared-memory rings with the bulk-copy engine while its warps compute (a warp per row);
//   otherwise up to H = 32768: a CTA per row (warp shuffles + a shared-memory step).
// Generic path (any H, any alignment): one CTA per row, three sweeps over the row (the second
// and third hit L2). With TF_LAUNCH_PDL the fast paths are launched as programmatic dependents
// and read x only after the preceding kernel on the stream has finished.
#include <algorithm>
#include <atomic>

#include "tf_async.cuh"
#include "tf_common.cuh"
#include "tf_plan.h"
#include "tf_rmsnorm.cuh"

namespace tfb {

// Status word of the streaming kernel's bounded waits (0 = none), read by tf_device_error.
__device__ int g_rms_error = 0;

namespace {

constexpr int kErrRowWait = 0x301;  // a row's bulk copy did not complete in time
constexpr unsigned long long kRowWaitLimitNs = 2000000000ull;

// A warp per row (four rows per CTA), rows of H <= 1024 elements (VPL = 4 16-byte vectors per
// lane), H % 8 == 0, aligned.
template <int VPL>
__global__ void __launch_bounds__(128) rmsnorm_fp8_warp_kernel(
    const uint4* __restrict__ x, int64_t T, int64_t H, int64_t ldx_vec,
    const uint4* __restrict__ weight, float eps, const float* __restrict__ static_scale,
    uint2* __restrict__ q, float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nvec = H / 8;
  uint4 v[VPL], g[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    g[i] = lane + 32 * i < nvec ? neg_weight(__ldg(weight + lane + 32 * i)) : make_uint4(0, 0, 0, 0);
  // x (and the outputs) may belong to the preceding kernel on the stream.
  pdl_wait();
  if (row >= T) return;
  const uint4* xr = x + row * ldx_vec;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int64_t j = lane + 32 * i;
    v[i] = j < nvec ? ldg_stream_v4(xr + j) : make_uint4(0, 0, 0, 0);
  }
  double sumsq = 0.0;
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc_sumsq(v[i], sumsq);
  const float rstd = rstd_of(warp_sum(sumsq), H, eps);
  const uint64_t rstd2 = f32x2(rstd, rstd);
  __half2 amax2 = __float2half2_rn(0.f);
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if (lane + 32 * i < nvec) v[i] = norm_vec_neg(v[i], g[i], rstd2, amax2);
  float scale;
  if (static_scale != nullptr) {
    scale = __ldg(static_scale);
  } else {
    scale = dyn_scale(warp_max(amax_of(amax2)));
    if (lane == 0) scale_out[row] = scale;
  }
  const Fp8Div d = fp8_div(scale);
  const int path = quant_path(d, amax_finite(amax2), static_scale == nullptr);
  pdl_launch_dependents();  // the next kernel may start its prologue (it waits for this grid)
  quant_row(v, nvec, [&](int i) { return static_cast<int64_t>(lane + 32 * i); }, d, path,
            q + row * nvec);
}

// Streaming form for many rows of 1024 to 4096 elements (H % 8 == 0, aligned): a persistent CTA
// per SM whose warps each own a shared-memory row buffer (kRowStages deep). A warp reads its row
// into registers, then has the bulk-copy engine (cp.async.bulk, completion on an mbarrier) bring
// its next row into the buffer while it computes the current one. One stage (one row of
// lookahead) leaves room for 16 warps per SM, which measured faster than two stages at 15. The weight is read once per CTA into shared
// memory (negated). Rows go to warps round-robin (warp w of the grid takes rows w, w + W, ...).
struct RmsStream {
  const uint8_t* x;
  int64_t T, H, ldx_bytes;
  const uint4* weight;
  float eps;
  const float* static_scale;
  uint2* q;
  float* scale_out;
  uint32_t row_bytes, stage_bytes, w_bytes;
};

constexpr int kRowStages = 1;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Warp-uniform bounded wait on a ring stage: every lane polls the mbarrier (so each observes the
// completed copy) and the warp leaves together; false after kRowWaitLimitNs (recording the
// error) or, with stop_on_error, once another warp has recorded one.
__device__ __forceinline__ bool warp_wait_row(uint64_t* bar, uint32_t parity,
                                              bool stop_on_error = true) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    int quit = 0;
    if ((threadIdx.x & 31) == 0)
      quit = (stop_on_error && *reinterpret_cast<volatile int*>(&g_rms_error) != 0) ||
             global_ns() - t0 > kRowWaitLimitNs;
    if (__shfl_sync(0xffffffffu, quit, 0)) {
      if ((threadIdx.x & 31) == 0) atomicCAS(&g_rms_error, 0, kErrRowWait);
      return false;
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(512, 1) rmsnorm_fp8_stream_kernel(const RmsStream p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = static_cast<int>(blockDim.x) >> 5;
  const int64_t nvec = p.H / 8;
  uint4* wsm = reinterpret_cast<uint4*>(smem);
  uint8_t* ring = smem + p.w_bytes + static_cast<size_t>(warp) * kRowStages * p.stage_bytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + p.w_bytes + static_cast<size_t>(nw) *
                                              kRowStages * p.stage_bytes) + 2 * warp;
  for (int64_t j = threadIdx.x; j < nvec; j += blockDim.x) wsm[j] = neg_weight(__ldg(p.weight + j));
  if (lane == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // x (and the outputs) may belong to the preceding kernel on the stream.
  pdl_wait();
  const int64_t G = static_cast<int64_t>(gridDim.x) * nw;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * nw + warp;
  if (lane == 0) {
    for (int s = 0; s < kRowStages; ++s) {
      const int64_t r = first + s * G;
      if (r < p.T) {
        mbar_expect_tx(bar + s, p.row_bytes);
        bulk_load(ring + s * p.stage_bytes, p.x + r * p.ldx_bytes, p.row_bytes, bar + s);
      }
    }
  }
  uint32_t it = 0;
  for (int64_t row = first; row < p.T; row += G, ++it) {
    const int s = static_cast<int>(it % kRowStages);
    if (!warp_wait_row(bar + s, (it / kRowStages) & 1)) {
      // Give up on this warp's rows; wait (bounded) for its other copies in flight first.
      for (int o = 1; o < kRowStages; ++o)
        if (row + o * G < p.T)
          warp_wait_row(bar + (it + o) % kRowStages, ((it + o) / kRowStages) & 1, false);
      break;
    }
    const uint4* buf = reinterpret_cast<const uint4*>(ring + s * p.stage_bytes);
    uint4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int64_t j = lane + 32 * i;
      v[i] = j < nvec ? buf[j] : make_uint4(0, 0, 0, 0);
    }
    __syncwarp();
    if (lane == 0 && row + kRowStages * G < p.T) {  // refill: the warp's row kRowStages ahead
      mbar_expect_tx(bar + s, p.row_bytes);
      bulk_load(ring + s * p.stage_bytes, p.x + (row + kRowStages * G) * p.ldx_bytes, p.row_bytes,
                bar + s);
    }
    double sumsq = 0.0;
#pragma unroll
    for (int i = 0; i < VPL; ++i) acc_sumsq(v[i], sumsq);
    const float rstd = rstd_of(warp_sum(sumsq), p.H, p.eps);
    const uint64_t rstd2 = f32x2(rstd, rstd);
    __half2 amax2 = __float2half2_rn(0.f);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int64_t j = lane + 32 * i;
      if (j < nvec) v[i] = norm_vec_neg(v[i], wsm[j], rstd2, amax2);
    }
    float scale;
    if (p.static_scale != nullptr) {
      scale = __ldg(p.static_scale);
    } else {
      scale = dyn_scale(warp_max(amax_of(amax2)));
      if (lane == 0) p.scale_out[row] = scale;
    }
    const Fp8Div d = fp8_div(scale);
    const int path = quant_path(d, amax_finite(amax2), p.static_scale == nullptr);
    quant_row(v, nvec, [&](int i) { return static_cast<int64_t>(lane + 32 * i); }, d, path,
              p.q + row * nvec);
  }
  pdl_launch_dependents();
}

// One CTA per row (rows of H <= blockDim.x * VPT * 8 elements, H % 8 == 0, aligned): each
// thread holds VPT 16-byte vectors of the row and of the (negated) weight in registers, so x is
// read once and q written once; a row costs two block-wide reductions (one barrier each).
template <int VPT>
__global__ void __launch_bounds__(1024) rmsnorm_fp8_row_kernel(
    const uint4* __restrict__ x, int64_t T, int64_t H, int64_t ldx_vec,
    const uint4* __restrict__ weight, float eps, const float* __restrict__ static_scale,
    uint2* __restrict__ q, float* __restrict__ scale_out) {
  __shared__ double sh_sum[32];
  __shared__ float sh_max[32];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nt = static_cast<int>(blockDim.x), nw = nt >> 5;
  const int64_t nvec = H / 8;
  const uint4* xr = x + row * ldx_vec;
  uint4 v[VPT], g[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t j = tid + static_cast<int64_t>(nt) * i;
    g[i] = j < nvec ? neg_weight(__ldg(weight + j)) : make_uint4(0, 0, 0, 0);
  }
  // x (and the outputs) may belong to the preceding kernel on the stream.
  pdl_wait();
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t j = tid + static_cast<int64_t>(nt) * i;
    v[i] = j < nvec ? ldg_stream_v4(xr + j) : make_uint4(0, 0, 0, 0);
  }
  double sumsq = 0.0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) acc_sumsq(v[i], sumsq);
  sumsq = warp_sum(sumsq);
  if (lane == 0) sh_sum[warp] = sumsq;
  __syncthreads();
  double total = 0.0;
  for (int w = 0; w < nw; ++w) total += sh_sum[w];
  const float rstd = rstd_of(total, H, eps);
  const uint64_t rstd2 = f32x2(rstd, rstd);

  __half2 amax2 = __float2half2_rn(0.f);
#pragma unroll
  for (int i = 0; i < VPT; ++i)
    if (tid + static_cast<int64_t>(nt) * i < nvec) v[i] = norm_vec_neg(v[i], g[i], rstd2, amax2);
  float scale;
  if (static_scale != nullptr) {
    scale = __ldg(static_scale);
  } else {
    const float m = warp_max(amax_of(amax2));
    if (lane == 0) sh_max[warp] = m;
    __syncthreads();
    float mx = 0.f;
    for (int w = 0; w < nw; ++w) mx = fmaxf(mx, sh_max[w]);
    scale = dyn_scale(mx);
    if (tid == 0) scale_out[row] = scale;
  }
  const Fp8Div d = fp8_div(scale);
  const int path = quant_path(d, amax_finite(amax2), static_scale == nullptr);
  pdl_launch_dependents();  // the next kernel may start its prologue (it waits for this grid)
  quant_row(v, nvec, [&](int i) { return tid + static_cast<int64_t>(nt) * i; }, d, path,
            q + row * nvec);
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

// q = e4m3(clamp(y / scale)) for rows of fp16 values already normalised, by a given scale; one
// thread per 8 values (kVec) or per value.
template <bool kVec>
__global__ void e4m3_quant_rows_kernel(const __half* __restrict__ y, int64_t R, int64_t C,
                                       int64_t ldy, const float* __restrict__ scale,
                                       int64_t stride, uint8_t* __restrict__ q) {
  const int64_t per_row = kVec ? C / 8 : C;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= R * per_row) return;
  const int64_t r = i / per_row, c = i - r * per_row;
  const Fp8Div d = fp8_div(__ldg(scale + r * stride));
  if constexpr (kVec) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(y + r * ldy) + c);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    __half2 amax2 = __float2half2_rn(0.f);
#pragma unroll
    for (int e = 0; e < 4; ++e) amax2 = __hmax2(amax2, __habs2(h[e]));
    v = neg_weight(v);
    uint2* out = reinterpret_cast<uint2*>(q + r * C) + c;
    if (d.fma_ok && amax_finite(amax2)) *out = quant_vec<kFma2>(v, d);
    else *out = quant_vec<kIeee>(v, d);
  } else {
    const __half ny = __hneg(y[r * ldy + c]);
    const __half2 pair = __halves2half2(ny, __float2half_rn(0.f));
    const bool finite = (__half_as_ushort(ny) & 0x7FFFu) < 0x7C00u;
    const uint16_t code = d.fma_ok && finite ? quant_pair<kFma2>(pair, d) : quant_pair<kIeee>(pair, d);
    q[r * C + c] = static_cast<uint8_t>(code & 0xFFu);
  }
}

// Dynamic per-row scales (scale = max(amax|y| / 448, 1 / (448 * 512)), the rule of the dynamic
// RMSNorm quantizer): one CTA per row, the row's amax, then its codes on one division path.
template <int kPath, bool kVec>
__device__ __forceinline__ void quant_row_dyn(const __half* yr, int64_t C, const Fp8Div& d,
                                              uint8_t* qr) {
  if constexpr (kVec) {
    for (int64_t j = threadIdx.x; j < C / 8; j += blockDim.x)
      reinterpret_cast<uint2*>(qr)[j] =
          quant_vec<kPath>(neg_weight(__ldg(reinterpret_cast<const uint4*>(yr) + j)), d);
  } else {
    for (int64_t j = threadIdx.x; j < C; j += blockDim.x) {
      const __half2 pair = __halves2half2(__hneg(yr[j]), __float2half_rn(0.f));
      qr[j] = static_cast<uint8_t>(quant_pair<kPath>(pair, d) & 0xFFu);
    }
  }
}

template <bool kVec>
__global__ void __launch_bounds__(256) e4m3_quant_rows_dyn_kernel(
    const __half* __restrict__ y, int64_t C, int64_t ldy, uint8_t* __restrict__ q,
    float* __restrict__ scale_out) {
  __shared__ float sh[32];
  const int64_t r = blockIdx.x;
  const __half* yr = y + r * ldy;
  float amax = 0.f;
  if constexpr (kVec) {
    __half2 a2 = __float2half2_rn(0.f);
    for (int64_t j = threadIdx.x; j < C / 8; j += blockDim.x) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(yr) + j);
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) a2 = __hmax2(a2, __habs2(h[e]));
    }
    amax = amax_of(a2);
  } else {
    for (int64_t j = threadIdx.x; j < C; j += blockDim.x)
      amax = fmaxf(amax, fabsf(__half2float(yr[j])));
  }
  amax = block_max(amax, sh);
  const float scale = dyn_scale(amax);
  if (threadIdx.x == 0) scale_out[r] = scale;
  const Fp8Div d = fp8_div(scale);
  uint8_t* qr = q + r * C;
  if (quant_path(d, amax <= 65504.f, true) == kFma1) quant_row_dyn<kFma1, kVec>(yr, C, d, qr);
  else quant_row_dyn<kIeee, kVec>(yr, C, d, qr);
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


// Vectors per thread of the CTA-per-row kernel for rows of nvec 16-byte vectors (0: the row
// does not fit, 1024 threads x 4 vectors): few rows keep one vector per thread (the shortest
// dependent chain per row); more rows hold two or four, so fewer threads share each row's
// reductions.
int rows_vpt(int64_t nvec, int64_t T) {
  for (int vpt : {T <= 128 ? 1 : 2, 2, 4})
    if (cdiv(nvec, vpt) <= 1024) return vpt;
  return 0;
}

// Vectors per lane of the streaming kernel (0: not used): rows of 1024 to 4096 elements, once
// there are enough of them to give every warp of the persistent grid a row (fewer rows are
// faster spread over a CTA each).
int stream_vpl(int64_t nvec, int64_t T) {
  if (nvec <= 128 || nvec > 512 || T < 4 * 148) return 0;
  for (int vpl : {8, 12, 14, 16})
    if (nvec <= 32 * vpl) return vpl;
  return 0;
}

int device_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// One launch of a row kernel, with the programmatic-dependent-launch attribute when enabled
// (the kernel waits on griddepcontrol before it reads x).
template <typename... KArgs, typename... Args>
int launch_rows(void (*kern)(KArgs...), unsigned grid, unsigned threads, cudaStream_t stream,
                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (launch_flags() & TF_LAUNCH_PDL) ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return check_launch();
}

// The streaming kernel: as many warps per CTA (<= 16) as kRowStages row buffers per warp allow
// beside the weight in 227 KB of shared memory; one CTA per SM.
template <int VPL>
int launch_stream(const RmsStream& p0, cudaStream_t stream) {
  constexpr int kSmemLimit = 227 * 1024;
  RmsStream p = p0;
  const int64_t nvec = p.H / 8;
  p.row_bytes = static_cast<uint32_t>(nvec * 16);
  p.stage_bytes = static_cast<uint32_t>(cdiv(p.row_bytes, 128) * 128);
  p.w_bytes = p.stage_bytes;
  const int nw = static_cast<int>(std::min<int64_t>(
      16, (kSmemLimit - p.w_bytes - 16 * 16) / (kRowStages * static_cast<int64_t>(p.stage_bytes))));
  const size_t smem = p.w_bytes + static_cast<size_t>(nw) * (kRowStages * p.stage_bytes + 16);
  static std::atomic<uint64_t> attr_set{0};  // devices whose shared-memory limit is raised
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(attr_set.load() >> dev & 1)) {
    const cudaError_t e = cudaFuncSetAttribute(rmsnorm_fp8_stream_kernel<VPL>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSmemLimit);
    if (e != cudaSuccess) {
      last_cuda_error() = static_cast<int>(e);
      return TF_ERR_CUDA;
    }
    if (dev < 64) attr_set.fetch_or(uint64_t{1} << dev);
  }
  const int64_t grid = std::min<int64_t>(device_sms(), cdiv(p.T, nw));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(32 * nw));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (launch_flags() & TF_LAUNCH_PDL) ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, rmsnorm_fp8_stream_kernel<VPL>, p);
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return check_launch();
}

}  // namespace

int rms_device_error(int* code) {
  const cudaError_t e = cudaMemcpyFromSymbol(code, g_rms_error, sizeof(int));
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

int rms_reset_device_error() {
  const int zero = 0;
  const cudaError_t e = cudaMemcpyToSymbol(g_rms_error, &zero, sizeof(int));
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

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
  auto xv = reinterpret_cast<const uint4*>(x);
  auto wv = reinterpret_cast<const uint4*>(weight);
  auto qv = reinterpret_cast<uint2*>(q);
  const int vpt = rows_vpt(nvec, T);
  const int vpl = stream_vpl(nvec, T);
  const int64_t ldv = ldx / 8;
  if (vec_ok && nvec <= 128 && T <= 0x7fffffffLL) {
    return launch_rows(rmsnorm_fp8_warp_kernel<4>, static_cast<unsigned>(cdiv(T, 4)), 128, stream,
                       xv, T, H, ldv, wv, eps, static_scale, qv, scale_out);
  } else if (vec_ok && vpl > 0) {
    const RmsStream p{reinterpret_cast<const uint8_t*>(x), T, H, ldx * 2, wv, eps, static_scale,
                      qv, scale_out, 0, 0, 0};
    switch (vpl) {
      case 8: return launch_stream<8>(p, stream);
      case 12: return launch_stream<12>(p, stream);
      case 14: return launch_stream<14>(p, stream);
      default: return launch_stream<16>(p, stream);
    }
  } else if (vec_ok && vpt > 0 && T <= 0x7fffffffLL) {
    const unsigned nt = static_cast<unsigned>(cdiv(cdiv(nvec, vpt), 32) * 32);
    const unsigned grid = static_cast<unsigned>(T);
    switch (vpt) {
      case 1: return launch_rows(rmsnorm_fp8_row_kernel<1>, grid, nt, stream, xv, T, H, ldv, wv, eps, static_scale, qv, scale_out);
      case 2: return launch_rows(rmsnorm_fp8_row_kernel<2>, grid, nt, stream, xv, T, H, ldv, wv, eps, static_scale, qv, scale_out);
      default: return launch_rows(rmsnorm_fp8_row_kernel<4>, grid, nt, stream, xv, T, H, ldv, wv, eps, static_scale, qv, scale_out);
    }
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

extern "C" int tf_e4m3_quant_rows(const uint16_t* y, int64_t R, int64_t C, int64_t ldy,
                                  const float* scale, int64_t scale_stride, uint8_t* q,
                                  float* scale_out, void* stream_) {
  using namespace tfb;
  if (R < 0 || C < 1 || ldy < C || (scale_stride != 0 && scale_stride != 1))
    return TF_ERR_INVALID_ARG;
  if (R == 0) return TF_OK;
  if (!y || !q || (!scale && !scale_out)) return TF_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  auto yh = reinterpret_cast<const __half*>(y);
  const bool vec = C % 8 == 0 && ldy % 8 == 0 && aligned16(y) &&
                   reinterpret_cast<uintptr_t>(q) % 8 == 0;
  if (!scale) {
    if (R > 0x7fffffffLL) return TF_ERR_UNSUPPORTED;
    if (vec)
      e4m3_quant_rows_dyn_kernel<true><<<static_cast<unsigned>(R), 256, 0, stream>>>(
          yh, C, ldy, q, scale_out);
    else
      e4m3_quant_rows_dyn_kernel<false><<<static_cast<unsigned>(R), 256, 0, stream>>>(
          yh, C, ldy, q, scale_out);
  } else if (vec) {
    const int64_t n = R * (C / 8);
    e4m3_quant_rows_kernel<true><<<static_cast<unsigned>(cdiv(n, 256)), 256, 0, stream>>>(
        yh, R, C, ldy, scale, scale_stride, q);
  } else {
    const int64_t n = R * C;
    e4m3_quant_rows_kernel<false><<<static_cast<unsigned>(cdiv(n, 256)), 256, 0, stream>>>(
        yh, R, C, ldy, scale, scale_stride, q);
  }
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
