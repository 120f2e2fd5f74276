// W4A16 linear on the warp-level tensor-core path: decode GEMV (M <= 8) and a 64-token tiled
// variant. y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]) with w = fp16(q - z) * s.
//
// Reference semantics: triton/w4a16.py:44-115 (in-register dequant with one fp16 rounding,
// fp32 accumulation, fp16 output, bias added in fp32 before the cast) and the split-K contract
// of w4a16.py:193-200,227-232 (fp32 partials summed in a fixed order, then bias, then cast).
//
// Why tensor cores for a GEMV: at M = 1 the kernel must turn ~13e12 int4 weights per second
// into products to keep pace with HBM. Dequantizing with the exact reference rounding already
// costs ~2 instructions per weight (LOP3 + HSUB2 + HMUL2 per fp16 pair, plus shifts), which is
// most of the SM's issue budget; an fp32 FMA per weight on top would make the kernel ALU-bound
// below the HBM roofline. So the warp dequantizes straight into mma.m16n8k16 A fragments and
// the tensor core performs the fp32 multiply-accumulate, for any M from 1 to 8 at the same
// instruction cost.
//
// Tiling. A warp owns 16 weight rows (n0..n0+15) and a strided subset of 128-wide K blocks.
// Lane L = 4*q + c loads a 16-byte vector of row n0+q and of row n0+q+8 covering k in
// [128b + 32c, 128b + 32c + 32): the 4 lanes of a quad read 64 contiguous bytes of each row.
// Each packed word (8 values of k) yields two m16n8k16 steps. The tensor core sums over the 16
// "logical" k of a step, so the logical-to-actual k mapping only has to agree between the A
// fragment (weights) and the B fragment (activations): word pairs 0,1 -> step 0 and pairs 2,3 ->
// step 1, which makes the B fragment of lane L exactly the 16 bytes x[m][k..k+7] of its own
// chunk (m = L/4). No shuffles, no shared-memory staging of the weights.
//
// Accumulators of the WARPS_K warps that split K are reduced through shared memory in warp
// order; cross-CTA split-K writes fp32 partials to the workspace and a second kernel reduces
// them in split order. Deterministic: graph replay and eager runs are bit-identical.
#include "tf_common.cuh"
#include "tf_plan.h"

namespace tfb {
namespace {

struct MmaParams {
  const __half* x;
  int64_t ldx;
  const int32_t* qw;
  const __half* scales;
  const int32_t* qzeros;
  const __half* bias;
  __half* y;
  int64_t ldy;
  float* partial;  // [split_k, M, N] fp32 when split_k > 1
  int64_t M, N, K;
  int group_size;
  int split_k;
  int blocks_per_split;
};

constexpr int kUnroll = 2;  // K blocks per pipeline stage per warp (two stages in registers)

template <int MT>
__device__ __forceinline__ void mma_block(float (&acc)[MT][4], const uint4& wa, const uint4& wb,
                                          bool kv, int64_t k, const MmaParams& p, int64_t rowA,
                                          int64_t rowB, bool okA, bool okB, int64_t m_base,
                                          int q) {
  __half2 zzA = zero_magic2(0), zzB = zero_magic2(0);
  __half2 ssA = __float2half2_rn(0.f), ssB = __float2half2_rn(0.f);
  if (kv) {
    const int64_t g = k / p.group_size;
    if (okA) {
      const __half s = __ldg(p.scales + g * p.N + rowA);
      ssA = __halves2half2(s, s);
      zzA = zero_magic2(zero_of(p.qzeros + g * (p.N / 8), rowA));
    }
    if (okB) {
      const __half s = __ldg(p.scales + g * p.N + rowB);
      ssB = __halves2half2(s, s);
      zzB = zero_magic2(zero_of(p.qzeros + g * (p.N / 8), rowB));
    }
  }
  const uint32_t wa_w[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wb_w[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t a0[4] = {dequant_pair(magic_pair(wa_w[i], 0), zzA, ssA),
                            dequant_pair(magic_pair(wb_w[i], 0), zzB, ssB),
                            dequant_pair(magic_pair(wa_w[i], 1), zzA, ssA),
                            dequant_pair(magic_pair(wb_w[i], 1), zzB, ssB)};
    const uint32_t a1[4] = {dequant_pair(magic_pair(wa_w[i], 2), zzA, ssA),
                            dequant_pair(magic_pair(wb_w[i], 2), zzB, ssB),
                            dequant_pair(magic_pair(wa_w[i], 3), zzA, ssA),
                            dequant_pair(magic_pair(wb_w[i], 3), zzB, ssB)};
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int64_t m = m_base + mt * 8 + q;
      uint4 xv = make_uint4(0, 0, 0, 0);
      if (kv && m < p.M) xv = ldg_v4(p.x + m * p.ldx + k + 8 * i);
      mma_16816(acc[mt], a0, xv.x, xv.y);
      mma_16816(acc[mt], a1, xv.z, xv.w);
    }
  }
}

template <int MT, int WARPS_N, int WARPS_K>
__global__ void __launch_bounds__(32 * WARPS_N * WARPS_K)
    w4a16_mma_kernel(const MmaParams p) {
  constexpr int kStep = WARPS_K * kUnroll;
  __shared__ float red[WARPS_K > 1 ? WARPS_N * WARPS_K * MT * 4 * 32 : 1];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn = warp / WARPS_K, wk = warp % WARPS_K;
  const int q = lane >> 2, c = lane & 3;
  const int64_t n0 = (static_cast<int64_t>(blockIdx.x) * WARPS_N + wn) * 16;
  const int64_t rowA = n0 + q, rowB = n0 + q + 8;
  const bool okA = rowA < p.N, okB = rowB < p.N;
  const int nblk = static_cast<int>((p.K + 127) / 128);
  const int b_begin = static_cast<int>(blockIdx.y) * p.blocks_per_split;
  const int b_end = min(nblk, b_begin + p.blocks_per_split);
  const int64_t ldw = p.K / 8;
  const int32_t* wA = p.qw + (okA ? rowA : 0) * ldw + 4 * c;
  const int32_t* wB = p.qw + (okB ? rowB : 0) * ldw + 4 * c;
  const int64_t m_base = static_cast<int64_t>(blockIdx.z) * (8 * MT);

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[mt][r] = 0.f;

  auto load_stage = [&](int b, uint4 (&wa)[kUnroll], uint4 (&wb)[kUnroll]) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int bb = b + u * WARPS_K;
      const int64_t k = static_cast<int64_t>(bb) * 128 + 32 * c;
      const bool kv = bb < b_end && k < p.K;
      wa[u] = (kv && okA) ? ldg_stream_v4(wA + static_cast<int64_t>(bb) * 16) : make_uint4(0, 0, 0, 0);
      wb[u] = (kv && okB) ? ldg_stream_v4(wB + static_cast<int64_t>(bb) * 16) : make_uint4(0, 0, 0, 0);
    }
  };

  // Weights never depend on the preceding kernel, so the first stage is requested before the
  // programmatic-dependent-launch wait; activations and every store come after it.
  uint4 wa[kUnroll], wb[kUnroll];
  int b = b_begin + wk;
  load_stage(b, wa, wb);
  pdl_wait();
  for (; b < b_end; b += kStep) {
    uint4 na[kUnroll], nb[kUnroll];
    load_stage(b + kStep, na, nb);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int bb = b + u * WARPS_K;
      const int64_t k = static_cast<int64_t>(bb) * 128 + 32 * c;
      const bool kv = bb < b_end && k < p.K;
      mma_block<MT>(acc, wa[u], wb[u], kv, k, p, rowA, rowB, okA, okB, m_base, q);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      wa[u] = na[u];
      wb[u] = nb[u];
    }
  }
  pdl_launch_dependents();

  if constexpr (WARPS_K > 1) {
    float* mine = red + ((wn * WARPS_K + wk) * MT * 4) * 32;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int r = 0; r < 4; ++r) mine[(mt * 4 + r) * 32 + lane] = acc[mt][r];
    __syncthreads();
    if (wk != 0) return;
    const float* base = red + (wn * WARPS_K * MT * 4) * 32;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS_K; ++w) s += base[(w * MT * 4 + mt * 4 + r) * 32 + lane];
        acc[mt][r] = s;
      }
  }

  // C fragment: c0,c1 -> row q, tokens 2c, 2c+1; c2,c3 -> row q+8, same tokens.
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t n = (r < 2) ? rowA : rowB;
      const int64_t m = m_base + mt * 8 + 2 * c + (r & 1);
      if (n >= p.N || m >= p.M) continue;
      if (p.split_k == 1) {
        float v = acc[mt][r];
        if (p.bias) v += __half2float(__ldg(p.bias + n));
        p.y[m * p.ldy + n] = __float2half_rn(v);
      } else {
        p.partial[(static_cast<int64_t>(blockIdx.y) * p.M + m) * p.N + n] = acc[mt][r];
      }
    }
  }
}

// Fixed-order reduction of split-K partials: sum splits 0..S-1, add bias, cast (w4a16.py:227-232).
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ partial,
                                                            int split_k, int64_t M, int64_t N,
                                                            const __half* __restrict__ bias,
                                                            __half* __restrict__ y, int64_t ldy) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t MN = M * N;
  if (idx >= MN) return;
  float s = 0.f;
  for (int sp = 0; sp < split_k; ++sp) s += partial[sp * MN + idx];
  const int64_t m = idx / N, n = idx - m * N;
  if (bias) s += __half2float(bias[n]);
  y[m * ldy + n] = __float2half_rn(s);
}

template <int MT, int WN, int WK>
int launch_variant(const LinearPlan& plan, const MmaParams& p, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid_x, plan.grid_y, plan.grid_z);
  cfg.blockDim = dim3(32 * WN * WK);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w4a16_mma_kernel<MT, WN, WK>, p);
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

template <int MT>
int launch_mt(const LinearPlan& plan, const MmaParams& p, cudaStream_t stream, bool pdl) {
  switch (plan.warps_k) {
    case 1: return launch_variant<MT, 8, 1>(plan, p, stream, pdl);
    case 2: return launch_variant<MT, 4, 2>(plan, p, stream, pdl);
    case 4: return launch_variant<MT, 2, 4>(plan, p, stream, pdl);
    case 8: return launch_variant<MT, 1, 8>(plan, p, stream, pdl);
    default: return TF_ERR_INVALID_ARG;
  }
}

}  // namespace

int launch_mma_linear(const LinearPlan& plan, const LinearArgs& a, cudaStream_t stream) {
  MmaParams p;
  p.x = reinterpret_cast<const __half*>(a.x);
  p.ldx = a.ldx;
  p.qw = a.qw;
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.qzeros = a.qzeros;
  p.bias = reinterpret_cast<const __half*>(a.bias);
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.partial = plan.split_k > 1 ? static_cast<float*>(a.workspace) : nullptr;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.group_size = a.group_size;
  p.split_k = plan.split_k;
  p.blocks_per_split = plan.blocks_per_split;
  const bool pdl = (launch_flags() & 1u) != 0;
  int st;
  if (plan.kernel == kKernelGemv)
    st = launch_mt<1>(plan, p, stream, pdl);
  else
    st = launch_mt<8>(plan, p, stream, pdl);
  if (st != TF_OK || plan.split_k == 1) return st;
  const int64_t MN = a.M * a.N;
  splitk_reduce_kernel<<<static_cast<unsigned>(cdiv(MN, 256)), 256, 0, stream>>>(
      p.partial, plan.split_k, a.M, a.N, p.bias, p.y, a.ldy);
  return check_launch();
}

}  // namespace tfb
