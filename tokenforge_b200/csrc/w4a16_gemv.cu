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

// One K block (128 values of k) of one warp tile, as held in registers between the moment its
// loads are issued and the moment it is consumed.
template <int MT>
struct Slot {
  uint4 wa, wb;                 // packed weights of rows A = n0+q and B = n0+q+8 (16 B each)
  __half sa, sb;                // scales of the block's group for rows A and B
  uint32_t za, zb;              // qzeros words holding the rows' zero points
  uint4 x[MT == 1 ? 4 : 1];     // activations x[q][k..k+31] (decode tile only)
  int64_t k;                    // first k of this lane's 32-value chunk
  bool kv;                      // the block exists (k < K and inside this CTA's K range)
};

struct TileGeom {
  int64_t rowA, rowB, m_base;
  bool okA, okB;
  int q, c, b_end;
  const int32_t* wA;
  const int32_t* wB;
};

// Weights, scales and zero points: never written by the preceding kernel, so these loads may be
// issued before the programmatic-dependent-launch wait.
template <int MT>
__device__ __forceinline__ void load_weights(Slot<MT>& s, int bb, const MmaParams& p,
                                             const TileGeom& t) {
  s.k = static_cast<int64_t>(bb) * 128 + 32 * t.c;
  s.kv = bb < t.b_end && s.k < p.K;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  s.wa = (s.kv && t.okA) ? ldg_stream_v4(t.wA + static_cast<int64_t>(bb) * 16) : zero;
  s.wb = (s.kv && t.okB) ? ldg_stream_v4(t.wB + static_cast<int64_t>(bb) * 16) : zero;
  s.sa = s.sb = __ushort_as_half(0);
  s.za = s.zb = 0;
  if (s.kv) {
    const int64_t g = s.k / p.group_size;
    if (t.okA) {
      s.sa = __ldg(p.scales + g * p.N + t.rowA);
      s.za = static_cast<uint32_t>(__ldg(p.qzeros + g * (p.N / 8) + (t.rowA >> 3)));
    }
    if (t.okB) {
      s.sb = __ldg(p.scales + g * p.N + t.rowB);
      s.zb = static_cast<uint32_t>(__ldg(p.qzeros + g * (p.N / 8) + (t.rowB >> 3)));
    }
  }
}

// Activations (decode tile only; the 64-token tile reads them while computing).
template <int MT>
__device__ __forceinline__ void load_acts(Slot<MT>& s, const MmaParams& p, const TileGeom& t) {
  if constexpr (MT == 1) {
    const int64_t m = t.m_base + t.q;
    const bool ok = s.kv && m < p.M;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      s.x[i] = ok ? ldg_v4(p.x + m * p.ldx + s.k + 8 * i) : make_uint4(0, 0, 0, 0);
  }
}

template <int MT>
__device__ __forceinline__ void mma_slot(float (&acc)[MT][4], const Slot<MT>& s,
                                         const MmaParams& p, const TileGeom& t) {
  const int nibA = 4 * awq_nibble_of(static_cast<int>(t.rowA & 7));
  const int nibB = 4 * awq_nibble_of(static_cast<int>(t.rowB & 7));
  const __half2 zzA = zero_magic2((s.za >> nibA) & 0xFu);
  const __half2 zzB = zero_magic2((s.zb >> nibB) & 0xFu);
  const __half2 ssA = __halves2half2(s.sa, s.sa);
  const __half2 ssB = __halves2half2(s.sb, s.sb);
  const uint32_t wa_w[4] = {s.wa.x, s.wa.y, s.wa.z, s.wa.w};
  const uint32_t wb_w[4] = {s.wb.x, s.wb.y, s.wb.z, s.wb.w};
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
    if constexpr (MT == 1) {
      mma_16816(acc[0], a0, s.x[i].x, s.x[i].y);
      mma_16816(acc[0], a1, s.x[i].z, s.x[i].w);
    } else {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int64_t m = t.m_base + mt * 8 + t.q;
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (s.kv && m < p.M) xv = ldg_v4(p.x + m * p.ldx + s.k + 8 * i);
        mma_16816(acc[mt], a0, xv.x, xv.y);
        mma_16816(acc[mt], a1, xv.z, xv.w);
      }
    }
  }
}

template <int MT, int WARPS_N, int WARPS_K>
__global__ void __launch_bounds__(32 * WARPS_N * WARPS_K)
    w4a16_mma_kernel(const MmaParams p) {
  __shared__ float red[WARPS_K > 1 ? WARPS_N * WARPS_K * MT * 4 * 32 : 1];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn = warp / WARPS_K, wk = warp % WARPS_K;
  TileGeom t;
  t.q = lane >> 2;
  t.c = lane & 3;
  const int64_t n0 = (static_cast<int64_t>(blockIdx.x) * WARPS_N + wn) * 16;
  t.rowA = n0 + t.q;
  t.rowB = n0 + t.q + 8;
  t.okA = t.rowA < p.N;
  t.okB = t.rowB < p.N;
  const int nblk = static_cast<int>((p.K + 127) / 128);
  const int b_begin = static_cast<int>(blockIdx.y) * p.blocks_per_split;
  t.b_end = min(nblk, b_begin + p.blocks_per_split);
  const int64_t ldw = p.K / 8;
  t.wA = p.qw + (t.okA ? t.rowA : 0) * ldw + 4 * t.c;
  t.wB = p.qw + (t.okB ? t.rowB : 0) * ldw + 4 * t.c;
  t.m_base = static_cast<int64_t>(blockIdx.z) * (8 * MT);

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[mt][r] = 0.f;

  // Three K blocks in flight per warp (register ring). Weights, scales and zero points of the
  // first three are requested before the programmatic-dependent-launch wait; activations and
  // every store come after it.
  constexpr int W = WARPS_K;
  const int b0 = b_begin + wk;
  Slot<MT> s0, s1, s2;
  load_weights(s0, b0, p, t);
  load_weights(s1, b0 + W, p, t);
  load_weights(s2, b0 + 2 * W, p, t);
  pdl_wait();
  load_acts(s0, p, t);
  load_acts(s1, p, t);
  load_acts(s2, p, t);
  for (int b = b0; b < t.b_end; b += 3 * W) {
    mma_slot(acc, s0, p, t);
    load_weights(s0, b + 3 * W, p, t);
    load_acts(s0, p, t);
    if (b + W >= t.b_end) break;
    mma_slot(acc, s1, p, t);
    load_weights(s1, b + 4 * W, p, t);
    load_acts(s1, p, t);
    if (b + 2 * W >= t.b_end) break;
    mma_slot(acc, s2, p, t);
    load_weights(s2, b + 5 * W, p, t);
    load_acts(s2, p, t);
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
      const int64_t n = (r < 2) ? t.rowA : t.rowB;
      const int64_t m = t.m_base + mt * 8 + 2 * t.c + (r & 1);
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
  return launch_splitk_reduce(p.partial, plan.split_k, a.M, a.N, a.bias, a.y, a.ldy, stream);
}

int launch_splitk_reduce(const float* partial, int split, int64_t M, int64_t N,
                         const uint16_t* bias, uint16_t* y, int64_t ldy, cudaStream_t stream) {
  const int64_t MN = M * N;
  splitk_reduce_kernel<<<static_cast<unsigned>(cdiv(MN, 256)), 256, 0, stream>>>(
      partial, split, M, N, reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(y),
      ldy);
  return check_launch();
}

}  // namespace tfb
