// W4A16 linear on the warp-level tensor-core path in 64-token tiles: the prefill kernel for
// shapes the tcgen05 GEMM does not take (N not a multiple of 32 or K not a multiple of 64).
// y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]) with w = fp16(q - z) * s.
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
  int group_shift;  // log2(group size)
  int split_k;
  int blocks_per_split;
};

// One K block (128 values of k) of one warp tile, held in registers from the moment its loads
// are issued until it is consumed.
template <int MT>
struct Slot {
  uint4 wa, wb;              // packed weights of rows A = n0+q and B = n0+q+8 (16 B each)
  uint32_t s;                // scales of rows A (low half) and B (high half), fp16 bits
  uint32_t za, zb;           // qzeros words holding the rows' zero points
  uint4 x[MT == 1 ? 4 : 1];  // activations x[m][k..k+31] of this lane's chunk (decode tile)
};

// Per-lane constants of a warp tile. Rows at or beyond N and tokens at or beyond M are clamped
// to the last valid one for loading (their results are never stored), so the steady-state loop
// needs no predication; only a partial last K block (K % 128 != 0) is loaded with predicates.
struct TileGeom {
  const int32_t* wA;    // row A's packed words + 4c
  const int32_t* wB;
  const __half* sA;     // scales + row A
  const __half* sB;
  const int32_t* zA;    // qzeros + row A / 8
  const int32_t* zB;
  const __half* xrow;   // x + token * ldx + 32c
  int64_t rowA, rowB, m_base;
  int nibA, nibB;       // bit offset of the rows' zero points inside a qzeros word
  int q, c, b_end;
};

__device__ __forceinline__ uint4 zero4() { return make_uint4(0, 0, 0, 0); }

// Weights, scales and zero points: never written by the preceding kernel, so these loads may be
// issued before the programmatic-dependent-launch wait.
template <int MT>
__device__ __forceinline__ void load_weights(Slot<MT>& s, int bb, const MmaParams& p,
                                             const TileGeom& t) {
  if (bb >= t.b_end) return;  // warp-uniform: this slot is never consumed
  const int64_t k = static_cast<int64_t>(bb) * 128 + 32 * t.c;
  const int64_t g = k >> p.group_shift;
  const int64_t off = static_cast<int64_t>(bb) * 16;
  if ((static_cast<int64_t>(bb) + 1) * 128 <= p.K) {
    s.wa = ldg_stream_v4(t.wA + off);
    s.wb = ldg_stream_v4(t.wB + off);
    const uint32_t sa = __half_as_ushort(__ldg(t.sA + g * p.N));
    const uint32_t sb = __half_as_ushort(__ldg(t.sB + g * p.N));
    s.s = sa | (sb << 16);
    s.za = static_cast<uint32_t>(__ldg(t.zA + g * (p.N >> 3)));
    s.zb = static_cast<uint32_t>(__ldg(t.zB + g * (p.N >> 3)));
  } else {  // partial last block: lanes past K contribute exact zeros
    const bool in = k < p.K;
    s.wa = in ? ldg_stream_v4(t.wA + off) : zero4();
    s.wb = in ? ldg_stream_v4(t.wB + off) : zero4();
    const uint32_t sa = in ? __half_as_ushort(__ldg(t.sA + g * p.N)) : 0u;
    const uint32_t sb = in ? __half_as_ushort(__ldg(t.sB + g * p.N)) : 0u;
    s.s = sa | (sb << 16);
    s.za = in ? static_cast<uint32_t>(__ldg(t.zA + g * (p.N >> 3))) : 0u;
    s.zb = in ? static_cast<uint32_t>(__ldg(t.zB + g * (p.N >> 3))) : 0u;
  }
}

// Activations of the decode tile (the 64-token tile reads them while computing).
template <int MT>
__device__ __forceinline__ void load_acts(Slot<MT>& s, int bb, const MmaParams& p,
                                          const TileGeom& t) {
  if constexpr (MT == 1) {
    if (bb >= t.b_end) return;
    const int64_t off = static_cast<int64_t>(bb) * 128;
    if ((static_cast<int64_t>(bb) + 1) * 128 <= p.K) {
#pragma unroll
      for (int i = 0; i < 4; ++i) s.x[i] = ldg_v4(t.xrow + off + 8 * i);
    } else {
      const bool in = off + 32 * t.c < p.K;
#pragma unroll
      for (int i = 0; i < 4; ++i) s.x[i] = in ? ldg_v4(t.xrow + off + 8 * i) : zero4();
    }
  }
}

// A scale s admits the cheaper unpack below iff s/16 is exact in fp16: s is zero, non-finite,
// or at least 2^-10 in magnitude (so s/16 is still a normal number).
__device__ __forceinline__ bool scale_splits_exactly(uint32_t h) {
  const uint32_t mag = h & 0x7FFFu;
  return mag == 0u || mag >= 0x1400u;
}

__device__ __forceinline__ void mma_step(float (&acc)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  mma_16816(acc, a, b0, b1);
}

template <int MT>
__device__ __forceinline__ void mma_slot(float (&acc)[MT][4], const Slot<MT>& s, int bb,
                                         const MmaParams& p, const TileGeom& t) {
  const uint32_t za = (s.za >> t.nibA) & 0xFu, zb = (s.zb >> t.nibB) & 0xFu;
  const __half2 ss1A = __halves2half2(__ushort_as_half(s.s & 0xFFFFu), __ushort_as_half(s.s & 0xFFFFu));
  const __half2 ss1B = __halves2half2(__ushort_as_half(s.s >> 16), __ushort_as_half(s.s >> 16));
  const uint32_t wa[4] = {s.wa.x, s.wa.y, s.wa.z, s.wa.w};
  const uint32_t wb[4] = {s.wb.x, s.wb.y, s.wb.z, s.wb.w};
  const bool fast = __all_sync(0xffffffffu, scale_splits_exactly(s.s & 0xFFFFu) &&
                                                scale_splits_exactly(s.s >> 16));
  if (fast) {
    // Pairs 0 and 2 are (w & 0x000F000F) and ((w >> 8) & 0x000F000F): fp16 1024 + q. Pairs 1
    // and 3 use the mask 0x00F000F0 instead, giving 1024 + 16q: subtracting 1024 + 16z yields
    // 16(q - z) exactly, and multiplying by the exact s/16 gives the same correctly rounded
    // fp16(q - z) * s as the reference, with one shift per word instead of three.
    const __half2 zz1A = zero_magic2(za), zz1B = zero_magic2(zb);
    const __half2 zz16A = u32_as_h2(0x64006400u | (za << 4) | (za << 20));
    const __half2 zz16B = u32_as_h2(0x64006400u | (zb << 4) | (zb << 20));
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const __half2 ss16A = __hmul2(ss1A, sixteenth), ss16B = __hmul2(ss1B, sixteenth);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a8 = wa[i] >> 8, b8 = wb[i] >> 8;
      const uint32_t a0[4] = {dequant_pair((wa[i] & 0x000F000Fu) | 0x64006400u, zz1A, ss1A),
                              dequant_pair((wb[i] & 0x000F000Fu) | 0x64006400u, zz1B, ss1B),
                              dequant_pair((wa[i] & 0x00F000F0u) | 0x64006400u, zz16A, ss16A),
                              dequant_pair((wb[i] & 0x00F000F0u) | 0x64006400u, zz16B, ss16B)};
      const uint32_t a1[4] = {dequant_pair((a8 & 0x000F000Fu) | 0x64006400u, zz1A, ss1A),
                              dequant_pair((b8 & 0x000F000Fu) | 0x64006400u, zz1B, ss1B),
                              dequant_pair((a8 & 0x00F000F0u) | 0x64006400u, zz16A, ss16A),
                              dequant_pair((b8 & 0x00F000F0u) | 0x64006400u, zz16B, ss16B)};
      if constexpr (MT == 1) {
        mma_step(acc[0], a0, s.x[i].x, s.x[i].y);
        mma_step(acc[0], a1, s.x[i].z, s.x[i].w);
      } else {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int64_t m = min(t.m_base + mt * 8 + t.q, p.M - 1);
          const int64_t k = static_cast<int64_t>(bb) * 128 + 32 * t.c;
          const uint4 xv = k < p.K ? ldg_v4(p.x + m * p.ldx + k + 8 * i) : zero4();
          mma_step(acc[mt], a0, xv.x, xv.y);
          mma_step(acc[mt], a1, xv.z, xv.w);
        }
      }
    }
  } else {
    // Any scale in the warp too small for an exact s/16: unpack every pair at unit scale.
    const __half2 zz1A = zero_magic2(za), zz1B = zero_magic2(zb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a0[4] = {dequant_pair(magic_pair(wa[i], 0), zz1A, ss1A),
                              dequant_pair(magic_pair(wb[i], 0), zz1B, ss1B),
                              dequant_pair(magic_pair(wa[i], 1), zz1A, ss1A),
                              dequant_pair(magic_pair(wb[i], 1), zz1B, ss1B)};
      const uint32_t a1[4] = {dequant_pair(magic_pair(wa[i], 2), zz1A, ss1A),
                              dequant_pair(magic_pair(wb[i], 2), zz1B, ss1B),
                              dequant_pair(magic_pair(wa[i], 3), zz1A, ss1A),
                              dequant_pair(magic_pair(wb[i], 3), zz1B, ss1B)};
      if constexpr (MT == 1) {
        mma_step(acc[0], a0, s.x[i].x, s.x[i].y);
        mma_step(acc[0], a1, s.x[i].z, s.x[i].w);
      } else {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int64_t m = min(t.m_base + mt * 8 + t.q, p.M - 1);
          const int64_t k = static_cast<int64_t>(bb) * 128 + 32 * t.c;
          const uint4 xv = k < p.K ? ldg_v4(p.x + m * p.ldx + k + 8 * i) : zero4();
          mma_step(acc[mt], a0, xv.x, xv.y);
          mma_step(acc[mt], a1, xv.z, xv.w);
        }
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
  const int64_t ra = min(t.rowA, p.N - 1), rb = min(t.rowB, p.N - 1);
  const int nblk = static_cast<int>((p.K + 127) / 128);
  const int b_begin = static_cast<int>(blockIdx.y) * p.blocks_per_split;
  t.b_end = min(nblk, b_begin + p.blocks_per_split);
  const int64_t ldw = p.K / 8;
  t.wA = p.qw + ra * ldw + 4 * t.c;
  t.wB = p.qw + rb * ldw + 4 * t.c;
  t.sA = p.scales + ra;
  t.sB = p.scales + rb;
  t.zA = p.qzeros + (ra >> 3);
  t.zB = p.qzeros + (rb >> 3);
  t.nibA = 4 * awq_nibble_of(static_cast<int>(ra & 7));
  t.nibB = 4 * awq_nibble_of(static_cast<int>(rb & 7));
  t.m_base = static_cast<int64_t>(blockIdx.z) * (8 * MT);
  t.xrow = p.x + min(t.m_base + t.q, p.M - 1) * p.ldx + 32 * t.c;

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
  load_acts(s0, b0, p, t);
  load_acts(s1, b0 + W, p, t);
  load_acts(s2, b0 + 2 * W, p, t);
  for (int b = b0; b < t.b_end; b += 3 * W) {
    mma_slot(acc, s0, b, p, t);
    load_weights(s0, b + 3 * W, p, t);
    load_acts(s0, b + 3 * W, p, t);
    if (b + W >= t.b_end) break;
    mma_slot(acc, s1, b + W, p, t);
    load_weights(s1, b + 4 * W, p, t);
    load_acts(s1, b + 4 * W, p, t);
    if (b + 2 * W >= t.b_end) break;
    mma_slot(acc, s2, b + 2 * W, p, t);
    load_weights(s2, b + 5 * W, p, t);
    load_acts(s2, b + 5 * W, p, t);
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

int launch_mma_tiles(const LinearPlan& plan, const LinearArgs& a, cudaStream_t stream) {
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
  p.group_shift = a.group_size == 32 ? 5 : (a.group_size == 64 ? 6 : 7);
  p.split_k = plan.split_k;
  p.blocks_per_split = plan.blocks_per_split;
  const bool pdl = (launch_flags() & 1u) != 0;
  const int st = launch_mt<8>(plan, p, stream, pdl);
  if (st != TF_OK || plan.split_k == 1) return st;
  return launch_splitk_reduce(p.partial, plan.split_k, a.M, a.N, a.bias, a.y, a.ldy, stream);
}

}  // namespace tfb
