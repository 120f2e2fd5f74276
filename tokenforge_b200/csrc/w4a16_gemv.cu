// W4A16 decode GEMV for M = 1..8: y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]),
// w = fp16(q - z) * s rounded once, fp32 accumulation, fp16 output.
//
// Reference semantics: tokenforge/kernels/triton/w4a16.py:44-115 (the BLOCK_M == 1 / small-M
// paths) and its split-K contract w4a16.py:193-200,227-232 (fp32 partials summed in a fixed
// order, then bias, then the cast). Replaces the planned `_C.w4a16_gemv` (ops.py:86-88).
//
// The kernel is bound by the instructions that dequantize weights exactly (HSUB2 + HMUL2 per
// fp16 pair run at half rate on B200), so everything else is kept out of the inner loop:
//   * the CTA's activations x[0:M, k-range] are staged once in shared memory, so a K block costs
//     the warp one 16-byte shared load per packed word and no global address arithmetic;
//   * a warp owns 16 weight rows and walks 256-wide K blocks; lane L = 4q + c loads 32 bytes of
//     row n0+q and of row n0+q+8 (k in [256b + 64c, +64)), so each quad reads 128 contiguous bytes
//     per row, and three blocks (weights, scales, zero points) are held per warp in a register
//     ring, the first three requested before the programmatic-dependent-launch wait;
//   * rows beyond N and tokens beyond M are clamped for loading (never stored) instead of
//     predicated; only a partial last K block takes predicated loads;
//   * each packed word is unpacked with one shift: pairs 0 and 2 come from the mask 0x000F000F
//     of w and w >> 8 (fp16 1024 + q), pairs 1 and 3 from the mask 0x00F000F0 (1024 + 16q), whose
//     difference with 1024 + 16z is 16(q - z) exactly and is multiplied by the exact s/16, so both
//     give the reference's correctly rounded fp16(q - z) * s. When a scale in the warp is too
//     small for s/16 to be exact (s/16 * 16 != s), the block takes the three-shift unpack instead
//     (warp vote). Unpack and dequant are written in PTX (lop3, sub.rn / mul.rn.f16x2) so each
//     pair costs exactly three instructions.
// The dequantized pairs feed mma.m16n8k16 A fragments directly (the k order inside a step only
// has to agree between A and B); the tensor core does the fp32 multiply-accumulate.
// Warps that split K inside a CTA are summed through shared memory in warp order; CTAs that split
// K write fp32 partials reduced by a second kernel in split order: bit-identical on every run.
#include "tf_common.cuh"
#include "tf_plan.h"

namespace tfb {
namespace {

constexpr int kKB = 256;       // K values per block
constexpr int kCtaWarps = 8;   // warps per CTA (WARPS_N x WARPS_K)
constexpr int kPrefetch = 5;   // L2 prefetch distance in blocks (register loads run two ahead)

struct GemvParams {
  const __half* x;
  int64_t ldx;
  const int32_t* qw;
  const __half* scales;
  const int32_t* qzeros;
  const __half* bias;
  __half* y;
  int64_t ldy;
  float* partial;  // [split_k, M, N] fp32 when split_k > 1
  int M, N, K;
  int group_shift;  // log2(group size)
  int split_k;
  int bps;          // 256-wide K blocks per split
  int xs_stride;    // fp16 elements per staged activation row
};

// One K block of a warp tile in registers: this lane's 64 values of k for two weight rows.
struct GSlot {
  uint4 wa0, wa1, wb0, wb1;  // rows A and B: words 0-3 and 4-7 of the lane's chunk
  uint32_t s0, s1;           // 32-bit words of the scales rows holding rows A and B's scales ...
  uint32_t t0, t1;           // ... for the chunk's first and second 32-k half
  uint32_t za0, zb0, za1, zb1;  // qzeros words of those halves
};

struct GLane {
  const int32_t* wA;    // packed row A + this lane's word offset 8c
  const int32_t* wB;
  const uint32_t* sA;   // the 32-bit word of the scales row that holds row A's scale
  const uint32_t* sB;
  const int32_t* zA;    // qzeros + row A / 8
  const int32_t* zB;
  const uint4* xs;      // staged activations: token row q (clamped), + 64c
  uint32_t s_sel;       // byte_perm selector: row A's scale (low half), row B's (high half)
  int nibA, nibB;
  int kb0, b_end;       // this CTA's first block, this warp's end block (exclusive)
  int c;
};

__device__ __forceinline__ uint4 zero4() { return make_uint4(0, 0, 0, 0); }

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Ask L2 for block bb of this warp tile ahead of time (lane c == 0 of each quad fetches the
// 128-byte lines of its rows A and B, quad 0 the scales and qzeros lines), so the register loads
// issued one block ahead of use only wait for L2.
__device__ __forceinline__ void gprefetch(int bb, const GemvParams& p, const GLane& L) {
  if (bb >= L.b_end) return;
  if (L.c == 0) {
    prefetch_l2(L.wA + bb * (kKB / 8));
    prefetch_l2(L.wB + bb * (kKB / 8));
  }
  if (threadIdx.x % 32 < 2) {  // lanes 0, 1: rows n0..n0+15 of the block's first group
    const int g0 = (bb * kKB) >> p.group_shift;
    if (threadIdx.x % 32 == 0)
      prefetch_l2(L.sA + g0 * (p.N >> 1));
    else
      prefetch_l2(L.zA + g0 * (p.N >> 3));
  }
}

// Register loads of block bb (halves past K read as zero weights, scale 0, zero point 0).
template <bool kTwo>
__device__ __forceinline__ void gload(GSlot& s, int bb, const GemvParams& p, const GLane& L) {
  if (bb >= L.b_end) return;  // warp-uniform: the slot is never consumed
  const int k = bb * kKB + 64 * L.c;
  const int g0 = k >> p.group_shift;
  const int sw = p.N >> 1, n8 = p.N >> 3;
  const uint4* pa = reinterpret_cast<const uint4*>(L.wA + bb * (kKB / 8));
  const uint4* pb = reinterpret_cast<const uint4*>(L.wB + bb * (kKB / 8));
  if ((bb + 1) * kKB <= p.K) {
    s.wa0 = ldg_stream_v4(pa);
    s.wa1 = ldg_stream_v4(pa + 1);
    s.wb0 = ldg_stream_v4(pb);
    s.wb1 = ldg_stream_v4(pb + 1);
    s.s0 = __ldg(L.sA + g0 * sw);
    s.t0 = __ldg(L.sB + g0 * sw);
    s.za0 = static_cast<uint32_t>(__ldg(L.zA + g0 * n8));
    s.zb0 = static_cast<uint32_t>(__ldg(L.zB + g0 * n8));
    if constexpr (kTwo) {
      s.s1 = __ldg(L.sA + (g0 + 1) * sw);
      s.t1 = __ldg(L.sB + (g0 + 1) * sw);
      s.za1 = static_cast<uint32_t>(__ldg(L.zA + (g0 + 1) * n8));
      s.zb1 = static_cast<uint32_t>(__ldg(L.zB + (g0 + 1) * n8));
    }
  } else {  // partial last block
    const bool in0 = k < p.K, in1 = k + 32 < p.K;
    s.wa0 = in0 ? ldg_stream_v4(pa) : zero4();
    s.wa1 = in1 ? ldg_stream_v4(pa + 1) : zero4();
    s.wb0 = in0 ? ldg_stream_v4(pb) : zero4();
    s.wb1 = in1 ? ldg_stream_v4(pb + 1) : zero4();
    s.s0 = in0 ? __ldg(L.sA + g0 * sw) : 0u;
    s.t0 = in0 ? __ldg(L.sB + g0 * sw) : 0u;
    s.za0 = in0 ? static_cast<uint32_t>(__ldg(L.zA + g0 * n8)) : 0u;
    s.zb0 = in0 ? static_cast<uint32_t>(__ldg(L.zB + g0 * n8)) : 0u;
    if constexpr (kTwo) {
      s.s1 = in1 ? __ldg(L.sA + (g0 + 1) * sw) : 0u;
      s.t1 = in1 ? __ldg(L.sB + (g0 + 1) * sw) : 0u;
      s.za1 = in1 ? static_cast<uint32_t>(__ldg(L.zA + (g0 + 1) * n8)) : 0u;
      s.zb1 = in1 ? static_cast<uint32_t>(__ldg(L.zB + (g0 + 1) * n8)) : 0u;
    }
  }
}

// PTX forms of the unpack and dequant, so each pair costs exactly one LOP3, one fp16x2 subtract
// and one fp16x2 multiply (explicit .rn: never contracted into an FMA, which would round once
// less than the reference).
__device__ __forceinline__ uint32_t lop_mask_or(uint32_t w, uint32_t mask, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(mask), "r"(magic));
  return r;
}
__device__ __forceinline__ uint32_t hsub2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t dup_lo(uint32_t v) { return __byte_perm(v, v, 0x1010); }
__device__ __forceinline__ uint32_t dup_hi(uint32_t v) { return __byte_perm(v, v, 0x3232); }

// Loop-invariant bit patterns, held in registers for the whole kernel.
struct Consts {
  uint32_t m1;     // 0x000F000F: pairs 0 and 2
  uint32_t m16;    // 0x00F000F0: pairs 1 and 3 (value 16q)
  uint32_t magic;  // 0x64006400: fp16 1024 in both halves
};

struct HalfConsts {  // per 32-k half of a chunk: zero-point magics and scales for rows A and B
  uint32_t z1A, z1B, z16A, z16B, s1A, s1B, s16A, s16B;
  bool exact16;      // s/16 is exact for both rows (the one-shift unpack is valid)
};

__device__ __forceinline__ HalfConsts make_consts(uint32_t s, uint32_t za_w, uint32_t zb_w,
                                                  const GLane& L, const Consts& C) {
  HalfConsts h;
  const uint32_t za = (za_w >> L.nibA) & 0xFu, zb = (zb_w >> L.nibB) & 0xFu;
  h.z1A = (za * 0x00010001u) | C.magic;  // fp16 1024 + z in both halves
  h.z1B = (zb * 0x00010001u) | C.magic;
  h.z16A = (za * 0x00100010u) | C.magic;  // fp16 1024 + 16z
  h.z16B = (zb * 0x00100010u) | C.magic;
  const uint32_t s16 = hmul2_rn(s, 0x2C002C00u);  // s / 16 for rows A (low) and B (high)
  // s/16 is exact iff multiplying it back by 16 returns s (false for NaN: exact path taken).
  h.exact16 = hmul2_rn(s16, 0x4C004C00u) == s;
  h.s1A = dup_lo(s);
  h.s1B = dup_hi(s);
  h.s16A = dup_lo(s16);
  h.s16B = dup_hi(s16);
  return h;
}

// Pairs 0 and 2 are (w & 0x000F000F) and ((w >> 8) & 0x000F000F): fp16 1024 + q. Pairs 1 and 3
// use the mask 0x00F000F0, giving 1024 + 16q: subtracting 1024 + 16z leaves 16(q - z) exactly,
// and the exact s/16 turns it into the same correctly rounded fp16(q - z) * s as the reference.
__device__ __forceinline__ void word_fast(float (&acc)[4], uint32_t wa, uint32_t wb,
                                          const HalfConsts& h, const uint4& xv, const Consts& C) {
  const uint32_t a8 = wa >> 8, b8 = wb >> 8;
  const uint32_t f0[4] = {hmul2_rn(hsub2_rn(lop_mask_or(wa, C.m1, C.magic), h.z1A), h.s1A),
                          hmul2_rn(hsub2_rn(lop_mask_or(wb, C.m1, C.magic), h.z1B), h.s1B),
                          hmul2_rn(hsub2_rn(lop_mask_or(wa, C.m16, C.magic), h.z16A), h.s16A),
                          hmul2_rn(hsub2_rn(lop_mask_or(wb, C.m16, C.magic), h.z16B), h.s16B)};
  const uint32_t f1[4] = {hmul2_rn(hsub2_rn(lop_mask_or(a8, C.m1, C.magic), h.z1A), h.s1A),
                          hmul2_rn(hsub2_rn(lop_mask_or(b8, C.m1, C.magic), h.z1B), h.s1B),
                          hmul2_rn(hsub2_rn(lop_mask_or(a8, C.m16, C.magic), h.z16A), h.s16A),
                          hmul2_rn(hsub2_rn(lop_mask_or(b8, C.m16, C.magic), h.z16B), h.s16B)};
  mma_16816(acc, f0, xv.x, xv.y);
  mma_16816(acc, f1, xv.z, xv.w);
}

// Unit-scale unpack of every pair (three shifts per word): used for a block in which some scale
// is too small for s/16 to be exact.
__device__ __forceinline__ void word_exact(float (&acc)[4], uint32_t wa, uint32_t wb,
                                           const HalfConsts& h, const uint4& xv, const Consts& C) {
  uint32_t f[2][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t ma = lop_mask_or(wa >> (4 * j), C.m1, C.magic);
    const uint32_t mb = lop_mask_or(wb >> (4 * j), C.m1, C.magic);
    f[j >> 1][(j & 1) * 2 + 0] = hmul2_rn(hsub2_rn(ma, h.z1A), h.s1A);
    f[j >> 1][(j & 1) * 2 + 1] = hmul2_rn(hsub2_rn(mb, h.z1B), h.s1B);
  }
  mma_16816(acc, f[0], xv.x, xv.y);
  mma_16816(acc, f[1], xv.z, xv.w);
}

template <bool kTwo>
__device__ __forceinline__ void gcompute(float (&acc)[2][4], const GSlot& s, int bb,
                                         const GLane& L, int K, const Consts& C) {
  const uint4* xp = L.xs + (bb - L.kb0) * (kKB / 8);
  const HalfConsts h0 = make_consts(__byte_perm(s.s0, s.t0, L.s_sel), s.za0, s.zb0, L, C);
  HalfConsts h1 = h0;
  if constexpr (kTwo) {
    h1 = make_consts(__byte_perm(s.s1, s.t1, L.s_sel), s.za1, s.zb1, L, C);
  } else if ((bb + 1) * kKB > K) {  // warp-uniform: partial last block
    // A second half past K has zero weights and zero activations; give it s = 0, z = 0 as well
    // so it adds exact zeros whatever the first half's scale is.
    if (bb * kKB + 64 * L.c + 32 >= K) h1 = make_consts(0u, 0u, 0u, L, C);
  }
  const bool fast = __all_sync(0xffffffffu, h0.exact16 && h1.exact16);
  const uint32_t wa[8] = {s.wa0.x, s.wa0.y, s.wa0.z, s.wa0.w, s.wa1.x, s.wa1.y, s.wa1.z, s.wa1.w};
  const uint32_t wb[8] = {s.wb0.x, s.wb0.y, s.wb0.z, s.wb0.w, s.wb1.x, s.wb1.y, s.wb1.z, s.wb1.w};
  if (fast) {
#pragma unroll
    for (int j = 0; j < 8; ++j) word_fast(acc[j & 1], wa[j], wb[j], j < 4 ? h0 : h1, xp[j], C);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) word_exact(acc[j & 1], wa[j], wb[j], j < 4 ? h0 : h1, xp[j], C);
  }
}

template <int WARPS_N, int WARPS_K, bool kTwo>
__global__ void __launch_bounds__(32 * kCtaWarps, 2) w4a16_gemv_kernel(const GemvParams p) {
  static_assert(WARPS_N * WARPS_K == kCtaWarps, "CTA shape");
  extern __shared__ uint4 xs_smem[];
  __shared__ float red[kCtaWarps * 4 * 32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn = warp / WARPS_K, wk = warp % WARPS_K;
  const int q = lane >> 2;
  GLane L;
  L.c = lane & 3;
  const int n0 = (blockIdx.x * WARPS_N + wn) * 16;
  const int rowA = n0 + q, rowB = n0 + q + 8;
  const int ra = min(rowA, p.N - 1), rb = min(rowB, p.N - 1);
  const int nblk = (p.K + kKB - 1) / kKB;
  L.kb0 = blockIdx.y * p.bps;
  const int kb1 = min(nblk, L.kb0 + p.bps);
  L.b_end = kb1;
  const int64_t ldw = p.K / 8;
  L.wA = p.qw + ra * ldw + 8 * L.c;
  L.wB = p.qw + rb * ldw + 8 * L.c;
  L.sA = reinterpret_cast<const uint32_t*>(p.scales) + (ra >> 1);
  L.sB = reinterpret_cast<const uint32_t*>(p.scales) + (rb >> 1);
  L.s_sel = ((ra & 1) ? 0x3232u : 0x1010u) & 0x00FFu;
  L.s_sel |= ((rb & 1) ? 0x7676u : 0x5454u) & 0xFF00u;
  L.zA = p.qzeros + (ra >> 3);
  L.zB = p.qzeros + (rb >> 3);
  L.nibA = 4 * awq_nibble_of(ra & 7);
  L.nibB = 4 * awq_nibble_of(rb & 7);
  const int xq = min(q, p.M - 1);
  L.xs = xs_smem + (xq * p.xs_stride + 64 * L.c) / 8;
  Consts C;
  C.m1 = 0x000F000Fu;
  C.m16 = 0x00F000F0u;
  C.magic = 0x64006400u;

  // Weights, scales and zero points never depend on the preceding kernel: the L2 prefetches of
  // the first kPrefetch blocks and the register loads of the first two are issued before the
  // programmatic-dependent-launch wait.
  const int b0 = L.kb0 + wk;
  constexpr int W = WARPS_K;
#pragma unroll
  for (int d = 2; d < kPrefetch; ++d) gprefetch(b0 + d * W, p, L);
  GSlot s0, s1;
  gload<kTwo>(s0, b0, p, L);
  gload<kTwo>(s1, b0 + W, p, L);
  pdl_wait();

  // Stage x[0:M, kb0*256 : kb1*256] (zero past K) in shared memory.
  {
    const int vec_per_row = (kb1 - L.kb0) * (kKB / 8);
    const int total = p.M * vec_per_row;
    const int k_lo = L.kb0 * kKB;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int m = i / vec_per_row, v = i - m * vec_per_row;
      const int k = k_lo + 8 * v;
      const uint4 val = k < p.K ? ldg_v4(p.x + m * p.ldx + k) : zero4();
      xs_smem[(m * p.xs_stride) / 8 + v] = val;
    }
  }
  __syncthreads();

  // Two accumulators (even / odd packed words) keep the tensor-core accumulate chains short;
  // they are added in a fixed order at the end.
  float acc2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int b = b0; b < L.b_end; b += 2 * W) {
    gprefetch(b + kPrefetch * W, p, L);
    gcompute<kTwo>(acc2, s0, b, L, p.K, C);
    gload<kTwo>(s0, b + 2 * W, p, L);
    if (b + W >= L.b_end) break;
    gprefetch(b + (kPrefetch + 1) * W, p, L);
    gcompute<kTwo>(acc2, s1, b + W, L, p.K, C);
    gload<kTwo>(s1, b + 3 * W, p, L);
  }
  float acc[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r] = acc2[0][r] + acc2[1][r];
  pdl_launch_dependents();

  if constexpr (WARPS_K > 1) {
    float* mine = red + (warp * 4) * 32;
#pragma unroll
    for (int r = 0; r < 4; ++r) mine[r * 32 + lane] = acc[r];
    __syncthreads();
    if (wk != 0) return;
    const float* base = red + (wn * WARPS_K * 4) * 32;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS_K; ++w) v += base[(w * 4 + r) * 32 + lane];
      acc[r] = v;
    }
  }

  // C fragment: acc[0..1] -> row A, tokens 2c, 2c+1; acc[2..3] -> row B, same tokens.
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int n = (r < 2) ? rowA : rowB;
    const int m = 2 * L.c + (r & 1);
    if (n >= p.N || m >= p.M) continue;
    if (p.split_k == 1) {
      float v = acc[r];
      if (p.bias) v += __half2float(__ldg(p.bias + n));
      p.y[m * p.ldy + n] = __float2half_rn(v);
    } else {
      p.partial[(static_cast<int64_t>(blockIdx.y) * p.M + m) * p.N + n] = acc[r];
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

template <int WN, int WK, bool kTwo>
int launch_gemv_variant(const LinearPlan& plan, const GemvParams& p, size_t smem,
                        cudaStream_t stream, bool pdl) {
  auto kern = w4a16_gemv_kernel<WN, WK, kTwo>;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) {
      last_cuda_error() = static_cast<int>(e);
      return TF_ERR_CUDA;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid_x, plan.grid_y, 1);
  cfg.blockDim = dim3(32 * kCtaWarps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

template <bool kTwo>
int launch_gemv_two(const LinearPlan& plan, const GemvParams& p, size_t smem, cudaStream_t st,
                    bool pdl) {
  switch (plan.warps_k) {
    case 1: return launch_gemv_variant<8, 1, kTwo>(plan, p, smem, st, pdl);
    case 2: return launch_gemv_variant<4, 2, kTwo>(plan, p, smem, st, pdl);
    case 4: return launch_gemv_variant<2, 4, kTwo>(plan, p, smem, st, pdl);
    case 8: return launch_gemv_variant<1, 8, kTwo>(plan, p, smem, st, pdl);
    default: return TF_ERR_INVALID_ARG;
  }
}

}  // namespace

size_t gemv_smem_bytes(int64_t M, int bps) {
  const int64_t stride = static_cast<int64_t>(bps) * kKB + 8;  // +16 B per row: bank offset
  return static_cast<size_t>(M * stride * 2);
}

int launch_gemv(const LinearPlan& plan, const LinearArgs& a, cudaStream_t stream) {
  GemvParams p;
  p.x = reinterpret_cast<const __half*>(a.x);
  p.ldx = a.ldx;
  p.qw = a.qw;
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.qzeros = a.qzeros;
  p.bias = reinterpret_cast<const __half*>(a.bias);
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.partial = plan.split_k > 1 ? static_cast<float*>(a.workspace) : nullptr;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.group_shift = a.group_size == 32 ? 5 : (a.group_size == 64 ? 6 : 7);
  p.split_k = plan.split_k;
  p.bps = plan.blocks_per_split;
  p.xs_stride = plan.blocks_per_split * kKB + 8;
  const size_t x_bytes = gemv_smem_bytes(a.M, plan.blocks_per_split);
  const bool pdl = (launch_flags() & TF_LAUNCH_PDL) != 0;
  const int st = a.group_size == 32 ? launch_gemv_two<true>(plan, p, x_bytes, stream, pdl)
                                    : launch_gemv_two<false>(plan, p, x_bytes, stream, pdl);
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
