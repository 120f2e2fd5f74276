// W4A16 decode GEMVs: y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]), w = fp16(q - z) * s
// rounded once, fp32 accumulation, fp16 output. This file holds
//   * w4a16_gemv_kernel, M = 1..8 (described below), with variants that take e4m3 activations
//     (x8), fuse the row-parallel all-reduce over NVLink peer stores (peer_exchange), normalise
//     and quantise the staged rows first (kNorm: RMSNorm + FP8), or form the SiLU products while
//     staging (kSilu);
//   * w4a16_gemv16_kernel, M = 9..16 at group size 128: the same weight stream feeding two
//     8-token MMA n-tiles;
//   * splitk_reduce_kernel for K splits that span several clusters.
//
// Reference semantics: tokenforge/kernels/triton/w4a16.py:44-115 (the BLOCK_M == 1 / small-M
// paths) and its split-K contract w4a16.py:193-200,227-232 (partials summed in a fixed order,
// then bias, then the cast). Replaces the planned `_C.w4a16_gemv` (ops.py:86-88).
//
// The kernel is bound by the instructions that dequantize weights exactly (LOP3 + HSUB2 + HMUL2
// per fp16 pair; the fp16x2 ops run at half rate on B200), so everything else is amortized:
//   * a warp owns 32 weight rows as two mma.m16n8k16 tiles; lane L = 4q + c holds the four
//     contiguous rows 4q..4q+3 (tile 0 rows q / q+8 <- rows 4q / 4q+1, tile 1 <- 4q+2 / 4q+3), so
//     their four scales arrive in one 8-byte load already paired the way the fragments use them,
//     their zero points sit in one qzeros word, and one activation fragment feeds both tiles;
//   * the warp walks a contiguous range of 128-wide K blocks; lane c reads 16 bytes (k in
//     [128b + 32c, +32)) of each of its rows, so a quad reads 64 contiguous bytes per row;
//   * the CTA's activations x[0:M, k-range] are staged once in shared memory;
//   * weights, scales and zero points are loaded into registers two blocks ahead through four
//     row pointers kept in registers (no L2 prefetch: measured, its address work cost more than
//     it hid); the first loads are issued before the programmatic-dependent-launch wait;
//   * rows beyond N and tokens beyond M are clamped for loading (never stored); only a partial
//     last K block takes predicated loads;
//   * unpack and dequant are PTX (lop3, sub.rn / mul.rn.f16x2): three instructions per fp16 pair
//     plus one shift per packed word at group size 128 (bits 4-7 of each half unpack through the
//     0x5400 magic), bit-exact with the reference dequant.
// The dequantized pairs feed the tensor core directly (the k order inside an MMA step only has to
// agree between the A and B fragments); it performs the fp32 multiply-accumulate, four
// independent accumulator chains per lane.
// K is split over WARPS_K warps of a CTA (summed through shared memory in warp order) and over
// the CTAs of a thread-block cluster (rank 0 sums the ranks' partials through distributed shared
// memory in rank order): deterministic, no workspace, no second launch. CTAs that split K beyond
// one cluster write fp32 partials that a second kernel reduces in split order.
#include <atomic>

#include "tf_common.cuh"
#include "tf_plan.h"
#include "tf_rmsnorm.cuh"
#include "tf_w4a16_math.cuh"

namespace tfb {
namespace {

// Device buffer that fused all-reduce launches stamp (tf_peer_trace), or null.
std::atomic<uint64_t*> g_peer_trace{nullptr};

constexpr int kCtaWarps = 8;     // warps per CTA (WARPS_N x WARPS_K), two CTAs per SM ...
constexpr int kWideWarps = 16;   // ... or one 16-warp CTA per SM splitting K 16 ways
constexpr int kWarpRows = 32;    // weight rows per warp tile

struct GemvParams {
  const __half* x;
  int64_t ldx;
  // FP8 activations (x8 != null, x unused): e4m3 codes [M, K] with row stride ldx bytes, staged
  // as their exact fp16 values; y is multiplied by x_scale[m * x_scale_stride] in fp32 before
  // the bias (stride 1: per-token scales, 0: one static scale).
  const uint8_t* x8;
  const float* x_scale;
  int x_scale_stride;
  const int32_t* qw;
  const __half* scales;
  const int32_t* qzeros;
  const __half* bias;
  __half* y;
  int64_t ldy;
  float* partial;  // [split_k / cluster, M, N] fp32 when more than one cluster splits K
  int M, N, K;
  int group_shift;  // log2(group size)
  int bps;          // 128-wide K blocks per CTA
  int cluster;      // CTAs per cluster along the K split (1, 2, 4 or 8)
  int xs_stride;    // fp16 elements per staged activation row
  // Row-parallel all-reduce through peer mailboxes (peer_world > 1; see peer_exchange).
  int peer_rank, peer_world;
  int peer_max_m, peer_max_n;
  int peer_participants;                  // storing warps of the grid (one per 32-row tile)
  uint32_t* peer_ctl;                     // own mailbox header: call counter, arrivals, error
  uint64_t* peer_data[TF_MAX_PEERS];       // rank q's tagged partials [2][world][max_m][max_n]
  uint64_t* peer_trace;  // optional: per storing warp {entry, stored, arrived, done} globaltimer ns
  // Fused RMSNorm + FP8 prologue (kernels instantiated with kNorm): x is the un-normalised fp16
  // input, norm_w the RMSNorm weight [K]; every CTA covers the whole row.
  const __half* norm_w;
  float norm_eps;
  const float* norm_static;  // static per-tensor scale, or null for the dynamic per-token one
  float* norm_scale_out;     // per-token scales [M] (dynamic case; written by CTA 0), or null
};


__device__ __forceinline__ void gload(GSlot& s, int bb, const GemvParams& p, const GLane& L) {
  if (bb >= L.b_end) return;  // warp-uniform: the slot is never consumed
  const int k = bb * kKB + 32 * L.c;
  const int g = k >> p.group_shift;
  if ((bb + 1) * kKB <= p.K) {
#pragma unroll
    for (int j = 0; j < 4; ++j) s.w[j] = ldg_stream_v4(L.w[j] + bb * (kKB / 8));
    s.s = __ldg(L.s + g * (p.N >> 2));
    s.z = static_cast<uint32_t>(__ldg(L.z + g * (p.N >> 3)));
  } else {  // partial last block: a chunk past K reads as zero weights, scale 0, zero point 0
    const bool in = k < p.K;
#pragma unroll
    for (int j = 0; j < 4; ++j) s.w[j] = in ? ldg_stream_v4(L.w[j] + bb * (kKB / 8)) : zero4();
    s.s = in ? __ldg(L.s + g * (p.N >> 2)) : make_uint2(0u, 0u);
    s.z = in ? static_cast<uint32_t>(__ldg(L.z + g * (p.N >> 3))) : 0u;
  }
}

// Group size 128: block bb is group bb and K % 128 == 0, so every block is whole.
__device__ __forceinline__ void gload_grp(GSlot& s, int bb, const GemvParams& p, const GLane& L) {
  if (bb >= L.b_end) return;  // warp-uniform: the slot is never consumed
#pragma unroll
  for (int j = 0; j < 4; ++j) s.w[j] = ldg_stream_v4(L.w[j] + bb * (kKB / 8));
  s.s = __ldg(L.s + bb * (p.N >> 2));
  s.z = static_cast<uint32_t>(__ldg(L.z + bb * (p.N >> 3)));
}


__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t ld_volatile_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

constexpr uint64_t kPeerWaitNs = 2000000000ull;  // give up on a silent peer after 2 s

// Row-parallel all-reduce of one 32-row tile, run by the warp that holds the tile's final fp32
// partial (v, fragment layout as in the store below; bias is passed on one rank only). Every
// value travels as one 64-bit word (fp32 bits | call tag << 32) written with a single store into
// slot [parity][me] of each peer's mailbox, so a reader that sees the tag also sees the value
// (64-bit aligned stores are single-copy atomic): no fences or separate flags. Each lane then
// polls its own values from every peer (bounded wait), sums the ranks' partials in rank order
// (its own from registers), so all ranks write identical y, and the last storing warp of the
// grid advances the call counter. Calls alternate between two parities; a rank cannot get two
// calls ahead of a peer's reads, because finishing a call needs that peer's values of the call,
// which the peer writes only after its previous call (and its reads) ended. Tags are call + 1.
__device__ __forceinline__ void peer_exchange(const GemvParams& p, const float (&v)[2][4], int rr,
                                              int c, int lane, uint32_t call) {
  const uint64_t t_entry = p.peer_trace != nullptr ? globaltimer_ns() : 0;
  const int W = p.peer_world, me = p.peer_rank;
  const int par = static_cast<int>(call & 1u);
  const uint32_t tag = call + 1u;
  const size_t slot = static_cast<size_t>(p.peer_max_m) * p.peer_max_n;
  float own[2][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int n = rr + 2 * t + (r >> 1), m = 2 * c + (r & 1);
      own[t][r] = v[t][r];
      if (n < p.N && m < p.M && p.bias) own[t][r] += __half2float(__ldg(p.bias + n));
    }
  for (int q = 0; q < W; ++q) {
    if (q == me) continue;
    uint64_t* d = p.peer_data[q] + (static_cast<size_t>(par) * W + me) * slot;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int n = rr + 2 * t + (r >> 1), m = 2 * c + (r & 1);
        if (n < p.N && m < p.M)
          st_volatile_u64(d + static_cast<size_t>(m) * p.peer_max_n + n,
                          (static_cast<uint64_t>(tag) << 32) | __float_as_uint(own[t][r]));
      }
  }
  // Sum in rank order. Words are requested in batches of independent loads (all of the lane's
  // words of the one peer when world == 2; else, per tile, the words of all peers), so a batch
  // costs one round trip; only words whose tag is not yet the call's are polled again.
  const uint64_t t_stored = p.peer_trace != nullptr ? globaltimer_ns() : 0;
  const uint64_t* mine = p.peer_data[me] + static_cast<size_t>(par) * W * slot;
  bool timed_out = false;
  const uint64_t t0 = globaltimer_ns();
  size_t off[2][4];
  bool live[2][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int n = rr + 2 * t + (r >> 1), m = 2 * c + (r & 1);
      live[t][r] = n < p.N && m < p.M;
      off[t][r] = static_cast<size_t>(m) * p.peer_max_n + n;
    }
  auto poll = [&](uint64_t& w, const uint64_t* src) {
    if (static_cast<uint32_t>(w >> 32) != tag) {
      w = ld_volatile_u64(src);
      return true;
    }
    return false;
  };
  float sum[2][4];
  if (W == 2) {
    const int q = 1 - me;
    uint64_t w[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r)
        w[t][r] = live[t][r] ? ld_volatile_u64(mine + q * slot + off[t][r])
                             : (static_cast<uint64_t>(tag) << 32);
    while (true) {
      bool pending = false;
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int r = 0; r < 4; ++r) pending |= poll(w[t][r], mine + q * slot + off[t][r]);
      if (!pending || timed_out) break;
      if (globaltimer_ns() - t0 > kPeerWaitNs) timed_out = true;
    }
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float other = __uint_as_float(static_cast<uint32_t>(w[t][r]));
        sum[t][r] = me == 0 ? own[t][r] + other : other + own[t][r];
      }
  } else {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      uint64_t w[TF_MAX_PEERS][4];
#pragma unroll
      for (int q = 0; q < TF_MAX_PEERS; ++q)
#pragma unroll
        for (int r = 0; r < 4; ++r)
          w[q][r] = (q < W && q != me && live[t][r])
                        ? ld_volatile_u64(mine + q * slot + off[t][r])
                        : (static_cast<uint64_t>(tag) << 32);
      while (true) {
        bool pending = false;
#pragma unroll
        for (int q = 0; q < TF_MAX_PEERS; ++q)
#pragma unroll
          for (int r = 0; r < 4; ++r) pending |= poll(w[q][r], mine + q * slot + off[t][r]);
        if (!pending || timed_out) break;
        if (globaltimer_ns() - t0 > kPeerWaitNs) timed_out = true;
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < TF_MAX_PEERS; ++q) {
          if (q >= W) break;
          acc += (q == me) ? own[t][r] : __uint_as_float(static_cast<uint32_t>(w[q][r]));
        }
        sum[t][r] = acc;
      }
    }
  }
  uint64_t t_arrived = 0;
  if (p.peer_trace != nullptr) {
    __syncwarp();
    t_arrived = globaltimer_ns();
  }
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int n = rr + 2 * t + (r >> 1), m = 2 * c + (r & 1);
      if (live[t][r]) p.y[m * p.ldy + n] = __float2half_rn(sum[t][r]);
    }
  if (p.peer_trace != nullptr) {
    __syncwarp();
    if (lane == 0) {
      uint64_t* rec = p.peer_trace + 4 * static_cast<size_t>(rr / kWarpRows);
      rec[0] = t_entry;
      rec[1] = t_stored;
      rec[2] = t_arrived;
      rec[3] = globaltimer_ns();
    }
  }
  if (timed_out) atomicCAS(p.peer_ctl + 2, 0u, 1u);
  __syncwarp();
  if (lane == 0) {
    __threadfence();
    if (atomicAdd(p.peer_ctl + 1, 1u) == static_cast<uint32_t>(p.peer_participants - 1)) {
      atomicExch(p.peer_ctl + 1, 0u);
      __threadfence();
      atomicAdd(p.peer_ctl, 1u);
    }
  }
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Stages x[0:M, kb0*128 : kb1*128] (zero past K) in shared memory, rows xs_stride apart: every
// 16-byte piece is an asynchronous copy, all in flight together, so staging costs one L2 round
// trip (e4m3 codes are converted to their exact fp16 values on the way). Returns once this
// thread's copies have landed; the caller synchronises the CTA.
__device__ __forceinline__ void stage_activations(const GemvParams& p, uint4* xs_smem, int kb0,
                                                  int kb1) {
  {
    const int vec_per_row = (kb1 - kb0) * (kKB / 8);
    const int total = p.M * vec_per_row;
    const int k_lo = kb0 * kKB;
    if (p.x8 != nullptr) {
      // e4m3 codes: 8 bytes per 16-byte fp16 vector, converted exactly (every e4m3 value is an
      // fp16 value; NaN stays NaN). Two loads per thread are in flight before the stores.
      for (int i0 = threadIdx.x; i0 < total; i0 += 2 * blockDim.x) {
        uint2 raw[2];
        int idx[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = i0 + u * static_cast<int>(blockDim.x);
          idx[u] = i;
          raw[u] = make_uint2(0u, 0u);
          if (i < total) {
            const int m = i / vec_per_row, v = i - m * vec_per_row;
            const int k = k_lo + 8 * v;
            if (k < p.K) raw[u] = __ldg(reinterpret_cast<const uint2*>(p.x8 + m * p.ldx + k));
          }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = idx[u];
          if (i >= total) continue;
          const int m = i / vec_per_row, v = i - m * vec_per_row;
          const uint32_t w[2] = {raw[u].x, raw[u].y};
          uint32_t h[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint16_t pair = static_cast<uint16_t>(w[e >> 1] >> (16 * (e & 1)));
            asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h[e]) : "h"(pair));
          }
          xs_smem[(m * p.xs_stride) / 8 + v] = make_uint4(h[0], h[1], h[2], h[3]);
        }
      }
    } else
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int m = i / vec_per_row, v = i - m * vec_per_row;
      const int k = k_lo + 8 * v;
      uint4* dst = xs_smem + (m * p.xs_stride) / 8 + v;
      if (k < p.K) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                     "l"(p.x + m * p.ldx + k)
                     : "memory");
      } else {
        *dst = zero4();
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
}

// Fused SiLU prologue: x is the gate_up output [M, 2K] (row stride ldx), and the staged
// activations of the CTA's K range are fp16(silu(g) * u) with g = x[m, k], u = x[m, K + k],
// computed as the standalone silu_mul kernel computes them (silu_mul_f32), so y is
// bit-identical to silu_mul followed by this GEMV. Elementwise: every plan shape could use it.
__device__ __forceinline__ void stage_silu(const GemvParams& p, uint4* xs_smem, int kb0, int kb1) {
  const int vec_per_row = (kb1 - kb0) * (kKB / 8);
  const int total = p.M * vec_per_row;
  const int k_lo = kb0 * kKB;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int m = i / vec_per_row, v = i - m * vec_per_row;
    const int k = k_lo + 8 * v;
    uint4 out = zero4();
    if (k < p.K) {
      const __half* row = p.x + m * p.ldx;
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(row + k));
      const uint4 uv = __ldg(reinterpret_cast<const uint4*>(row + p.K + k));
      const __half2* g2 = reinterpret_cast<const __half2*>(&gv);
      const __half2* u2 = reinterpret_cast<const __half2*>(&uv);
      __half2* o2 = reinterpret_cast<__half2*>(&out);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 gf = __half22float2(g2[e]), uf = __half22float2(u2[e]);
        o2[e] = __floats2half2_rn(silu_mul_f32(gf.x, uf.x), silu_mul_f32(gf.y, uf.y));
      }
    }
    xs_smem[(m * p.xs_stride) / 8 + v] = out;
  }
}

// Replaces the staged -y values of one row by the fp16 values of their e4m3 codes.
template <int kPath>
__device__ __forceinline__ void quant_staged(uint4* row, int nvec, int tid, int nt, const Fp8Div& d) {
  for (int j = tid; j < nvec; j += nt) {
    const uint2 c = quant_vec<kPath>(row[j], d);
    uint4 v;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(v.x) : "h"(static_cast<uint16_t>(c.x)));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(v.y) : "h"(static_cast<uint16_t>(c.x >> 16)));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(v.z) : "h"(static_cast<uint16_t>(c.y)));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(v.w) : "h"(static_cast<uint16_t>(c.y >> 16)));
    row[j] = v;
  }
}

// Fused RMSNorm + FP8 prologue on the staged rows (the CTA holds all K of each of the M rows):
// the rule of rmsnorm_fp8_quant (tf_rmsnorm.cuh) applied in shared memory. Pass 1 sums the
// squares in fp64, pass 2 writes -y = -(fp16(x * rstd) * weight) in place and takes amax|y|,
// pass 3 replaces it by the exact fp16 value of y's e4m3 code e4m3(y / scale). The GEMV then runs
// exactly as on rmsnorm_fp8_quant's (codes, scale) and multiplies y by scale[m] in fp32, so its
// output is bit-identical to the two-kernel path. red: >= 3 * 8 * warps floats of scratch.
__device__ __forceinline__ void norm_quant_staged(const GemvParams& p, uint4* xs, float* red,
                                               float* scale_sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = static_cast<int>(blockDim.x) >> 5, nt = static_cast<int>(blockDim.x);
  const int nvec = p.K / 8;
  double* sh_sum = reinterpret_cast<double*>(red);  // [M][nw]
  float* sh_max = red + 2 * 8 * nw;                 // [M][nw]
  const uint4* wv = reinterpret_cast<const uint4*>(p.norm_w);
  for (int m = 0; m < p.M; ++m) {
    const uint4* row = xs + (m * p.xs_stride) / 8;
    double s = 0.0;
    for (int j = tid; j < nvec; j += nt) acc_sumsq(row[j], s);
    s = warp_sum(s);
    if (lane == 0) sh_sum[m * nw + warp] = s;
  }
  __syncthreads();
  // Pass 2 leaves -y in the staging buffer (the form quant_vec divides); pass 3 replaces it by
  // the fp16 value of y's e4m3 code, on the FMA division path when the row's |y| are finite.
  for (int m = 0; m < p.M; ++m) {
    double tot = 0.0;
    for (int w = 0; w < nw; ++w) tot += sh_sum[m * nw + w];
    const float rstd = rstd_of(tot, p.K, p.norm_eps);
    const uint64_t rstd2 = f32x2(rstd, rstd);
    uint4* row = xs + (m * p.xs_stride) / 8;
    __half2 a2 = __float2half2_rn(0.f);
    for (int j = tid; j < nvec; j += nt)
      row[j] = norm_vec_neg(row[j], neg_weight(__ldg(wv + j)), rstd2, a2);
    const float amax = warp_max(amax_of(a2));
    if (lane == 0) sh_max[m * nw + warp] = amax;
  }
  __syncthreads();
  for (int m = 0; m < p.M; ++m) {
    float mx = 0.f;
    for (int w = 0; w < nw; ++w) mx = fmaxf(mx, sh_max[m * nw + w]);
    float scale;
    if (p.norm_static != nullptr) {
      scale = __ldg(p.norm_static);
    } else {
      scale = dyn_scale(mx);
      if (tid == 0 && p.norm_scale_out != nullptr && blockIdx.x == 0 && blockIdx.y == 0)
        p.norm_scale_out[m] = scale;
    }
    if (tid == 0) scale_sh[m] = scale;
    const Fp8Div d = fp8_div(scale);
    const int path = quant_path(d, mx <= 65504.f, p.norm_static == nullptr);
    uint4* row = xs + (m * p.xs_stride) / 8;
    if (path == kFma1) quant_staged<kFma1>(row, nvec, tid, nt, d);
    else if (path == kFma2) quant_staged<kFma2>(row, nvec, tid, nt, d);
    else quant_staged<kIeee>(row, nvec, tid, nt, d);
  }
  __syncthreads();
}

template <int WARPS_N, int WARPS_K, bool kCluster, bool kFact, bool kNorm = false,
          bool kSilu = false>
__global__ void __launch_bounds__(32 * WARPS_N * WARPS_K, kWideWarps / (WARPS_N * WARPS_K))
    w4a16_gemv_kernel(const GemvParams p) {
  constexpr int kWarps = WARPS_N * WARPS_K;
  static_assert(kWarps == kCtaWarps || kWarps == kWideWarps, "CTA shape");
  extern __shared__ uint4 xs_smem[];
  // Per warp: two tiles x four fragment values x 32 lanes.
  __shared__ float red[kWarps * 2 * 4 * 32];
  __shared__ float norm_scale_sh[kNorm ? 8 : 1];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn = warp / WARPS_K, wk = warp % WARPS_K;
  const int q = lane >> 2;
  GLane L;
  L.c = lane & 3;
  const int n0 = (blockIdx.x * WARPS_N + wn) * kWarpRows;
  const int rr = n0 + 4 * q;                // first of the lane's rows (as stored)
  const int r0 = min(rr, p.N - 4);          // N % 8 == 0: rows r0..r0+3 are all valid
  const int nblk = (p.K + kKB - 1) / kKB;
  L.kb0 = blockIdx.y * p.bps;
  const int kb1 = min(nblk, L.kb0 + p.bps);
  // Warp wk of a row group takes a contiguous share of the CTA's K blocks.
  const int share = (kb1 - L.kb0 + WARPS_K - 1) / WARPS_K;
  const int b0 = L.kb0 + wk * share;
  L.b_end = min(kb1, b0 + share);
  const int ldw = p.K / 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) L.w[j] = p.qw + (r0 + j) * ldw + 4 * L.c;
  L.s = reinterpret_cast<const uint2*>(p.scales + r0);
  L.z = p.qzeros + (r0 >> 3);
#pragma unroll
  for (int j = 0; j < 4; ++j) L.nib[j] = 4 * awq_nibble_of((r0 + j) & 7);
  const int xq = min(q, p.M - 1);
  L.xs = xs_smem + (xq * p.xs_stride + 32 * L.c) / 8;
  const uint32_t mask = 0x000F000Fu, magic = 0x64006400u;

  // Weights, scales and zero points never depend on the preceding kernel: the register loads of
  // the first two blocks are issued before the programmatic-dependent-launch wait.
  GSlot s0, s1;
  auto load = [&](GSlot& sl, int b) {
    if constexpr (kFact) gload_grp(sl, b, p, L);
    else gload(sl, b, p, L);
  };
  load(s0, b0);
  load(s1, b0 + 1);
  // The next kernel on the stream may be scheduled once every CTA of this grid has passed this
  // point (so all of them are running or done): its CTAs take SM slots as ours retire and issue
  // their own weight loads early, and its griddepcontrol.wait still waits for this grid to end.
  pdl_launch_dependents();
  pdl_wait();
  // The peer call counter is read after the wait: the previous call on this stream has ended.
  const uint32_t call = p.peer_world > 1 ? *reinterpret_cast<volatile uint32_t*>(p.peer_ctl) : 0u;

  if constexpr (kSilu)
    stage_silu(p, xs_smem, L.kb0, kb1);
  else
    stage_activations(p, xs_smem, L.kb0, kb1);
  __syncthreads();
  if constexpr (kNorm) norm_quant_staged(p, xs_smem, red, norm_scale_sh);

  // Group size 128 (kFact): the scale and zero point are loaded once per block and every weight
  // is dequantized as the reference does (gcompute_w16); other group sizes look up the group of
  // every word (gcompute). Both sum x * fp16((q - z) * s) on the tensor core in fp32.
  float acc[2][2][4] = {};
  auto step = [&](const GSlot& sl, int b) {
    if constexpr (kFact) gcompute_w16(acc, sl, b, L);
    else gcompute(acc, sl, b, L, mask, magic);
  };
  for (int b = b0; b < L.b_end; b += 2) {
    step(s0, b);
    load(s0, b + 2);
    if (b + 1 >= L.b_end) break;
    step(s1, b + 1);
    load(s1, b + 3);
  }

  // Fixed-order reductions: the accumulator chains, then the WARPS_K warps (warp order), then the
  // CTAs of the cluster (rank order).
  float* mine = red + warp * (2 * 4 * 32);
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int r = 0; r < 4; ++r) mine[(t * 4 + r) * 32 + lane] = acc[t][0][r] + acc[t][1][r];
  __syncthreads();
  float v[2][4];
  if (wk == 0) {
    const float* base = red + (wn * WARPS_K) * (2 * 4 * 32);
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS_K; ++w) a += base[w * (2 * 4 * 32) + (t * 4 + r) * 32 + lane];
        v[t][r] = a;
      }
  }
  bool store = wk == 0;
  if constexpr (kCluster) {
    __syncthreads();
    if (wk == 0) {
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int r = 0; r < 4; ++r) mine[(t * 4 + r) * 32 + lane] = v[t][r];
    }
    cluster_sync();  // every rank's CTA partial is in its shared memory
    const uint32_t rank = cluster_rank();
    if (rank == 0 && wk == 0) {
      for (int cr = 1; cr < p.cluster; ++cr)
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int r = 0; r < 4; ++r) v[t][r] += ld_cluster_f32(mine + (t * 4 + r) * 32 + lane, cr);
    }
    cluster_sync();  // rank 0 has read the others' shared memory; they may exit
    store = store && rank == 0;
  }
  if (!store) return;

  if (kNorm || p.x_scale != nullptr) {  // FP8 activations: the per-token scale, before the bias
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int m = min(2 * L.c + (r & 1), p.M - 1);
        v[t][r] *= kNorm ? norm_scale_sh[m] : __ldg(p.x_scale + m * p.x_scale_stride);
      }
  }
  // Fragment value r of tile t: row 4q + 2t (r < 2) or 4q + 2t + 1 (r >= 2), token 2c + (r & 1).
  const int split = static_cast<int>(blockIdx.y) / p.cluster;
  const bool direct = static_cast<int>(gridDim.y) == p.cluster;
  if (p.peer_world > 1) {  // the host admits peers only for direct plans
    peer_exchange(p, v, rr, L.c, lane, call);
    return;
  }
#pragma unroll
  for (int t = 0; t < 2; ++t) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int n = rr + 2 * t + (r >> 1);
      const int m = 2 * L.c + (r & 1);
      if (n >= p.N || m >= p.M) continue;
      if (direct) {
        float o = v[t][r];
        if (p.bias) o += __half2float(__ldg(p.bias + n));
        p.y[m * p.ldy + n] = __float2half_rn(o);
      } else {
        p.partial[(static_cast<int64_t>(split) * p.M + m) * p.N + n] = v[t][r];
      }
    }
  }
}

// ---------------------------------------------------------------- 16-token decode GEMV
// M = 9..16 with group size 128: the M <= 8 kernel's weight streaming and per-weight dequant,
// with every dequantized block fed to two 8-token MMA n-tiles (tokens 0-7 and 8-15), so the
// dequant work of a weight is shared by sixteen tokens instead of eight. The accumulators of both
// n-tiles double the per-thread state, so this kernel runs 8-warp CTAs at two per SM with the
// register budget that allows; the K split (warps, cluster DSMEM, cross-cluster partials) and
// every sum order are the M <= 8 kernel's.
__device__ __forceinline__ void gcompute_w16_2(float (&a0)[2][4], float (&a1)[2][4], const GSlot& s,
                                               int bb, const GLane& L, const uint4* xs1) {
  uint32_t z0[4], z1[4], sc[4];
  zero_points(z0, z1, s.z, L.nib[0]);
  scale_pairs(sc, s);
  const uint4* xp0 = L.xs + (bb - L.kb0) * (kKB / 8);
  const uint4* xp1 = xs1 + (bb - L.kb0) * (kKB / 8);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 xv0 = xp0[i], xv1 = xp1[i];
    const uint32_t w[4] = {(&s.w[0].x)[i], (&s.w[1].x)[i], (&s.w[2].x)[i], (&s.w[3].x)[i]};
    W16Frag f;
    dequant_word(f, w, z0, z1, sc);
    mma_16816(a0[0], f.t0a, xv0.x, xv0.y);
    mma_16816(a0[1], f.t1a, xv0.x, xv0.y);
    mma_16816(a1[0], f.t0a, xv1.x, xv1.y);
    mma_16816(a1[1], f.t1a, xv1.x, xv1.y);
    mma_16816(a0[0], f.t0b, xv0.z, xv0.w);
    mma_16816(a0[1], f.t1b, xv0.z, xv0.w);
    mma_16816(a1[0], f.t0b, xv1.z, xv1.w);
    mma_16816(a1[1], f.t1b, xv1.z, xv1.w);
  }
}

template <int WARPS_N, int WARPS_K, bool kCluster>
__global__ void __launch_bounds__(32 * WARPS_N * WARPS_K, 2) w4a16_gemv16_kernel(const GemvParams p) {
  constexpr int kWarps = WARPS_N * WARPS_K;
  static_assert(kWarps == kCtaWarps, "CTA shape");
  extern __shared__ uint4 xs_smem[];
  __shared__ float red[kWarps * 2 * 8 * 32];  // per warp: two n-tiles x eight values x 32 lanes

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn = warp / WARPS_K, wk = warp % WARPS_K;
  const int q = lane >> 2;
  GLane L;
  L.c = lane & 3;
  const int n0 = (blockIdx.x * WARPS_N + wn) * kWarpRows;
  const int rr = n0 + 4 * q;
  const int r0 = min(rr, p.N - 4);
  const int nblk = (p.K + kKB - 1) / kKB;
  L.kb0 = blockIdx.y * p.bps;
  const int kb1 = min(nblk, L.kb0 + p.bps);
  const int share = (kb1 - L.kb0 + WARPS_K - 1) / WARPS_K;
  const int b0 = L.kb0 + wk * share;
  L.b_end = min(kb1, b0 + share);
  const int ldw = p.K / 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) L.w[j] = p.qw + (r0 + j) * ldw + 4 * L.c;
  L.s = reinterpret_cast<const uint2*>(p.scales + r0);
  L.z = p.qzeros + (r0 >> 3);
#pragma unroll
  for (int j = 0; j < 4; ++j) L.nib[j] = 4 * awq_nibble_of((r0 + j) & 7);
  L.xs = xs_smem + (min(q, p.M - 1) * p.xs_stride + 32 * L.c) / 8;
  const uint4* xs1 = xs_smem + (min(q + 8, p.M - 1) * p.xs_stride + 32 * L.c) / 8;

  GSlot s0, s1;
  gload_grp(s0, b0, p, L);
  gload_grp(s1, b0 + 1, p, L);
  pdl_launch_dependents();
  pdl_wait();
  stage_activations(p, xs_smem, L.kb0, kb1);
  __syncthreads();

  float y[2][2][4] = {};  // [n-tile][row tile][value]: x * fp16((q - z) * s) summed in fp32
  for (int b = b0; b < L.b_end; b += 2) {
    gcompute_w16_2(y[0], y[1], s0, b, L, xs1);
    gload_grp(s0, b + 2, p, L);
    if (b + 1 >= L.b_end) break;
    gcompute_w16_2(y[0], y[1], s1, b + 1, L, xs1);
    gload_grp(s1, b + 3, p, L);
  }

  // Fixed-order reductions: the WARPS_K warps (warp order), then the cluster's CTAs (rank order).
  float* mine = red + warp * (2 * 8 * 32);
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) mine[(nt * 8 + t * 4 + r) * 32 + lane] = y[nt][t][r];
  __syncthreads();
  float v[2][2][4];
  if (wk == 0) {
    const float* base = red + (wn * WARPS_K) * (2 * 8 * 32);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float a = 0.f;
#pragma unroll
          for (int w = 0; w < WARPS_K; ++w)
            a += base[w * (2 * 8 * 32) + (nt * 8 + t * 4 + r) * 32 + lane];
          v[nt][t][r] = a;
        }
  }
  bool store = wk == 0;
  if constexpr (kCluster) {
    __syncthreads();
    if (wk == 0) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int r = 0; r < 4; ++r) mine[(nt * 8 + t * 4 + r) * 32 + lane] = v[nt][t][r];
    }
    cluster_sync();
    const uint32_t rank = cluster_rank();
    if (rank == 0 && wk == 0) {
      for (int cr = 1; cr < p.cluster; ++cr)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int r = 0; r < 4; ++r)
              v[nt][t][r] += ld_cluster_f32(mine + (nt * 8 + t * 4 + r) * 32 + lane, cr);
    }
    cluster_sync();
    store = store && rank == 0;
  }
  if (!store) return;

  const int split = static_cast<int>(blockIdx.y) / p.cluster;
  const bool direct = static_cast<int>(gridDim.y) == p.cluster;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int n = rr + 2 * t + (r >> 1);
        const int m = 8 * nt + 2 * L.c + (r & 1);
        if (n >= p.N || m >= p.M) continue;
        float o = v[nt][t][r];
        if (p.x_scale != nullptr) o *= __ldg(p.x_scale + m * p.x_scale_stride);
        if (direct) {
          if (p.bias) o += __half2float(__ldg(p.bias + n));
          p.y[m * p.ldy + n] = __float2half_rn(o);
        } else {
          p.partial[(static_cast<int64_t>(split) * p.M + m) * p.N + n] = o;
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

// One launch of a GEMV kernel over the plan's grid: raises the dynamic shared-memory limit when
// static + dynamic shared memory passes the default 48 KB, and adds the programmatic-dependent-
// launch and cluster attributes the plan asks for.
template <typename Kernel>
int launch_gemv_grid(Kernel kern, const LinearPlan& plan, const GemvParams& p, size_t smem,
                     size_t static_smem, int threads, bool cluster, cudaStream_t stream, bool pdl) {
  if (smem + static_smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) {
      last_cuda_error() = static_cast<int>(e);
      return TF_ERR_CUDA;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid_x, plan.grid_y, 1);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = static_cast<unsigned>(p.cluster);
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

template <int WN, int WK, bool kCluster, bool kFact, bool kNorm = false, bool kSilu = false>
int launch_gemv_variant(const LinearPlan& plan, const GemvParams& p, size_t smem,
                        cudaStream_t stream, bool pdl) {
  // Static shared memory: the reduction buffer, 1 KB per warp.
  constexpr size_t kStaticSmem = static_cast<size_t>(WN) * WK * 2 * 4 * 32 * sizeof(float);
  return launch_gemv_grid(w4a16_gemv_kernel<WN, WK, kCluster, kFact, kNorm, kSilu>, plan, p, smem,
                          kStaticSmem, 32 * WN * WK, kCluster, stream, pdl);
}

template <int WN, int WK, bool kCluster>
int launch_gemv16_variant(const LinearPlan& plan, const GemvParams& p, size_t smem,
                          cudaStream_t stream, bool pdl) {
  constexpr size_t kStaticSmem = static_cast<size_t>(WN) * WK * 2 * 8 * 32 * sizeof(float);
  return launch_gemv_grid(w4a16_gemv16_kernel<WN, WK, kCluster>, plan, p, smem, kStaticSmem,
                          32 * WN * WK, kCluster, stream, pdl);
}

template <bool kCluster>
int launch_gemv16_shape(const LinearPlan& plan, const GemvParams& p, size_t smem, cudaStream_t st,
                        bool pdl) {
  switch (plan.warps_k) {
    case 1: return launch_gemv16_variant<8, 1, kCluster>(plan, p, smem, st, pdl);
    case 2: return launch_gemv16_variant<4, 2, kCluster>(plan, p, smem, st, pdl);
    case 4: return launch_gemv16_variant<2, 4, kCluster>(plan, p, smem, st, pdl);
    case 8: return launch_gemv16_variant<1, 8, kCluster>(plan, p, smem, st, pdl);
    default: return TF_ERR_INVALID_ARG;
  }
}

template <bool kCluster, bool kFact, bool kNorm = false, bool kSilu = false>
int launch_gemv_shape(const LinearPlan& plan, const GemvParams& p, size_t smem, cudaStream_t st,
                      bool pdl) {
  switch (plan.warps_k) {
    case 1: return launch_gemv_variant<8, 1, kCluster, kFact, kNorm, kSilu>(plan, p, smem, st, pdl);
    case 2: return launch_gemv_variant<4, 2, kCluster, kFact, kNorm, kSilu>(plan, p, smem, st, pdl);
    case 4: return launch_gemv_variant<2, 4, kCluster, kFact, kNorm, kSilu>(plan, p, smem, st, pdl);
    case 8: return launch_gemv_variant<1, 8, kCluster, kFact, kNorm, kSilu>(plan, p, smem, st, pdl);
    case 16:
      if constexpr (kCluster) return TF_ERR_INVALID_ARG;
      else return launch_gemv_variant<1, 16, false, kFact, kNorm, kSilu>(plan, p, smem, st, pdl);
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
  p.x8 = a.x8;
  p.x_scale = a.x_scale;
  p.x_scale_stride = static_cast<int>(a.x_scale_stride);
  p.qw = a.qw;
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.qzeros = a.qzeros;
  p.bias = reinterpret_cast<const __half*>(a.bias);
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.group_shift = a.group_size == 32 ? 5 : (a.group_size == 64 ? 6 : 7);
  p.bps = plan.blocks_per_split;
  p.cluster = plan.cluster;
  p.xs_stride = plan.blocks_per_split * kKB + 8;
  const int outer = plan.split_k / plan.cluster;  // splits reduced by the second kernel
  p.partial = outer > 1 ? static_cast<float*>(a.workspace) : nullptr;
  p.peer_world = 0;
  p.peer_rank = 0;
  p.peer_ctl = nullptr;
  p.peer_trace = nullptr;
  p.norm_w = reinterpret_cast<const __half*>(a.norm_w);
  p.norm_eps = a.norm_eps;
  p.norm_static = a.norm_static;
  p.norm_scale_out = a.norm_scale_out;
  if (a.peers != nullptr) {
    const TfPeerSet& ps = *a.peers;
    const PeerLayout lay = peer_layout(ps.world, ps.max_m, ps.max_n);
    p.peer_world = ps.world;
    p.peer_rank = ps.rank;
    p.peer_max_m = ps.max_m;
    p.peer_max_n = ps.max_n;
    p.peer_participants = static_cast<int>(plan.grid_x) * gemv_warps_n(plan.warps_k);
    p.peer_ctl = static_cast<uint32_t*>(ps.mailbox[ps.rank]);
    p.peer_trace = g_peer_trace.load();
    for (int q = 0; q < TF_MAX_PEERS; ++q) {
      char* base = q < ps.world ? static_cast<char*>(ps.mailbox[q]) : nullptr;
      p.peer_data[q] = base ? reinterpret_cast<uint64_t*>(base + lay.data_off) : nullptr;
    }
  }
  const size_t smem = gemv_smem_bytes(a.M, plan.blocks_per_split);
  const bool pdl = (launch_flags() & TF_LAUNCH_PDL) != 0;
  // Group size 128 (one K block per group): the scale is applied once per block after the
  // tensor-core sums; other group sizes dequantize every weight.
  const bool fact = a.group_size == kKB;
  int st;
  if (a.M > 8) {
    // 16-token kernel: group size 128, no peers, no fused RMSNorm (checked by the planner).
    if (!fact || a.peers != nullptr || a.norm_w != nullptr || a.M > 16) return TF_ERR_UNSUPPORTED;
    st = plan.cluster > 1 ? launch_gemv16_shape<true>(plan, p, smem, stream, pdl)
                          : launch_gemv16_shape<false>(plan, p, smem, stream, pdl);
    if (st != TF_OK || outer == 1) return st;
    return launch_splitk_reduce(p.partial, outer, a.M, a.N, a.bias, a.y, a.ldy, stream);
  }
  if (a.silu) {
    // The fused SiLU product: single-pass plans (checked by the caller).
    if (plan.cluster != 1 || plan.split_k != 1 || a.peers != nullptr || a.norm_w != nullptr)
      return TF_ERR_UNSUPPORTED;
    return fact ? launch_gemv_shape<false, true, false, true>(plan, p, smem, stream, pdl)
                : launch_gemv_shape<false, false, false, true>(plan, p, smem, stream, pdl);
  }
  if (a.norm_w != nullptr) {
    // The fused RMSNorm needs every CTA to hold whole rows (checked by the caller).
    if (plan.cluster != 1 || plan.split_k != 1 || a.peers != nullptr) return TF_ERR_UNSUPPORTED;
    return fact ? launch_gemv_shape<false, true, true>(plan, p, smem, stream, pdl)
                : launch_gemv_shape<false, false, true>(plan, p, smem, stream, pdl);
  }
  if (plan.cluster > 1)
    st = fact ? launch_gemv_shape<true, true>(plan, p, smem, stream, pdl)
              : launch_gemv_shape<true, false>(plan, p, smem, stream, pdl);
  else
    st = fact ? launch_gemv_shape<false, true>(plan, p, smem, stream, pdl)
              : launch_gemv_shape<false, false>(plan, p, smem, stream, pdl);
  if (st != TF_OK || outer == 1) return st;
  return launch_splitk_reduce(p.partial, outer, a.M, a.N, a.bias, a.y, a.ldy, stream);
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

// Peer-exchange tracing of the fused all-reduce GEMV (see the header): later launches of
// tf_w4a16_linear_allreduce in this process stamp `records` (device memory, 4 uint64 per 32-row
// tile of the layer, indexed by tile), or nothing when it is null.
extern "C" int tf_peer_trace(uint64_t* records) {
  tfb::g_peer_trace.store(records);
  return TF_OK;
}
