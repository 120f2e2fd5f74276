// W4A16 GEMM on the sm_100a tensor cores: TMA + in-shared-memory dequant + tcgen05.mma into
// TMEM. Prefill sizes (M >= 9) of y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]).
//
// Reference semantics: tokenforge/kernels/triton/w4a16.py:44-115 (dequant with one fp16
// rounding, fp16 x fp16 products accumulated in fp32, fp32 bias, fp16 output) and the split-K
// contract of w4a16.py:193-200,227-232 (fp32 partials reduced in split order).
//
// The product is computed transposed, D[n, m] = W[n, :] . x[m, :]: the dequantized weights
// are the MMA's A operand (M = 128 weight rows) and the activations its B operand
// (N = BM tokens, 16..256), so one dequantized weight tile serves BM tokens and small M wastes
// no tensor-core rows. Both operands are K-major with the 128-byte swizzle.
//
// CTA = 12 warps, persistent over (n-tile, m-tile, k-split) work units:
//   warp 0      TMA producer: per 64-wide K block, the x tile [BM x 64] fp16 (128B swizzle),
//               the packed weight tile [128 x 8] int32, and the scale / zero-point rows of the
//               block's group(s), into a ring of shared-memory stages;
//   warp 1      TMEM allocator and MMA issuer: one thread issues 4 x tcgen05.mma (K = 16 each)
//               per stage into a TMEM accumulator [128 lanes x BM columns] fp32, double buffered
//               across work units, and commits stage release / accumulator-ready barriers;
//   warps 4-7   epilogue: tcgen05.ld of the accumulator (warp w owns TMEM lanes 32(w%4)..),
//               bias, fp16 conversion and stores (or fp32 split-K partials);
//   warps 8-11  dequant: thread t turns row t of the packed tile into a 128-byte row of fp16
//               (LOP3 + 0x6400 magic, HSUB2 zero point, HMUL2 scale: bit-exact dequant) and
//               stores it at the swizzled position the MMA descriptor expects.
// Every mbarrier wait is bounded (2 s); on timeout the kernel records an error code in a device
// status word, stops issuing work, waits (bounded) for its own copies and MMAs, frees its TMEM
// and returns. No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "tf_common.cuh"
#include "tf_plan.h"

namespace tfb {

__device__ int g_device_error = 0;

namespace {

constexpr int kBlockN = 128;  // weight rows per tile = MMA M
constexpr int kBlockK = 64;   // K per stage: one 128-byte swizzle row of fp16
constexpr int kThreads = 384;
constexpr int kProducerWarp = 0, kMmaWarp = 1, kEpiWarp0 = 4, kDeqWarp0 = 8;
constexpr int kSmemLimit = 227 * 1024;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

enum WaitSite : int {
  kErrProducerEmpty = 0x101,
  kErrDeqFull = 0x102,
  kErrMmaAccEmpty = 0x103,
  kErrMmaDeq = 0x104,
  kErrMmaFull = 0x105,
  kErrEpiAccFull = 0x106,
  kErrDrain = 0x107,
};

template <int BM>
struct TcLayout {
  static constexpr int kXBytes = BM * 128;         // [BM x 64] fp16
  static constexpr int kABytes = kBlockN * 128;    // [128 x 64] fp16
  static constexpr int kWBytes = kBlockN * 32;     // [128 x 8] int32
  static constexpr int kSBytes = 2 * kBlockN * 2;  // up to two group rows of 128 fp16
  static constexpr int kZBytes = 2 * 16 * 4;       // up to two group rows of 16 int32
  static constexpr int kAOff = kXBytes;
  static constexpr int kWOff = kAOff + kABytes;
  static constexpr int kSOff = kWOff + kWBytes;
  static constexpr int kZOff = kSOff + kSBytes;
  static constexpr int kStageBytes = ((kZOff + kZBytes) + 1023) / 1024 * 1024;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kStagesFit = (kSmemLimit - 1024 - kBarrierBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit < 6 ? kStagesFit : 6;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarrierBytes;
  static constexpr int kTmemCols = (2 * BM < 32) ? 32 : 2 * BM;  // power of two for BM = 16..256
  static_assert(kStages >= 2, "shared memory too small for two stages");
};

struct TcParams {
  int64_t M, N, K;
  int group_size;
  int m_tiles, k_splits, kb_per_split, kb_total, units;
  uint32_t tx_bytes;
  const __half* bias;
  __half* y;
  int64_t ldy;
  float* partial;
};

// ----------------------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete. Bounded: after kWaitLimitNs (or as soon
// as another thread has recorded an error) it records `site` and returns false.
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int site) {
  const unsigned long long t0 = global_ns();
  while (true) {
    for (int i = 0; i < 128; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&g_device_error) != 0) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicCAS(&g_device_error, 0, site);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, site);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulate, issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_16cols(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile with the 128-byte swizzle: rows of 128 bytes,
// 8-row core groups 1024 bytes apart (stride byte offset), descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;          // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;          // version
  d |= static_cast<uint64_t>(2) << 61;          // SWIZZLE_128B
  return d;
}

// Instruction descriptor: fp16 A and B, fp32 D, both K-major, M = 128, N = BM.
template <int BM>
__device__ __forceinline__ constexpr uint32_t instr_desc() {
  return (1u << 4) | (static_cast<uint32_t>(BM >> 3) << 17) | (static_cast<uint32_t>(kBlockN >> 4) << 24);
}

struct Unit {
  int64_t n0;
  int m_tile, ks, kb0, kb1;
};

__device__ __forceinline__ Unit decode_unit(int u, const TcParams& p) {
  Unit w;
  w.ks = u % p.k_splits;
  const int rest = u / p.k_splits;
  const int mt = rest % p.m_tiles;
  const int nt = rest / p.m_tiles;
  w.n0 = static_cast<int64_t>(nt) * kBlockN;
  w.m_tile = mt;
  w.kb0 = w.ks * p.kb_per_split;
  w.kb1 = min(p.kb_total, w.kb0 + p.kb_per_split);
  return w;
}

template <int BM>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_s,
                    const __grid_constant__ CUtensorMap tm_z, const TcParams p) {
  using L = TcLayout<BM>;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * L::kStageBytes);
  uint64_t* deq = full + S;
  uint64_t* empty = deq + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&deq[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_s);
    prefetch_tmap(&tm_z);
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, L::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Inputs may be produced by the preceding kernel on the stream (programmatic launch).
  pdl_wait();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        const Unit w = decode_unit(u, p);
        const int m0 = w.m_tile * BM;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, kErrProducerEmpty)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * L::kStageBytes;
          const int g0 = (kb * kBlockK) / p.group_size;
          mbar_expect_tx(&full[s], p.tx_bytes);
          tma_load_2d(st, &tm_x, &full[s], kb * kBlockK, m0);
          tma_load_2d(st + L::kWOff, &tm_w, &full[s], kb * (kBlockK / 8), static_cast<int>(w.n0));
          tma_load_2d(st + L::kSOff, &tm_s, &full[s], static_cast<int>(w.n0), g0);
          tma_load_2d(st + L::kZOff, &tm_z, &full[s], static_cast<int>(w.n0 / 8), g0);
        }
      }
      // Drain: every armed stage must have landed before the CTA may exit.
      const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0;
      for (uint32_t j = first; j < it; ++j)
        if (!mbar_wait(&full[j % S], (j / S) & 1u, kErrDrain)) break;
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc<BM>();
      uint32_t it = 0, tc = 0;
      bool ok = true;
      bool issued = false;
      uint32_t last_s = 0, last_ph = 0;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++tc) {
        const Unit w = decode_unit(u, p);
        const uint32_t b = tc & 1u, aph = (tc >> 1) & 1u;
        if (!mbar_wait(&acc_empty[b], aph ^ 1u, kErrMmaAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * BM;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!mbar_wait(&deq[s], ph, kErrMmaDeq) || !mbar_wait(&full[s], ph, kErrMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = smem + s * L::kStageBytes;
          const uint64_t a_desc = sw128_desc(smem_u32(st + L::kAOff));
          const uint64_t b_desc = sw128_desc(smem_u32(st));
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk)
            umma_f16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc,
                     (kb > w.kb0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          issued = true;
          last_s = s;
          last_ph = ph;
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
      }
      // Error exit: let the MMAs already issued finish before the TMEM is released.
      if (!ok && issued) mbar_wait(&empty[last_s], last_ph, kErrDrain);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    const int q = warp - kEpiWarp0;  // TMEM lanes 32q .. 32q+31
    uint32_t tc = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++tc) {
      const Unit w = decode_unit(u, p);
      const uint32_t b = tc & 1u, aph = (tc >> 1) & 1u;
      if (!mbar_wait(&acc_full[b], aph, kErrEpiAccFull)) break;
      tc_fence_after();
      const int64_t n = w.n0 + 32 * q + lane;
      const int64_t m0 = static_cast<int64_t>(w.m_tile) * BM;
      const bool n_ok = n < p.N;
      float bv = 0.f;
      if (n_ok && p.k_splits == 1 && p.bias != nullptr) bv = __half2float(p.bias[n]);
      constexpr int kChunk = BM < 32 ? 16 : 32;
#pragma unroll 1
      for (int c0 = 0; c0 < BM; c0 += kChunk) {
        uint32_t r[32];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + b * BM + c0;
        if constexpr (kChunk == 32)
          tmem_ld_32cols(taddr, r);
        else
          tmem_ld_16cols(taddr, r);
        tmem_ld_wait();
        if (n_ok) {
#pragma unroll
          for (int j = 0; j < kChunk; ++j) {
            const int64_t m = m0 + c0 + j;
            if (m < p.M) {
              const float v = __uint_as_float(r[j]);
              if (p.k_splits == 1)
                p.y[m * p.ldy + n] = __float2half_rn(v + bv);
              else
                p.partial[(static_cast<int64_t>(w.ks) * p.M + m) * p.N + n] = v;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  } else if (warp >= kDeqWarp0 && warp < kDeqWarp0 + 4) {
    const int t = threadIdx.x - kDeqWarp0 * 32;  // weight row within the tile
    const int two_groups = p.group_size < kBlockK;  // G = 32: two groups per K block
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
      const Unit w = decode_unit(u, p);
      for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
        const uint32_t s = it % S, ph = (it / S) & 1u;
        if (!mbar_wait(&full[s], ph, kErrDeqFull)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * L::kStageBytes;
        const uint4* wrow = reinterpret_cast<const uint4*>(st + L::kWOff + t * 32);
        const uint4 w0 = wrow[0], w1 = wrow[1];
        const __half* srow = reinterpret_cast<const __half*>(st + L::kSOff);
        const uint32_t* zrow = reinterpret_cast<const uint32_t*>(st + L::kZOff);
        const int nib = 4 * awq_nibble_of(t & 7);
        const __half s0 = srow[t];
        const __half s1 = two_groups ? srow[kBlockN + t] : s0;
        const uint32_t z0 = (zrow[t >> 3] >> nib) & 0xFu;
        const uint32_t z1 = two_groups ? ((zrow[16 + (t >> 3)] >> nib) & 0xFu) : z0;
        const __half2 zz0 = zero_magic2(z0), zz1 = zero_magic2(z1);
        const __half2 ss0 = __halves2half2(s0, s0), ss1 = __halves2half2(s1, s1);
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint8_t* arow = st + L::kAOff + t * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const __half2 zz = j < 4 ? zz0 : zz1;
          const __half2 ss = j < 4 ? ss0 : ss1;
          uint4 o;
          o.x = dequant_pair(magic_pair(words[j], 0), zz, ss);
          o.y = dequant_pair(magic_pair(words[j], 1), zz, ss);
          o.z = dequant_pair(magic_pair(words[j], 2), zz, ss);
          o.w = dequant_pair(magic_pair(words[j], 3), zz, ss);
          *reinterpret_cast<uint4*>(arow + ((j ^ (t & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ----------------------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

template <int BM>
int launch_bm(const LinearPlan& pl, const LinearArgs& a, cudaStream_t stream) {
  using L = TcLayout<BM>;
  const int G = a.group_size;
  const uint32_t rows = G < kBlockK ? 2u : 1u;  // group rows per K block
  CUtensorMap mx, mw, ms, mz;
  if (!make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, a.K, a.M, a.ldx * 2, kBlockK, BM,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, a.qw, a.K / 8, a.N, a.K / 2, kBlockK / 8,
                kBlockN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.scales, a.N, a.K / G, a.N * 2, kBlockN,
                rows, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map(&mz, CU_TENSOR_MAP_DATA_TYPE_INT32, a.qzeros, a.N / 8, a.K / G, a.N / 2,
                kBlockN / 8, rows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return TF_ERR_ALIGNMENT;

  TcParams p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.group_size = G;
  p.m_tiles = static_cast<int>(cdiv(a.M, BM));
  p.k_splits = pl.split_k;
  p.kb_total = static_cast<int>(a.K / kBlockK);
  p.kb_per_split = pl.blocks_per_split;
  p.units = static_cast<int>(cdiv(a.N, kBlockN)) * p.m_tiles * p.k_splits;
  p.tx_bytes = static_cast<uint32_t>(L::kXBytes + L::kWBytes + rows * (kBlockN * 2) + rows * 64);
  p.bias = reinterpret_cast<const __half*>(a.bias);
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.partial = pl.split_k > 1 ? static_cast<float*>(a.workspace) : nullptr;

  static std::once_flag attr_once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(w4a16_tc_kernel<BM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    L::kSmemBytes);
  });
  if (attr_err != cudaSuccess) {
    last_cuda_error() = static_cast<int>(attr_err);
    return TF_ERR_CUDA;
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::min(p.units, num_sms())));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (launch_flags() & TF_LAUNCH_PDL) ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w4a16_tc_kernel<BM>, mx, mw, ms, mz, p);
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  if (pl.split_k == 1) return TF_OK;
  return launch_splitk_reduce(p.partial, pl.split_k, a.M, a.N, a.bias, a.y, a.ldy, stream);
}

}  // namespace

bool tc_gemm_supported(int64_t M, int64_t N, int64_t K, int group_size) {
  (void)group_size;
  return M >= 1 && N % 32 == 0 && K % kBlockK == 0 && K / 8 <= (int64_t(1) << 31) &&
         M <= (int64_t(1) << 31) && N <= (int64_t(1) << 31);
}

// Work split for the tensor-core GEMM: tile_m by bucket, then the number of K splits that
// minimises the busiest CTA's share of K blocks over 148 persistent CTAs (at least 8 blocks per
// split), preferring fewer splits on ties.
void plan_tc(int64_t M, int64_t N, int64_t K, LinearPlan* pl) {
  const int64_t n_tiles = cdiv(N, kBlockN), m_tiles = cdiv(M, pl->tile_m);
  const int64_t base = n_tiles * m_tiles;
  const int64_t kb = K / kBlockK;
  const int sms = 148;
  int best_s = 1;
  double best = static_cast<double>(cdiv(base, sms));
  for (int s = 2; s <= 8; ++s) {
    const int64_t per = cdiv(kb, s);
    if (per < 8) break;
    const int64_t splits = cdiv(kb, per);
    const double t = static_cast<double>(cdiv(base * splits, sms)) * per / kb;
    if (t < best * 0.97) {
      best = t;
      best_s = static_cast<int>(splits);
    }
  }
  const int64_t per = cdiv(kb, best_s);
  pl->split_k = static_cast<int>(cdiv(kb, per));
  pl->cluster = 1;
  pl->blocks_per_split = static_cast<int>(per);
  pl->tile_n = kBlockN;
  pl->warps_k = 1;
  pl->grid_x = static_cast<unsigned>(n_tiles);
  pl->grid_y = static_cast<unsigned>(pl->split_k);
  pl->grid_z = static_cast<unsigned>(m_tiles);
  pl->workspace = pl->split_k > 1 ? static_cast<size_t>(pl->split_k * M * N) * sizeof(float) : 0;
}

int launch_tc_gemm(const LinearPlan& pl, const LinearArgs& a, cudaStream_t stream) {
  switch (pl.tile_m) {
    case 16: return launch_bm<16>(pl, a, stream);
    case 32: return launch_bm<32>(pl, a, stream);
    case 64: return launch_bm<64>(pl, a, stream);
    case 128: return launch_bm<128>(pl, a, stream);
    case 256: return launch_bm<256>(pl, a, stream);
    default: return TF_ERR_UNSUPPORTED;
  }
}

}  // namespace tfb

extern "C" int tf_device_error(int* out_code) {
  if (!out_code) return TF_ERR_INVALID_ARG;
  const cudaError_t e = cudaMemcpyFromSymbol(out_code, tfb::g_device_error, sizeof(int));
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

extern "C" int tf_reset_device_error(void) {
  const int zero = 0;
  const cudaError_t e = cudaMemcpyToSymbol(tfb::g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}
