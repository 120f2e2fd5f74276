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

#include "tf_async.cuh"
#include "tf_common.cuh"
#include "tf_plan.h"

namespace tfb {

__device__ int g_device_error = 0;

namespace {

constexpr int kBlockN = 128;  // weight rows per tile = MMA M
constexpr int kBlockK = 64;   // K per swizzle atom: one 128-byte row of fp16
// K per pipeline stage: two atoms (128) for token tiles of up to 64, where the per-stage
// hand-offs, not the tensor core or HBM, set the pace; one atom for the larger tiles.
__host__ __device__ constexpr int stage_k_for(int bm) { return bm <= 64 ? 128 : 64; }
constexpr int kProducerWarp = 0, kMmaWarp = 1, kEpiWarp0 = 4, kDeqWarp0 = 8;
// Dequant warps: 8 (two per SM sub-partition, each converting half of every row of a stage) for
// the token tiles of up to 64, where the weight stream is the bottleneck and registers allow 16
// warps; 4 for the tensor-bound larger tiles, whose epilogue needs more registers per thread.
template <int BM>
__host__ __device__ constexpr int deq_warps() { return BM <= 64 ? 8 : 4; }
template <int BM>
__host__ __device__ constexpr int cta_threads() { return 32 * (kDeqWarp0 + deq_warps<BM>()); }
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

// Shared memory: a deep ring of packed stages (what TMA brings from HBM: x tile, int4 weight
// tile, scale and zero-point rows) and a shallow ring of dequantized fp16 weight tiles. The
// packed stages are small (about 7 KB at BM = 16), so many of them keep HBM busy while the
// dequant warps and the tensor core work a few stages behind.
template <int BM, int KB>
struct TcLayout {
  static constexpr int kAtoms = KB / kBlockK;       // 64-wide swizzle atoms per stage
  static constexpr int kXAtom = BM * 128;           // [BM x 64] fp16 (MMA B operand)
  static constexpr int kAAtom = kBlockN * 128;      // [128 x 64] fp16 (MMA A operand)
  static constexpr int kXBytes = kAtoms * kXAtom;
  static constexpr int kABytes = kAtoms * kAAtom;
  static constexpr int kWBytes = kBlockN * KB / 2;  // [128 x KB/8] int32
  static constexpr int kMaxGroups = KB / 32;        // group rows per stage at G = 32
  static constexpr int kSBytes = kMaxGroups * kBlockN * 2;
  static constexpr int kZBytes = kMaxGroups * 16 * 4;
  static constexpr int kXOff = 0;                  // within a packed stage
  static constexpr int kWOff = kXOff + kXBytes;
  static constexpr int kSOff = kWOff + kWBytes;
  static constexpr int kZOff = kSOff + kSBytes;
  static constexpr int kPStageBytes = ((kZOff + kZBytes) + 1023) / 1024 * 1024;
  // Dequantized tiles in flight: the tensor-bound large tiles need four so that the dequant
  // warps run ahead of the MMAs (two measured 20% slower at M = 1024).
  static constexpr int kAStages = KB == 128 ? 3 : 4;
  static constexpr int kBarrierBytes = 1024;
  static constexpr int kPStagesFit =
      (kSmemLimit - 1024 - kBarrierBytes - kAStages * kABytes) / kPStageBytes;
  static constexpr int kPStages = kPStagesFit < 32 ? kPStagesFit : 32;
  static constexpr int kAOff0 = kPStages * kPStageBytes;  // first dequantized stage
  static constexpr int kBarOff = kAOff0 + kAStages * kABytes;
  static constexpr int kSmemBytes = 1024 + kBarOff + kBarrierBytes;
  static constexpr int kTmemCols = (2 * BM < 32) ? 32 : 2 * BM;  // power of two for BM = 16..256
  static_assert(kPStages >= 2, "shared memory too small for two packed stages");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
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
  // Stream-K (stream_k != 0): CTA c takes stages [c * stages_per_cta, (c + 1) * stages_per_cta)
  // of the (n-tile, m-tile, K stage) sequence; a tile split across CTAs is summed by the last
  // of them to finish (tickets: one counter per tile, zero at launch) from fp32 partials, two
  // slots per CTA ([slot][BM tokens][128 rows]) in `partial`.
  int stream_k;
  int64_t stages_per_cta, total_stages;
  uint32_t* tickets;
};

// ----------------------------------------------------------------------------- PTX wrappers

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
  int tile;    // n-tile * m_tiles + m-tile
  bool split;  // stream-K: part of a tile whose other stages belong to other CTAs
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

// The work of one CTA, in the same order for every warp role: round-robin units (u = blockIdx.x,
// + gridDim.x, ...) or, with stream-K, the pieces of its contiguous stage range.
struct WorkIter {
  int64_t pos, end;
};

__device__ __forceinline__ WorkIter work_begin(const TcParams& p) {
  WorkIter it;
  if (p.stream_k) {
    it.pos = static_cast<int64_t>(blockIdx.x) * p.stages_per_cta;
    it.end = min(p.total_stages, it.pos + p.stages_per_cta);
  } else {
    it.pos = blockIdx.x;
    it.end = p.units;
  }
  return it;
}

__device__ __forceinline__ bool work_next(const TcParams& p, WorkIter& it, Unit& w) {
  if (it.pos >= it.end) return false;
  if (!p.stream_k) {
    w = decode_unit(static_cast<int>(it.pos), p);
    w.tile = static_cast<int>(it.pos);
    w.split = false;
    it.pos += gridDim.x;
    return true;
  }
  const int64_t t = it.pos / p.kb_total;
  const int kb0 = static_cast<int>(it.pos - t * p.kb_total);
  const int64_t room = kb0 + (it.end - it.pos);
  const int kb1 = room < p.kb_total ? static_cast<int>(room) : p.kb_total;
  w.tile = static_cast<int>(t);
  w.m_tile = static_cast<int>(t % p.m_tiles);
  w.n0 = (t / p.m_tiles) * kBlockN;
  w.ks = 0;
  w.kb0 = kb0;
  w.kb1 = kb1;
  w.split = !(kb0 == 0 && kb1 == p.kb_total);
  it.pos += kb1 - kb0;
  return true;
}

// Stream-K partial slot of CTA c's piece of tile t: slot 2c for the piece that starts its
// range, 2c + 1 for the piece that ends it (a CTA whose range lies inside one tile has one).
__device__ __forceinline__ int64_t stream_slot(const TcParams& p, int64_t c, int64_t t) {
  return 2 * c + (c * p.stages_per_cta >= t * p.kb_total ? 0 : 1);
}

template <int BM, int KB>
__global__ void __launch_bounds__(cta_threads<BM>(), 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_s,
                    const __grid_constant__ CUtensorMap tm_z, const TcParams p) {
  using L = TcLayout<BM, KB>;
  constexpr int SP = L::kPStages, SA = L::kAStages;
  constexpr int kDeq = deq_warps<BM>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // pfull: the stage's TMA bytes landed. pempty: the dequant warps read its weights (one
  // arrival each) and the MMAs that read its x tile completed (1). afull: the dequant warps
  // wrote the fp16 tile. aempty: the MMAs that read it completed.
  uint64_t* pfull = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* pempty = pfull + SP;
  uint64_t* afull = pempty + SP;
  uint64_t* aempty = afull + SA;
  uint64_t* acc_full = aempty + SA;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  auto pstage = [&](uint32_t s) { return smem + s * L::kPStageBytes; };
  auto astage = [&](uint32_t a) { return smem + L::kAOff0 + a * L::kABytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < SP; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], kDeq + 1);
    }
    for (int a = 0; a < SA; ++a) {
      mbar_init(&afull[a], kDeq);
      mbar_init(&aempty[a], 1);
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
      WorkIter wi = work_begin(p);
      Unit w;
      while (ok && work_next(p, wi, w)) {
        const int m0 = w.m_tile * BM;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const uint32_t s = it % SP, ph = (it / SP) & 1u;
          if (!mbar_wait(&pempty[s], ph ^ 1u, kErrProducerEmpty)) {
            ok = false;
            break;
          }
          uint8_t* st = pstage(s);
          const int g0 = (kb * KB) / p.group_size;
          mbar_expect_tx(&pfull[s], p.tx_bytes);
#pragma unroll
          for (int at = 0; at < L::kAtoms; ++at)
            tma_load_2d(st + L::kXOff + at * L::kXAtom, &tm_x, &pfull[s], kb * KB + at * kBlockK,
                        m0);
          tma_load_2d(st + L::kWOff, &tm_w, &pfull[s], kb * (KB / 8), static_cast<int>(w.n0));
          tma_load_2d(st + L::kSOff, &tm_s, &pfull[s], static_cast<int>(w.n0), g0);
          tma_load_2d(st + L::kZOff, &tm_z, &pfull[s], static_cast<int>(w.n0 / 8), g0);
        }
      }
      // Drain: every armed stage must have landed before the CTA may exit.
      const uint32_t first = it > static_cast<uint32_t>(SP) ? it - SP : 0;
      for (uint32_t j = first; j < it; ++j)
        if (!mbar_wait(&pfull[j % SP], (j / SP) & 1u, kErrDrain)) break;
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc<BM>();
      uint32_t it = 0, tc = 0;
      bool ok = true;
      bool issued = false;
      uint32_t last_a = 0, last_aph = 0;
      WorkIter wi = work_begin(p);
      Unit w;
      for (; ok && work_next(p, wi, w); ++tc) {
        const uint32_t b = tc & 1u, aph = (tc >> 1) & 1u;
        if (!mbar_wait(&acc_empty[b], aph ^ 1u, kErrMmaAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * BM;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const uint32_t s = it % SP, ph = (it / SP) & 1u;
          const uint32_t a = it % SA, aph = (it / SA) & 1u;
          if (!mbar_wait(&afull[a], aph, kErrMmaDeq) || !mbar_wait(&pfull[s], ph, kErrMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int at = 0; at < L::kAtoms; ++at) {
            const uint64_t a_desc = sw128_desc(smem_u32(astage(a) + at * L::kAAtom));
            const uint64_t b_desc = sw128_desc(smem_u32(pstage(s) + L::kXOff + at * L::kXAtom));
#pragma unroll
            for (int kk = 0; kk < kBlockK / 16; ++kk)
              umma_f16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc,
                       (kb > w.kb0 || at > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&pempty[s]);
          umma_commit(&aempty[a]);
          issued = true;
          last_a = a;
          last_aph = aph;
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
      }
      // Error exit: let the MMAs already issued finish before the TMEM is released.
      if (!ok && issued) mbar_wait(&aempty[last_a], last_aph, kErrDrain);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    const int q = warp - kEpiWarp0;  // TMEM lanes 32q .. 32q+31
    uint32_t tc = 0;
    WorkIter wi = work_begin(p);
    Unit w;
    for (; work_next(p, wi, w); ++tc) {
      const uint32_t b = tc & 1u, aph = (tc >> 1) & 1u;
      if (!mbar_wait(&acc_full[b], aph, kErrEpiAccFull)) break;
      tc_fence_after();
      const int64_t n = w.n0 + 32 * q + lane;
      const int64_t m0 = static_cast<int64_t>(w.m_tile) * BM;
      const bool n_ok = n < p.N;
      float bv = 0.f;
      if (n_ok && p.k_splits == 1 && p.bias != nullptr) bv = __half2float(p.bias[n]);
      // Stream-K piece: the whole [BM x 128] fp32 tile goes to this CTA's slot, row-contiguous
      // per token so that a warp's 32 rows are one 128-byte segment.
      float* slot = w.split ? p.partial + stream_slot(p, blockIdx.x, w.tile) * (BM * kBlockN)
                            : nullptr;
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
        if (w.split) {
#pragma unroll
          for (int j = 0; j < kChunk; ++j)
            __stcg(slot + (c0 + j) * kBlockN + 32 * q + lane, __uint_as_float(r[j]));
        } else if (n_ok) {
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
      if (w.split) {
        // The last CTA to finish its piece of this tile sums the pieces' rows 32q .. 32q+31 in
        // stage order (deterministic whatever the arrival order), adds the bias and writes y.
        // One ticket per (tile, warp quarter): no warp waits on another.
        __threadfence();
        __syncwarp();
        uint32_t ticket = 0;
        if (lane == 0) ticket = atomicAdd(p.tickets + 4 * static_cast<int64_t>(w.tile) + q, 1u);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        const int64_t c_first = static_cast<int64_t>(w.tile) * p.kb_total / p.stages_per_cta;
        const int64_t c_last =
            (static_cast<int64_t>(w.tile + 1) * p.kb_total - 1) / p.stages_per_cta;
        if (ticket == static_cast<uint32_t>(c_last - c_first)) {
          __threadfence();
          if (n_ok) {
            const float bias_v = p.bias != nullptr ? __half2float(p.bias[n]) : 0.f;
            // 16 tokens at a time: each piece's 16 values are independent loads, so a piece
            // costs one L2 round trip per 16 tokens.
            constexpr int kFix = 16;
#pragma unroll 1
            for (int j0 = 0; j0 < BM && m0 + j0 < p.M; j0 += kFix) {
              float acc[kFix];
              const float* src0 = p.partial + stream_slot(p, c_first, w.tile) * (BM * kBlockN) +
                                  j0 * kBlockN + 32 * q + lane;
#pragma unroll
              for (int j = 0; j < kFix; ++j) acc[j] = __ldcg(src0 + j * kBlockN);
              for (int64_t c = c_first + 1; c <= c_last; ++c) {
                const float* src = p.partial + stream_slot(p, c, w.tile) * (BM * kBlockN) +
                                   j0 * kBlockN + 32 * q + lane;
#pragma unroll
                for (int j = 0; j < kFix; ++j) acc[j] += __ldcg(src + j * kBlockN);
              }
#pragma unroll
              for (int j = 0; j < kFix; ++j) {
                const int64_t m = m0 + j0 + j;
                if (m < p.M) p.y[m * p.ldy + n] = __float2half_rn(acc[j] + bias_v);
              }
            }
          }
        }
      }
    }
  } else if (warp >= kDeqWarp0 && warp < kDeqWarp0 + kDeq) {
    const int d = warp - kDeqWarp0;
    const int t = 32 * (d & 3) + lane;             // weight row within the tile
    constexpr int kRowWords = KB / 8;              // packed words of a row per stage
    constexpr int kWords = kRowWords / (kDeq / 4);  // of them, converted by this thread
    const int j0 = (d >> 2) * kWords;              // first of them
    const int gshift = p.group_size == 32 ? 2 : (p.group_size == 64 ? 3 : 4);  // word -> group
    const int nib = 4 * awq_nibble_of(t & 7);
    uint32_t it = 0;
    bool ok = true;
    WorkIter wi = work_begin(p);
    Unit w;
    while (ok && work_next(p, wi, w)) {
      for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
        const uint32_t s = it % SP, ph = (it / SP) & 1u;
        const uint32_t a = it % SA, aph = (it / SA) & 1u;
        if (!mbar_wait(&pfull[s], ph, kErrDeqFull) ||
            !mbar_wait(&aempty[a], aph ^ 1u, kErrDeqFull)) {
          ok = false;
          break;
        }
        uint8_t* st = pstage(s);
        const uint32_t* wrow = reinterpret_cast<const uint32_t*>(st + L::kWOff + t * (KB / 2)) + j0;
        uint32_t words[kWords];
#pragma unroll
        for (int j = 0; j < kWords; j += 4) {
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + j);
          words[j] = v.x;
          words[j + 1] = v.y;
          words[j + 2] = v.z;
          words[j + 3] = v.w;
        }
        const __half* srow = reinterpret_cast<const __half*>(st + L::kSOff);
        const uint32_t* zrow = reinterpret_cast<const uint32_t*>(st + L::kZOff);
        // The stage's group rows start at its first group; word j of the row is in group
        // (j >> gshift) of those. One group per stage (G >= KB, e.g. G = 128) takes the path
        // with the zero point and scale held in registers for the whole row.
        uint8_t* arow = astage(a) + t * 128;
        auto convert = [&](int jj, __half2 zz, __half2 ss) {
          const int j = j0 + jj;  // 16-byte chunk j of the row: k offsets 8j .. 8j+7
          uint4 o;
          o.x = dequant_pair(magic_pair(words[jj], 0), zz, ss);
          o.y = dequant_pair(magic_pair(words[jj], 1), zz, ss);
          o.z = dequant_pair(magic_pair(words[jj], 2), zz, ss);
          o.w = dequant_pair(magic_pair(words[jj], 3), zz, ss);
          const int at = j >> 3, ch = j & 7;
          *reinterpret_cast<uint4*>(arow + at * L::kAAtom + ((ch ^ (t & 7)) << 4)) = o;
        };
        if (p.group_size >= KB) {
          const __half sv = srow[t];
          const __half2 zz = zero_magic2((zrow[t >> 3] >> nib) & 0xFu);
          const __half2 ss = __halves2half2(sv, sv);
#pragma unroll
          for (int jj = 0; jj < kWords; ++jj) convert(jj, zz, ss);
        } else {
#pragma unroll
          for (int jj = 0; jj < kWords; ++jj) {
            const int gi = (j0 + jj) >> gshift;
            const __half sv = srow[gi * kBlockN + t];
            convert(jj, zero_magic2((zrow[gi * 16 + (t >> 3)] >> nib) & 0xFu),
                    __halves2half2(sv, sv));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&afull[a]);
          mbar_arrive(&pempty[s]);
        }
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

template <int BM, int KB>
int launch_bm(const LinearPlan& pl, const LinearArgs& a, cudaStream_t stream) {
  using L = TcLayout<BM, KB>;
  const int G = a.group_size;
  const uint32_t rows = G < KB ? static_cast<uint32_t>(KB / G) : 1u;  // group rows per stage
  CUtensorMap mx, mw, ms, mz;
  if (!make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, a.K, a.M, a.ldx * 2, kBlockK, BM,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, a.qw, a.K / 8, a.N, a.K / 2, KB / 8,
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
  p.kb_total = static_cast<int>(a.K / KB);
  p.kb_per_split = pl.blocks_per_split;
  p.units = static_cast<int>(cdiv(a.N, kBlockN)) * p.m_tiles * p.k_splits;
  p.tx_bytes = static_cast<uint32_t>(L::kXBytes + L::kWBytes + rows * (kBlockN * 2) + rows * 64);
  static_assert(L::kXBytes % 1024 == 0 && L::kWOff % 16 == 0, "stage layout alignment");
  p.bias = reinterpret_cast<const __half*>(a.bias);
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.partial = pl.split_k > 1 ? static_cast<float*>(a.workspace) : nullptr;
  p.stream_k = pl.stream_k;
  p.stages_per_cta = pl.blocks_per_split;
  p.total_stages = static_cast<int64_t>(p.units) * p.kb_total;
  p.tickets = nullptr;
  if (pl.stream_k) {
    // Stream-K: the tickets (one per tile and 32-row quarter) follow the partial slots and must
    // read zero when the kernel starts.
    const size_t partial = static_cast<size_t>(2 * pl.grid_x) * BM * kBlockN * sizeof(float);
    p.partial = static_cast<float*>(a.workspace);
    p.tickets = reinterpret_cast<uint32_t*>(static_cast<char*>(a.workspace) + partial);
    const cudaError_t me = cudaMemsetAsync(p.tickets, 0, static_cast<size_t>(p.units) * 4 *
                                                             sizeof(uint32_t), stream);
    if (me != cudaSuccess) {
      last_cuda_error() = static_cast<int>(me);
      return TF_ERR_CUDA;
    }
  }

  static std::once_flag attr_once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(w4a16_tc_kernel<BM, KB>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
  });
  if (attr_err != cudaSuccess) {
    last_cuda_error() = static_cast<int>(attr_err);
    return TF_ERR_CUDA;
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.stream_k ? pl.grid_x : static_cast<unsigned>(std::min(p.units, num_sms())));
  cfg.blockDim = dim3(cta_threads<BM>());
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (launch_flags() & TF_LAUNCH_PDL) ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w4a16_tc_kernel<BM, KB>, mx, mw, ms, mz, p);
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
int tc_stage_k(int tile_m, int64_t K) {
  const int kb = stage_k_for(tile_m);
  return K % kb == 0 ? kb : kBlockK;
}

void plan_tc(int64_t M, int64_t N, int64_t K, LinearPlan* pl) {
  const int64_t n_tiles = cdiv(N, kBlockN), m_tiles = cdiv(M, pl->tile_m);
  const int64_t base = n_tiles * m_tiles;
  const int stage_k = tc_stage_k(pl->tile_m, K);
  const int64_t kb = K / stage_k;
  const int64_t min_per = 8 * kBlockK / stage_k;  // at least 512 of K per split
  const int sms = 148;
  pl->stream_k = 0;
  // Tiles that do not divide over the SMs (o and down, N = 3584: 28 n-tiles) are dealt as
  // stream-K: every persistent CTA takes the same number of K stages of the tile sequence, and a
  // tile cut between CTAs is summed by the last of them (fp32 partials, two slots per CTA).
  // Only where a CTA's run covers at least half a tile (a tile is cut into at most about three
  // pieces); with shorter runs the last CTA's sum of many pieces costs more than the split-K
  // reduce launch it replaces.
  const int64_t sk_total = base * kb;
  const int64_t sk_per = cdiv(sk_total, sms);
  if (static_cast<double>(cdiv(base, sms)) > 1.05 * static_cast<double>(base) / sms &&
      2 * sk_per >= kb) {
    const int64_t grid = cdiv(sk_total, sk_per);
    pl->stream_k = 1;
    pl->split_k = 1;
    pl->cluster = 1;
    pl->blocks_per_split = static_cast<int>(sk_per);
    pl->tile_n = kBlockN;
    pl->warps_k = 1;
    pl->grid_x = static_cast<unsigned>(grid);
    pl->grid_y = 1;
    pl->grid_z = 1;
    const size_t partial = static_cast<size_t>(2 * grid) * pl->tile_m * kBlockN * sizeof(float);
    pl->workspace = partial + static_cast<size_t>(base) * 4 * sizeof(uint32_t);
    return;
  }
  int best_s = 1;
  double best = static_cast<double>(cdiv(base, sms));
  for (int s = 2; s <= 8; ++s) {
    const int64_t per = cdiv(kb, s);
    if (per < min_per) break;
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
  const bool wide = tc_stage_k(pl.tile_m, a.K) == 128;
  switch (pl.tile_m) {
    case 16: return wide ? launch_bm<16, 128>(pl, a, stream) : launch_bm<16, 64>(pl, a, stream);
    case 32: return wide ? launch_bm<32, 128>(pl, a, stream) : launch_bm<32, 64>(pl, a, stream);
    case 64: return wide ? launch_bm<64, 128>(pl, a, stream) : launch_bm<64, 64>(pl, a, stream);
    case 128: return launch_bm<128, 64>(pl, a, stream);
    case 256: return launch_bm<256, 64>(pl, a, stream);
    default: return TF_ERR_UNSUPPORTED;
  }
}

}  // namespace tfb

// The GEMM's status word first (0x1xx codes), else the RMSNorm streaming kernel's (0x3xx).
extern "C" int tf_device_error(int* out_code) {
  if (!out_code) return TF_ERR_INVALID_ARG;
  const cudaError_t e = cudaMemcpyFromSymbol(out_code, tfb::g_device_error, sizeof(int));
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return *out_code != 0 ? TF_OK : tfb::rms_device_error(out_code);
}

extern "C" int tf_reset_device_error(void) {
  const int zero = 0;
  const cudaError_t e = cudaMemcpyToSymbol(tfb::g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return tfb::rms_reset_device_error();
}
