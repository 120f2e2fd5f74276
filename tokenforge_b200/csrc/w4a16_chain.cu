// Persistent decode chain: a fixed sequence of W4A16 linears at decode sizes (M <= 8 tokens,
// group size 128) run by ONE cooperative launch with one CTA per SM.
//
// Why: at decode every linear is a few MB of weights (Qwen2.5-7B: 6.7 MB for o, 8.6 MB for qkv)
// and one launch per linear pays a fixed cost (launch, ramp-up, the CTAs' cross-warp reduction
// and the tail of the last wave) of about 4 us per layer, more than streaming o's weights takes.
// Here the HBM weight stream does not stop at layer boundaries: every warp streams its own
// weight chunks with TMA into a private shared-memory ring that runs ahead into the next layers
// while the current layer's dependency wait, activation staging and reductions proceed.
//
// Reference semantics: each op computes what tf_w4a16_linear computes for it (the reference's
// tokenforge/kernels/triton/w4a16.py:44-115 at BLOCK_M <= 8 plus the split-K contract of
// w4a16.py:193-200,227-232: fp32 partials summed in a fixed order, then bias, then one rounding
// to fp16). The K split differs from the per-layer GEMV's, so results agree within the W4A16
// tolerance rather than bit for bit; for a given chain they are deterministic.
//
// Work decomposition (host planner, plan_chain):
//   * chunk = 32 weight rows x 256 K (two quantization groups): 4 KB of packed weights (one TMA
//     box, 128-byte swizzle), 128 B of scales and 32 B of zero points (two more boxes);
//   * unit = R row tiles of 32 rows x a chunk range [c0, c1) of one op, run by all 16 warps of
//     the CTA: warp w takes row tile w % R and, of the unit's chunks, c0 + w / R + i * (16 / R);
//     the 16 / R warps sharing a row tile are summed in warp order through shared memory;
//   * per op, whole row-tile groups round-robin over the CTAs (small ops, and ops whose tile
//     groups divide evenly), or exact stream-K: the op's (tile group, chunk) sequence cut into
//     one equal range per CTA, a tile group spanning several CTAs being finished by the last CTA
//     to arrive (fp32 partials in a workspace, summed in piece order, so the result does not
//     depend on arrival order);
//   * units longer than the activation buffer allows are cut into sub-units that keep
//     accumulating in registers.
// Dependencies: op l with `wait` set reads its activations only after every CTA has finished
// all ops before l (a per-op arrival counter; the waiting thread polls it with acquire loads).
// Counters grow by one launch's worth per run (an epoch read at kernel start), so nothing is
// reset between runs; the last CTA to exit advances the epoch. Every wait is bounded (2 s): on a
// timeout the kernel records a code in the chain's error word and stops waiting, so a chain
// never hangs; its output is then undefined. No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "tf_async.cuh"
#include "tf_common.cuh"
#include "tf_plan.h"
#include "tf_w4a16_math.cuh"

namespace tfb {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = 32 * kWarps;
constexpr int kRing = 3;                      // chunk slots per warp (two in flight while one is read)
constexpr int kChunkK = 256;                  // K values per chunk
constexpr int kTileRows = 32;                 // weight rows per row tile
constexpr int kWBytes = kTileRows * 128;      // packed weights of a chunk: 32 rows x 128 bytes
constexpr int kSBytes = 2 * kTileRows * 2;    // scales: [2 groups][32 rows] fp16
constexpr int kZBytes = 2 * 4 * 4;            // zero points: [2 groups][4 words]
// A slot's scale and zero-point boxes each start on a 128-byte boundary (the alignment TMA
// requires of a shared-memory destination).
constexpr int kSZBytes = 256;
constexpr int kZOffInSZ = 128;
constexpr uint32_t kTxBytes = kWBytes + kSBytes + kZBytes;
static_assert(kSBytes <= kZOffInSZ && kZOffInSZ + kZBytes <= kSZBytes, "scale/zero slot layout");
constexpr int kMaxM = 8;
constexpr int kRedFloats = 8 * 32;            // per warp: 8 fragment values x 32 lanes
constexpr unsigned long long kChainWaitNs = 2000000000ull;

// Shared-memory layout (offsets from a 1024-byte aligned base; the swizzled TMA boxes need it).
constexpr int kOffW = 0;
constexpr int kOffSZ = kOffW + kWarps * kRing * kWBytes;
constexpr int kOffBar = kOffSZ + kWarps * kRing * kSZBytes;
constexpr int kOffMisc = kOffBar + kWarps * kRing * 8;  // epoch, last-arrival flags of 16 tiles
// The staged activations and the cross-warp reduction buffer share one region: a unit's partials
// are written only after every warp has finished reading its activations.
constexpr int kOffX = kOffMisc + 128;
constexpr int kRedBytes = kWarps * kRedFloats * 4;
constexpr int kSmemCap = 227 * 1024;
constexpr int kAlignSlack = 1024;
static_assert(kOffW % 1024 == 0 && kWBytes % 1024 == 0, "128-byte-swizzled boxes need 1 KB alignment");
static_assert(kOffSZ % 128 == 0 && kSZBytes % 128 == 0, "TMA destinations need 128-byte alignment");
static_assert(kOffBar % 8 == 0 && kOffX % 16 == 0, "shared-memory alignment");

// Error codes recorded in the chain's error word (first one wins).
constexpr uint32_t kErrDepWait = 0x201;    // an op's dependency counter did not complete in time
constexpr uint32_t kErrChunkWait = 0x202;  // a weight chunk's TMA did not complete in time

struct alignas(64) ChainOpDev {
  CUtensorMap mw;  // qweight_t int32 [N, K/8]: box 32 rows x 32 words, 128-byte swizzle
  CUtensorMap ms;  // scales fp16 [K/G, N]: box 2 groups x 32 columns
  CUtensorMap mz;  // qzeros int32 [K/G, N/8]: box 2 groups x 4 words
  const __half* x;
  const __half* bias;
  __half* y;
  int64_t ldx, ldy;
  int32_t n, k, wait, tiles;
};

enum UnitFlags : uint8_t { kFirst = 1, kLast = 2, kSplit = 4 };

struct ChainUnitDev {
  int32_t tile0;    // first row tile of the unit
  uint16_t op;
  uint8_t rtiles;   // R: row tiles per unit (1, 2, 4, 8 or 16)
  uint8_t flags;    // kFirst: zero the accumulators; kLast: reduce and write; kSplit: a piece
  uint16_t c0, c1;  // chunk range
  uint16_t piece, pieces;
  int32_t slot;     // kSplit: partial slot of (piece 0, tile 0); (piece p, tile r) = slot + p * R + r
  int32_t counter;  // kSplit: arrival counter of tile 0; tile r uses counter + r
};
static_assert(sizeof(ChainUnitDev) == 24, "unit record layout");

struct ChainParams {
  const ChainOpDev* ops;
  const ChainUnitDev* units;
  const int32_t* cta_units;  // [grid + 1]: unit range of each CTA
  uint32_t* ctl;             // [0] epoch, [1] exited CTAs, [2] error word
  uint32_t* done;            // [n_ops]: CTAs that have finished each op (grows every run)
  uint32_t* counters;        // split tiles' arrival counters (grow every run)
  float* partials;           // [slots][kRedFloats]: a piece's partial in fragment order
  int n_ops;
  int M;
  int x_stride;              // fp16 elements per staged activation row
};

__device__ __forceinline__ void record_error(uint32_t* ctl, uint32_t code) {
  atomicCAS(ctl + 2, 0u, code);
}

__device__ __forceinline__ bool error_set(const uint32_t* ctl) {
  return *reinterpret_cast<const volatile uint32_t*>(ctl + 2) != 0u;
}

// Bounded wait on a chunk's full barrier; false (and the error recorded) after the limit. Once
// any wait of the launch has given up, the others stop waiting at once.
__device__ __noinline__ bool chunk_wait_slow(uint64_t* bar, uint32_t parity, uint32_t* ctl) {
  const unsigned long long t0 = global_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (error_set(ctl)) return false;
    if (global_ns() - t0 > kChainWaitNs) {
      record_error(ctl, kErrChunkWait);
      return false;
    }
  }
}

__device__ __forceinline__ bool chunk_wait(uint64_t* bar, uint32_t parity, uint32_t* ctl) {
  if (mbar_try_wait(bar, parity)) return true;
  return chunk_wait_slow(bar, parity, ctl);
}

__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

// The sequence of (unit, chunk) one warp consumes, walked ahead by the TMA issue side. The
// current unit's fields are cached, so stepping within a unit reads no memory.
struct ChunkWalk {
  int u, u_end;
  int c, c1, step;  // next chunk of unit u, end of its range, this warp's stride
  int op, tile;
  bool live;
};

// Moves to the first unit at or after w.u in which this warp has a chunk; false at the end.
// Entering an op's first unit prefetches the tensor maps of the op after it, so the descriptor
// is on chip before its first copy.
__device__ __forceinline__ bool walk_enter(ChunkWalk& w, const ChainParams& p, int warp, int lane) {
  for (; w.u < w.u_end; ++w.u) {
    const ChainUnitDev U = p.units[w.u];
    const int R = U.rtiles;
    const int tile = U.tile0 + warp % R;
    const int c = U.c0 + warp / R;
    if (tile < p.ops[U.op].tiles && c < U.c1) {
      if (lane == 0 && U.op != w.op && U.op + 1 < p.n_ops) {
        const ChainOpDev* nx = p.ops + U.op + 1;
        prefetch_tmap(&nx->mw);
        prefetch_tmap(&nx->ms);
        prefetch_tmap(&nx->mz);
      }
      w.c = c;
      w.c1 = U.c1;
      w.step = kWarps / R;
      w.op = U.op;
      w.tile = tile;
      return true;
    }
  }
  return false;
}

__device__ __forceinline__ void walk_next(ChunkWalk& w, const ChainParams& p, int warp, int lane) {
  w.c += w.step;
  if (w.c < w.c1) return;
  ++w.u;
  w.live = walk_enter(w, p, warp, lane);
}

// Lane 0: the three TMA boxes of one chunk into ring slot `slot` of warp `warp`. `reuse`: the
// slot held an earlier chunk, read by the warp through the generic proxy.
__device__ __forceinline__ void issue_chunk(const ChainParams& p, uint8_t* smem, int warp,
                                            int slot, int op, int tile, int chunk, bool reuse) {
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar) + warp * kRing + slot;
  uint8_t* wdst = smem + kOffW + (warp * kRing + slot) * kWBytes;
  uint8_t* szdst = smem + kOffSZ + (warp * kRing + slot) * kSZBytes;
  if (reuse) fence_proxy_async_smem();
  mbar_expect_tx(bar, kTxBytes);
  const ChainOpDev* o = p.ops + op;
  tma_load_2d(wdst, &o->mw, bar, chunk * 32, tile * kTileRows);
  tma_load_2d(szdst, &o->ms, bar, tile * kTileRows, chunk * 2);
  tma_load_2d(szdst + kZOffInSZ, &o->mz, bar, tile * 4, chunk * 2);
}

// Block b (0 or 1) of a chunk in the ring as this lane's GSlot: rows 4q..4q+3, 16 bytes each at
// logical 16-byte column 4b + c of the 128-byte swizzled rows; physical column = logical ^ (row
// % 8) = 4 (b ^ (q % 2)) + (c ^ j) for row 4q + j. loff[j] = row * 128 + 16 (c ^ j) and
// boff = 64 (b ^ (q % 2)) are per-lane constants.
__device__ __forceinline__ void ring_block(GSlot& s, const uint8_t* w, const uint8_t* sz,
                                           const uint32_t (&loff)[4], uint32_t boff, int b, int q) {
#pragma unroll
  for (int j = 0; j < 4; ++j) s.w[j] = *reinterpret_cast<const uint4*>(w + loff[j] + boff);
  s.s = *reinterpret_cast<const uint2*>(sz + b * 64 + q * 8);
  s.z = *reinterpret_cast<const uint32_t*>(sz + kZOffInSZ + b * 16 + (q >> 1) * 4);
}

// Stages x[0:M, c0 * 256 : c1 * 256] (zero past K) into shared memory, rows x_stride apart, with
// L2-only asynchronous copies (the activations may have been written by other CTAs of this
// launch). Returns once this thread's copies have landed; the caller synchronises the CTA.
__device__ __forceinline__ void stage_x(const ChainParams& p, const ChainOpDev& o, __half* xs,
                                        int c0, int c1) {
  const int vec_per_row = (c1 - c0) * (kChunkK / 8);
  const int total = p.M * vec_per_row;
  const int k_lo = c0 * kChunkK;
  for (int i = threadIdx.x; i < total; i += kThreads) {
    const int m = i / vec_per_row, v = i - m * vec_per_row;
    const int k = k_lo + 8 * v;
    uint4* dst = reinterpret_cast<uint4*>(xs + m * p.x_stride) + v;
    if (k < o.k) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)),
                   "l"(o.x + m * o.ldx + k)
                   : "memory");
    } else {
      *dst = make_uint4(0, 0, 0, 0);
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Fragment value f (t * 4 + r) of lane ln in a warp's 32-row tile: row 4 (ln / 4) + 2t + r / 2,
// token 2 (ln % 4) + r % 2 (the m16n8 accumulator layout of the two 16-row MMA tiles).
__device__ __forceinline__ void write_value(const ChainOpDev& o, int M, int tile, int f, int ln,
                                            float v) {
  const int n = tile * kTileRows + 4 * (ln >> 2) + 2 * (f >> 2) + ((f & 3) >> 1);
  const int m = 2 * (ln & 3) + (f & 1);
  if (m >= M || n >= o.n) return;
  if (o.bias) v += __half2float(__ldg(o.bias + n));
  o.y[static_cast<int64_t>(m) * o.ldy + n] = __float2half_rn(v);
}

__global__ void __launch_bounds__(kThreads, 1) w4a16_chain_kernel(const ChainParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  float* red = reinterpret_cast<float*>(smem + kOffX);  // aliases xs (see kOffX)
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  __half* xs = reinterpret_cast<__half*>(smem + kOffX);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = lane >> 2, c = lane & 3;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kRing; ++s) mbar_init(&bars[warp * kRing + s], 1);
    fence_barrier_init();
  }
  if (tid == 0) misc[0] = *reinterpret_cast<const volatile uint32_t*>(p.ctl);
  __syncthreads();
  const uint32_t epoch = misc[0];
  const uint32_t done_target = (epoch + 1u) * gridDim.x;

  const int u_begin = p.cta_units[blockIdx.x], u_end = p.cta_units[blockIdx.x + 1];
  uint8_t* ring_w = smem + kOffW + warp * kRing * kWBytes;
  uint8_t* ring_sz = smem + kOffSZ + warp * kRing * kSZBytes;
  uint32_t loff[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) loff[j] = (4 * q + j) * 128 + 16 * (c ^ j);
  const uint32_t boff0 = 64u * (q & 1), boff1 = 64u - boff0;

  // TMA issue side of this warp: `issued` chunks so far, walking ahead of consumption.
  ChunkWalk walk;
  walk.u = u_begin;
  walk.u_end = u_end;
  walk.op = -1;
  walk.live = walk_enter(walk, p, warp, lane);
  int issued = 0;
  // Keeps kRing chunks in flight: slot (issued % kRing) last held chunk issued - kRing, which the
  // warp has finished reading (consumed > issued - kRing).
  auto top_up = [&](int consumed) {
    __syncwarp();
    while (walk.live && issued < consumed + kRing) {
      if (lane == 0)
        issue_chunk(p, smem, warp, issued % kRing, walk.op, walk.tile, walk.c, issued >= kRing);
      ++issued;
      walk_next(walk, p, warp, lane);
    }
  };
  top_up(0);

  int consumed = 0;
  int arrived = -1;  // ops whose arrival this CTA has published
  int passed = -1;   // the CTA has waited for every op before `passed`
  const uint4* xs4 = reinterpret_cast<const uint4*>(xs);
  float acc[2][2][4] = {};  // x * fp16((q - z) * s) in fp32: two chains per row tile
  bool timed_out = false;

  for (int u = u_begin; u < u_end; ++u) {
    const ChainUnitDev U = p.units[u];
    const ChainOpDev& o = p.ops[U.op];
    // Finishing earlier ops: publish this CTA's arrival for every op before this one (its
    // outputs of those ops are written and fenced), then wait for the ops this one reads.
    if (U.op - 1 > arrived) {
      __threadfence();
      __syncthreads();
      if (tid == 0)
        for (int l = arrived + 1; l < U.op; ++l) red_release_gpu_add(p.done + l, 1u);
      arrived = U.op - 1;
    }
    if (U.op > passed) {
      if (o.wait && U.op > 0 && tid == 0) {
        const uint32_t* f = p.done + (U.op - 1);
        const unsigned long long t0 = global_ns();
        while (static_cast<int32_t>(ld_acquire_gpu(f) - done_target) < 0) {
          if (error_set(p.ctl)) break;
          if (global_ns() - t0 > kChainWaitNs) {
            record_error(p.ctl, kErrDepWait);
            break;
          }
        }
      }
      passed = U.op;
    }
    __syncthreads();  // dependency passed; the previous unit's reads of xs and red are done
    stage_x(p, o, xs, U.c0, U.c1);
    __syncthreads();

    const int R = U.rtiles, P = kWarps / R;
    const int tile = U.tile0 + warp % R;
    const int j = warp / R;
    if (U.flags & kFirst) {
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[t][0][r] = acc[t][1][r] = 0.f;
    }
    GLane L;
    L.c = c;
    L.kb0 = 2 * U.c0;
    L.nib[0] = (q & 1) ? 8 : 0;  // rows 4q..4q+3: zero points in nibbles {0,4,1,5} or {2,6,3,7}
    L.xs = xs4 + (min(q, p.M - 1) * p.x_stride + 32 * c) / 8;
    if (tile < o.tiles) {
      for (int ch = U.c0 + j; ch < U.c1; ch += P) {
        top_up(consumed);
        const int slot = consumed % kRing;
        if (!chunk_wait(&bars[warp * kRing + slot], (consumed / kRing) & 1u, p.ctl)) timed_out = true;
        const uint8_t* wt = ring_w + slot * kWBytes;
        const uint8_t* sz = ring_sz + slot * kSZBytes;
        GSlot s0, s1;
        ring_block(s0, wt, sz, loff, boff0, 0, q);
        ring_block(s1, wt, sz, loff, boff1, 1, q);
        gcompute_w16(acc, s0, 2 * ch, L);
        gcompute_w16(acc, s1, 2 * ch + 1, L);
        ++consumed;
      }
    }
    if (!(U.flags & kLast)) continue;

    // Reduce: every warp publishes its tile's partial (over the activations, which every warp
    // has finished reading); then all threads of the CTA sum the P warps of each row tile in
    // warp order, one fragment value each, and write it.
    __syncthreads();
    float* mine = red + warp * kRedFloats;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int r = 0; r < 4; ++r) mine[(t * 4 + r) * 32 + lane] = acc[t][0][r] + acc[t][1][r];
    __syncthreads();
    const int nvals = R * kRedFloats;
    const bool split = (U.flags & kSplit) != 0;
#pragma unroll
    for (int i = 0; i < kRedFloats * kWarps / kThreads; ++i) {  // R * 256 values, <= 8 per thread
      const int v = tid + i * kThreads;
      if (v >= nvals) continue;
      const int r_in = v / kRedFloats, fl = v % kRedFloats;
      float a = 0.f;
      for (int jj = 0; jj < P; ++jj) a += red[(r_in + jj * R) * kRedFloats + fl];
      if (!split) {
        if (U.tile0 + r_in < o.tiles) write_value(o, p.M, U.tile0 + r_in, fl >> 5, fl & 31, a);
      } else {
        p.partials[static_cast<int64_t>(U.slot + U.piece * R + r_in) * kRedFloats + fl] = a;
      }
    }
    if (!split) continue;
    // A piece of tiles split across CTAs: the last CTA to publish its piece of a tile sums all
    // pieces in piece order and writes the tile.
    __threadfence();
    __syncthreads();
    if (tid < R) {
      const uint32_t old = atom_acq_rel_gpu_add(p.counters + U.counter + tid, 1u);
      misc[8 + tid] = (old + 1u == (epoch + 1u) * U.pieces) ? 1u : 0u;
    }
    __syncthreads();
    __threadfence();
#pragma unroll
    for (int i = 0; i < kRedFloats * kWarps / kThreads; ++i) {
      const int v = tid + i * kThreads;
      if (v >= nvals) continue;
      const int r_in = v / kRedFloats, fl = v % kRedFloats;
      if (!misc[8 + r_in] || U.tile0 + r_in >= o.tiles) continue;
      float a = 0.f;
      for (int pc = 0; pc < U.pieces; ++pc)
        a += ld_cg_f32(p.partials + static_cast<int64_t>(U.slot + pc * R + r_in) * kRedFloats + fl);
      write_value(o, p.M, U.tile0 + r_in, fl >> 5, fl & 31, a);
    }
  }

  // Publish the remaining arrivals, drain this warp's copies if a wait gave up, and let the last
  // CTA out advance the epoch for the next run.
  __threadfence();
  __syncthreads();
  if (tid == 0)
    for (int l = arrived + 1; l < p.n_ops; ++l) red_release_gpu_add(p.done + l, 1u);
  if (timed_out) {
    for (int n = max(0, issued - kRing); n < issued; ++n)
      chunk_wait(&bars[warp * kRing + n % kRing], (n / kRing) & 1u, p.ctl);
  }
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.ctl + 1, 1u);
    if (prev == gridDim.x - 1u) {
      p.ctl[1] = 0u;
      __threadfence();
      atomicExch(p.ctl, epoch + 1u);
    }
  }
}

// ----------------------------------------------------------------------------- host side

struct PlanUnit {
  int cta, op, tile0, rtiles, c0, c1, piece, pieces, flags, slot, counter;
};

struct ChainPlan {
  std::vector<std::vector<PlanUnit>> per_cta;
  int slots = 0, counters = 0, max_chunks = 0;
};

int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Largest chunk range one unit may stage for M tokens: the activations of the range must fit
// the shared memory left after the rings, barriers and reduction buffer.
int max_unit_chunks(int M) {
  const int budget = kSmemCap - kAlignSlack - kOffX;
  return std::min((budget / (2 * M) - 8) / kChunkK, 65535);
}

void emit_piece(ChainPlan& pl, int cta, int op, int tile0, int R, int c0, int c1, int piece,
                int pieces, int slot, int counter, int cmax) {
  for (int a = c0; a < c1; a += cmax) {
    const int b = std::min(c1, a + cmax);
    int flags = (a == c0 ? kFirst : 0) | (b == c1 ? kLast : 0) | (piece >= 0 ? kSplit : 0);
    pl.per_cta[cta].push_back({cta, op, tile0, R, a, b, std::max(piece, 0), std::max(pieces, 1),
                               flags, slot, counter});
    pl.max_chunks = std::max(pl.max_chunks, b - a);
  }
}

// The unit schedule of a chain (see the file header). Every (op, row tile, chunk) is covered
// by exactly one unit; each CTA's units are in op order.
int plan_chain(const int64_t* n, const int64_t* k, int n_ops, int M, int ctas, ChainPlan* out) {
  if (n_ops < 1 || ctas < 1 || M < 1 || M > kMaxM) return TF_ERR_INVALID_ARG;
  const int cmax = max_unit_chunks(M);
  if (cmax < 1) return TF_ERR_UNSUPPORTED;
  ChainPlan pl;
  pl.per_cta.assign(ctas, {});
  int rot = 0;
  for (int op = 0; op < n_ops; ++op) {
    const int T = static_cast<int>(n[op] / kTileRows);
    const int C = static_cast<int>(cdiv(k[op], kChunkK));
    int R = 1;
    for (int r = 16; r >= 2; r /= 2)
      if (ceil_div(T, r) >= ctas) {
        R = r;
        break;
      }
    const int groups = ceil_div(T, R);
    const double mean = static_cast<double>(T) * C / ctas;
    const double whole_max = static_cast<double>(ceil_div(groups, ctas)) * R * C;
    const bool small = T <= ctas && C * R <= 2 * kWarps;
    if (small || whole_max <= 1.15 * mean) {
      for (int g = 0; g < groups; ++g)
        emit_piece(pl, (rot + g) % ctas, op, g * R, R, 0, C, -1, 1, 0, 0, cmax);
      rot = (rot + groups) % ctas;
      continue;
    }
    // Exact stream-K over the (tile group, chunk) sequence.
    const int64_t total = static_cast<int64_t>(groups) * C;
    struct Piece { int cta, g, a, b; };
    std::vector<Piece> pieces;
    for (int i = 0; i < ctas; ++i) {
      const int64_t a = total * i / ctas, b = total * (i + 1) / ctas;
      for (int64_t s = a; s < b;) {
        const int g = static_cast<int>(s / C);
        const int64_t e = std::min<int64_t>(b, static_cast<int64_t>(g + 1) * C);
        pieces.push_back({(rot + i) % ctas, g, static_cast<int>(s - int64_t(g) * C),
                          static_cast<int>(e - int64_t(g) * C)});
        s = e;
      }
    }
    // Pieces are in (group, chunk) order: number them per group.
    for (size_t i = 0; i < pieces.size();) {
      size_t e = i;
      while (e < pieces.size() && pieces[e].g == pieces[i].g) ++e;
      const int cnt = static_cast<int>(e - i);
      int slot = 0, counter = 0;
      if (cnt > 1) {
        slot = pl.slots;
        counter = pl.counters;
        pl.slots += cnt * R;
        pl.counters += R;
      }
      for (size_t x = i; x < e; ++x)
        emit_piece(pl, pieces[x].cta, op, pieces[x].g * R, R, pieces[x].a, pieces[x].b,
                   cnt > 1 ? static_cast<int>(x - i) : -1, cnt, slot, counter, cmax);
      i = e;
    }
    rot = (rot + ctas) % ctas;
  }
  *out = std::move(pl);
  return TF_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 chain_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult qr;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool chain_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
               uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swizzle) {
  auto fn = chain_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int validate_chain_op(const TfChainOp& op, int64_t M) {
  if (op.N < kTileRows || op.K < 128) return TF_ERR_INVALID_ARG;
  if (op.N % kTileRows != 0 || op.K % 128 != 0) return TF_ERR_UNSUPPORTED;
  if (op.N * (op.K / 8) >= (int64_t(1) << 31) || op.K >= (int64_t(1) << 20) ||
      op.N >= (int64_t(1) << 24))
    return TF_ERR_UNSUPPORTED;
  if (!op.x || !op.qweight_t || !op.scales || !op.qzeros || !op.y) return TF_ERR_INVALID_ARG;
  if (op.ldx < op.K || op.ldy < op.N) return TF_ERR_INVALID_ARG;
  if (!aligned16(op.x) || op.ldx % 8 != 0 || !aligned16(op.qweight_t) || !aligned16(op.scales) ||
      !aligned16(op.qzeros))
    return TF_ERR_ALIGNMENT;
  if (M * op.ldx >= (int64_t(1) << 31) || M * op.ldy >= (int64_t(1) << 31))
    return TF_ERR_UNSUPPORTED;
  return TF_OK;
}

}  // namespace
}  // namespace tfb

struct TfChain {
  int device = 0;
  int grid = 0;
  size_t smem = 0;
  void* mem = nullptr;  // one device allocation: ops | units | cta ranges | control | partials
  tfb::ChainParams params{};
};

extern "C" {

int tf_decode_chain_plan(const int64_t* n, const int64_t* k, int32_t n_ops, int64_t M,
                         int32_t num_ctas, TfChainUnitInfo* out, int32_t capacity,
                         int32_t* n_units) {
  if (!n || !k || !n_units || n_ops < 1 || num_ctas < 1) return TF_ERR_INVALID_ARG;
  for (int i = 0; i < n_ops; ++i)
    if (n[i] < tfb::kTileRows || n[i] % tfb::kTileRows || k[i] < 128 || k[i] % 128)
      return TF_ERR_UNSUPPORTED;
  tfb::ChainPlan pl;
  const int st = tfb::plan_chain(n, k, n_ops, static_cast<int>(M), num_ctas, &pl);
  if (st != TF_OK) return st;
  int count = 0;
  for (const auto& v : pl.per_cta) {
    for (const auto& u : v) {
      if (out && count < capacity) {
        TfChainUnitInfo& o = out[count];
        o.cta = u.cta;
        o.op = u.op;
        o.tile0 = u.tile0;
        o.rtiles = u.rtiles;
        o.c0 = u.c0;
        o.c1 = u.c1;
        o.piece = (u.flags & tfb::kSplit) ? u.piece : -1;
        o.pieces = u.pieces;
        o.flags = u.flags;
      }
      ++count;
    }
  }
  *n_units = count;
  return (out && count > capacity) ? TF_ERR_TOO_LARGE : TF_OK;
}

int tf_decode_chain_create(const TfChainOp* ops, int32_t n_ops, int64_t M, int32_t group_size,
                           TfChain** out) {
  using namespace tfb;
  if (!out || !ops || n_ops < 1 || n_ops > 65535) return TF_ERR_INVALID_ARG;
  *out = nullptr;
  if (M < 1 || M > kMaxM) return TF_ERR_UNSUPPORTED;
  if (group_size != 128) return TF_ERR_UNSUPPORTED;
  std::vector<int64_t> ns(n_ops), ks(n_ops);
  for (int i = 0; i < n_ops; ++i) {
    const int st = validate_chain_op(ops[i], M);
    if (st != TF_OK) return st;
    ns[i] = ops[i].N;
    ks[i] = ops[i].K;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  int sms = 0, coop = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  if (!coop) return TF_ERR_UNSUPPORTED;
  ChainPlan pl;
  int st = plan_chain(ns.data(), ks.data(), n_ops, static_cast<int>(M), sms, &pl);
  if (st != TF_OK) return st;

  std::vector<ChainOpDev> hops(n_ops);
  for (int i = 0; i < n_ops; ++i) {
    const TfChainOp& s = ops[i];
    ChainOpDev& d = hops[i];
    std::memset(static_cast<void*>(&d), 0, sizeof(d));
    const uint64_t G = 128;
    if (!chain_map(&d.mw, CU_TENSOR_MAP_DATA_TYPE_INT32, s.qweight_t, s.K / 8, s.N, s.K / 2, 32,
                   kTileRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !chain_map(&d.ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, s.scales, s.N, s.K / G, s.N * 2,
                   kTileRows, 2, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !chain_map(&d.mz, CU_TENSOR_MAP_DATA_TYPE_INT32, s.qzeros, s.N / 8, s.K / G, s.N / 2, 4,
                   2, CU_TENSOR_MAP_SWIZZLE_NONE))
      return TF_ERR_ALIGNMENT;
    d.x = reinterpret_cast<const __half*>(s.x);
    d.bias = reinterpret_cast<const __half*>(s.bias);
    d.y = reinterpret_cast<__half*>(s.y);
    d.ldx = s.ldx;
    d.ldy = s.ldy;
    d.n = static_cast<int32_t>(s.N);
    d.k = static_cast<int32_t>(s.K);
    d.wait = s.wait ? 1 : 0;
    d.tiles = static_cast<int32_t>(s.N / kTileRows);
  }
  std::vector<ChainUnitDev> hunits;
  std::vector<int32_t> ranges(sms + 1, 0);
  for (int cta = 0; cta < sms; ++cta) {
    ranges[cta] = static_cast<int32_t>(hunits.size());
    for (const PlanUnit& u : pl.per_cta[cta]) {
      ChainUnitDev d;
      d.tile0 = u.tile0;
      d.op = static_cast<uint16_t>(u.op);
      d.rtiles = static_cast<uint8_t>(u.rtiles);
      d.flags = static_cast<uint8_t>(u.flags);
      d.c0 = static_cast<uint16_t>(u.c0);
      d.c1 = static_cast<uint16_t>(u.c1);
      d.piece = static_cast<uint16_t>(u.piece);
      d.pieces = static_cast<uint16_t>(u.pieces);
      d.slot = u.slot;
      d.counter = u.counter;
      hunits.push_back(d);
    }
  }
  ranges[sms] = static_cast<int32_t>(hunits.size());

  const size_t off_ops = 0;
  const size_t off_units = align_up(off_ops + sizeof(ChainOpDev) * n_ops, 256);
  const size_t off_ranges = align_up(off_units + sizeof(ChainUnitDev) * hunits.size(), 256);
  const size_t off_ctl = align_up(off_ranges + sizeof(int32_t) * ranges.size(), 256);
  const size_t ctl_words = 4 + static_cast<size_t>(n_ops) + static_cast<size_t>(pl.counters);
  const size_t off_part = align_up(off_ctl + sizeof(uint32_t) * ctl_words, 256);
  const size_t total = off_part + sizeof(float) * kRedFloats * static_cast<size_t>(std::max(pl.slots, 1));

  TfChain* ch = new (std::nothrow) TfChain();
  if (!ch) return TF_ERR_INVALID_ARG;
  ch->device = dev;
  ch->grid = sms;
  const int x_stride = pl.max_chunks * kChunkK + 8;
  ch->smem = static_cast<size_t>(kAlignSlack + kOffX) +
             std::max(static_cast<size_t>(M) * x_stride * 2, static_cast<size_t>(kRedBytes));
  e = cudaMalloc(&ch->mem, total);
  char* base = static_cast<char*>(ch->mem);
  if (e == cudaSuccess)
    e = cudaMemcpy(base + off_ops, hops.data(), sizeof(ChainOpDev) * n_ops, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(base + off_units, hunits.data(), sizeof(ChainUnitDev) * hunits.size(),
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(base + off_ranges, ranges.data(), sizeof(int32_t) * ranges.size(),
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(base + off_ctl, 0, sizeof(uint32_t) * ctl_words);
  // The attribute is the cap, not this chain's size: chains of different sizes share the kernel.
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(w4a16_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemCap);
  int per_sm = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, w4a16_chain_kernel, kThreads,
                                                      ch->smem);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    last_cuda_error() = static_cast<int>(e);
    if (ch->mem) cudaFree(ch->mem);
    delete ch;
    return e != cudaSuccess ? TF_ERR_CUDA : TF_ERR_UNSUPPORTED;
  }
  ChainParams& p = ch->params;
  p.ops = reinterpret_cast<const ChainOpDev*>(base + off_ops);
  p.units = reinterpret_cast<const ChainUnitDev*>(base + off_units);
  p.cta_units = reinterpret_cast<const int32_t*>(base + off_ranges);
  p.ctl = reinterpret_cast<uint32_t*>(base + off_ctl);
  p.done = p.ctl + 4;
  p.counters = p.done + n_ops;
  p.partials = reinterpret_cast<float*>(base + off_part);
  p.n_ops = n_ops;
  p.M = static_cast<int>(M);
  p.x_stride = x_stride;
  *out = ch;
  return TF_OK;
}

int tf_decode_chain_run(TfChain* chain, void* stream) {
  if (!chain) return TF_ERR_INVALID_ARG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(chain->grid));
  cfg.blockDim = dim3(tfb::kThreads);
  cfg.dynamicSmemBytes = chain->smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, tfb::w4a16_chain_kernel, chain->params);
  if (e != cudaSuccess) {
    cudaGetLastError();
    tfb::last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

int tf_decode_chain_error(TfChain* chain, int* out_code) {
  if (!chain || !out_code) return TF_ERR_INVALID_ARG;
  uint32_t v = 0;
  uint32_t* err = chain->params.ctl + 2;
  cudaError_t e = cudaMemcpy(&v, err, sizeof(v), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v != 0) e = cudaMemset(err, 0, sizeof(v));
  if (e != cudaSuccess) {
    cudaGetLastError();
    tfb::last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  *out_code = static_cast<int>(v);
  return TF_OK;
}

int tf_decode_chain_destroy(TfChain* chain) {
  if (!chain) return TF_ERR_INVALID_ARG;
  cudaError_t e = cudaSuccess;
  if (chain->mem) e = cudaFree(chain->mem);
  delete chain;
  if (e != cudaSuccess) {
    cudaGetLastError();
    tfb::last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

}  // extern "C"
