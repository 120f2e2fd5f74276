// C ABI entry points for W4A16 linear, launch planning and status reporting.
//
// The launch table replaces the reference's autotune cache and heuristic config
// (tokenforge/kernels/autotune.py:190-193, tokenforge/kernels/config.py:71-92): a fixed table
// indexed by M bucket picks the kernel family and token tile; N and K then fix the split of K
// across warps and CTAs by a closed-form rule. Nothing is measured or cached at run time, so a
// given (M, N, K, G) always launches the same grid and produces bit-identical output.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "tf_common.cuh"
#include "tf_plan.h"

namespace tfb {

int& last_cuda_error() {
  thread_local int e = 0;
  return e;
}

namespace {

uint32_t g_launch_flags = 0;

constexpr int kNumSms = 148;  // B200: 2 dies x 74 SMs

struct BucketEntry {
  int max_m;   // bucket upper bound
  int kernel;  // LinearKernel
  int tile_m;  // tokens per CTA tile
};

// Fixed per-M-bucket launch table. Buckets 1..128 are the reference's M_BUCKETS
// (config.py:8); larger buckets extend it to the prefill sizes of the benchmark configs.
constexpr BucketEntry kTable[] = {
    {1, kKernelGemv, 8},      {2, kKernelGemv, 8},      {4, kKernelGemv, 8},
    {8, kKernelGemv, 8},      {16, kKernelGemv, 16},    {32, kKernelTcGemm, 32},
    {64, kKernelTcGemm, 64},  {128, kKernelTcGemm, 128}, {256, kKernelTcGemm, 256},
    {512, kKernelTcGemm, 256}, {1024, kKernelTcGemm, 256}, {2048, kKernelTcGemm, 256},
    {4096, kKernelTcGemm, 256}, {1 << 30, kKernelTcGemm, 256},
};

// Decode GEMV: 32-row warp tiles over 128-wide K blocks, K split over WARPS_K warps of an 8-warp
// CTA and over the C CTAs of a cluster. (WARPS_K, C) is the pair that brings the CTA count closest to two
// per SM without exceeding it (ties: fewer warps per tile, then smaller clusters), keeping at least
// one block per warp. C grows further if the CTA's staged activations would exceed 100 KB of
// shared memory; beyond clusters of 8, K is also split across clusters (fp32 partials + reduce).
int plan_gemv(int64_t M, int64_t N, int64_t K, LinearPlan* pl) {
  pl->tile_m = M > 8 ? 16 : 8;  // 16: two 8-token MMA n-tiles per warp
  pl->tile_n = 32;
  const int64_t n_tiles = cdiv(N, 32);
  const int64_t kblocks = cdiv(K, 128);
  const int64_t target = 2 * kNumSms;
  auto x_bytes = [&](int64_t sp) { return 2 * M * (cdiv(kblocks, sp) * 128 + 8); };
  const int64_t x_cap = M > 8 ? 96 * 1024 : 100 * 1024;
  // 16 tokens: the CTA search prefers K shares whose activations stay within 64 KB per CTA
  // (measured: gate_up at M = 12 staged 86 KB per CTA and ran 37% slower than with a 2-CTA
  // cluster); x_cap still bounds what a cluster of 8 may stage.
  const int64_t x_soft = 64 * 1024;
  int best_wk = 1, best_c = 1;
  int64_t best_ctas = -1;
  for (int c = 1; c <= 8; c *= 2) {
    for (int wk = 1; wk <= 8; wk *= 2) {
      if (static_cast<int64_t>(wk) * c > kblocks && !(wk == 1 && c == 1)) continue;
      // 16 tokens: count the cluster's K split toward the staged activations' cap here, so the
      // CTA count is not doubled after the choice (M <= 8 keeps its measured plans).
      if (M > 8 && c < 8 && x_bytes(c) > x_soft && !(wk == 1 && c == 1)) continue;
      const int64_t ctas = cdiv(n_tiles, 8 / wk) * c;
      if (ctas > target && !(wk == 1 && c == 1)) continue;
      const bool better = ctas > best_ctas ||
                          (ctas == best_ctas && static_cast<int64_t>(wk) * c <
                                                    static_cast<int64_t>(best_wk) * best_c);
      if (better) {
        best_ctas = ctas;
        best_wk = wk;
        best_c = c;
      }
    }
  }
  // Shared-memory bound on the staged activations: M x (K / splits) fp16 <= 100 KB (96 KB for
  // the 16-token kernel, whose reduction buffer is 16 KB), so that two CTAs fit an SM.
  int64_t splits = best_c;
  while (x_bytes(splits) > x_cap && splits < kblocks) splits *= 2;
  int cluster = static_cast<int>(std::min<int64_t>(splits, 8));
  const int64_t per = cdiv(kblocks, splits);
  splits = cdiv(kblocks, per);
  if (splits % cluster != 0) splits = cdiv(splits, cluster) * cluster;  // whole clusters
  // A cluster of two 8-warp CTAs that each take one row tile is one 16-warp CTA (one per SM)
  // splitting K 16 ways: same warps, but the split is summed in shared memory instead of
  // through two cluster barriers (about 1 us per launch). Its staged activations may use most
  // of the SM's shared memory.
  if (M <= 8 && best_wk == 8 && cluster == 2 && splits == 2 && x_bytes(1) <= 200 * 1024) {
    best_wk = 16;
    cluster = 1;
    splits = 1;
  }
  const int64_t per_split = cdiv(kblocks, splits);
  const int64_t gx = cdiv(n_tiles, gemv_warps_n(best_wk));
  if (gx > 0x7fffffffLL || splits > 65535) return TF_ERR_UNSUPPORTED;
  pl->warps_k = best_wk;
  pl->cluster = cluster;
  pl->split_k = static_cast<int>(splits);
  pl->blocks_per_split = static_cast<int>(per_split);
  pl->grid_x = static_cast<unsigned>(gx);
  pl->grid_y = static_cast<unsigned>(splits);
  pl->grid_z = 1;
  const int64_t outer = splits / cluster;
  pl->workspace = outer > 1 ? static_cast<size_t>(outer * M * N) * sizeof(float) : 0;
  return TF_OK;
}

// 64-token warp-MMA tiles: 16-row warp tiles, 128-wide K blocks split over up to 8 warps.
int plan_mma(int64_t M, int64_t N, int64_t K, LinearPlan* pl) {
  pl->tile_m = 64;
  pl->tile_n = 16;
  const int64_t n_tiles = cdiv(N, 16);
  const int64_t kblocks = cdiv(K, 128);
  int wk = 8;
  while (wk > 1 && 2 * wk > kblocks) wk >>= 1;
  pl->warps_k = wk;
  const int wn = 8 / wk;
  const int64_t gx = cdiv(n_tiles, wn);
  const int64_t gz = cdiv(M, 64);
  const int64_t ctas = gx * gz;
  int64_t split = 1;
  if (ctas < kNumSms && kblocks >= 4 * wk) {
    split = std::min<int64_t>(8, cdiv(2 * kNumSms, ctas));
    split = std::min<int64_t>(split, kblocks / (2 * wk));
    split = std::max<int64_t>(split, 1);
  }
  const int64_t per = cdiv(kblocks, split);
  split = cdiv(kblocks, per);
  if (gx > 0x7fffffffLL || gz > 65535 || split > 65535) return TF_ERR_UNSUPPORTED;
  pl->split_k = static_cast<int>(split);
  pl->cluster = 1;
  pl->blocks_per_split = static_cast<int>(per);
  pl->grid_x = static_cast<unsigned>(gx);
  pl->grid_y = static_cast<unsigned>(split);
  pl->grid_z = static_cast<unsigned>(gz);
  pl->workspace = split > 1 ? static_cast<size_t>(split * M * N) * sizeof(float) : 0;
  return TF_OK;
}

// The decode GEMV indexes with 32-bit integers.
bool gemv_fits(int64_t M, int64_t N, int64_t K, int64_t ldx, int group_size) {
  const int64_t lim = int64_t(1) << 31;
  return N * (K / 8) < lim && (K / group_size + 1) * N < lim && M * ldx < lim && K < lim;
}

}  // namespace

uint32_t launch_flags() { return g_launch_flags; }

int plan_linear(int64_t M, int64_t N, int64_t K, int group_size, LinearPlan* pl) {
  if (M < 1 || N < 1 || K < 1) return TF_ERR_INVALID_ARG;
  if (group_size != 32 && group_size != 64 && group_size != 128) return TF_ERR_INVALID_ARG;
  if (N % 8 != 0 || K % group_size != 0) return TF_ERR_INVALID_ARG;
  *pl = LinearPlan{};
  int idx = 0;
  while (M > kTable[idx].max_m) ++idx;
  pl->m_bucket = kTable[idx].max_m;
  pl->kernel = kTable[idx].kernel;
  if (pl->kernel == kKernelTcGemm && !tc_gemm_supported(M, N, K, group_size))
    pl->kernel = kKernelMmaGemm;
  if (pl->kernel == kKernelGemv && M > 8 && group_size != 128) {
    // The 16-token GEMV folds one scale per 128-wide block: other group sizes take a GEMM.
    pl->kernel = tc_gemm_supported(M, N, K, group_size) ? kKernelTcGemm : kKernelMmaGemm;
  }
  if (pl->kernel == kKernelGemv && !gemv_fits(M, N, K, K, group_size))
    pl->kernel = kKernelMmaGemm;
  if (pl->kernel == kKernelTcGemm) {
    pl->tile_m = kTable[idx].tile_m;
    plan_tc(M, N, K, pl);
    return TF_OK;
  }
  if (pl->kernel == kKernelGemv) return plan_gemv(M, N, K, pl);
  return plan_mma(M, N, K, pl);
}

namespace {

int validate_linear(const LinearArgs& a) {
  if (a.M < 0 || a.N < 1 || a.K < 1) return TF_ERR_INVALID_ARG;
  if (a.group_size != 32 && a.group_size != 64 && a.group_size != 128) return TF_ERR_INVALID_ARG;
  if (a.N % 8 != 0 || a.K % a.group_size != 0) return TF_ERR_INVALID_ARG;
  if (a.ldx < a.K || a.ldy < a.N) return TF_ERR_INVALID_ARG;
  if (a.M == 0) return TF_OK;
  if (!a.x || !a.qw || !a.scales || !a.qzeros || !a.y) return TF_ERR_INVALID_ARG;
  // fp16 activations are read 16 bytes at a time, e4m3 codes 8 bytes at a time.
  const uintptr_t x_align = a.x8 != nullptr ? 8 : 16;
  if (reinterpret_cast<uintptr_t>(a.x) % x_align != 0 || a.ldx % 8 != 0 || !aligned16(a.qw))
    return TF_ERR_ALIGNMENT;
  return TF_OK;
}

int run_linear(const LinearArgs& a, cudaStream_t stream, int force_kernel) {
  int st = validate_linear(a);
  if (st != TF_OK || a.M == 0) return st;
  LinearPlan pl;
  st = plan_linear(a.M, a.N, a.K, a.group_size, &pl);
  if (st != TF_OK) return st;
  if (force_kernel == kKernelGemv && a.M > 8) return TF_ERR_UNSUPPORTED;
  if (force_kernel == kKernelGemv && pl.kernel != kKernelGemv) return TF_ERR_UNSUPPORTED;
  if (force_kernel == kKernelTcGemm && pl.kernel == kKernelGemv) {
    // tf_w4a16_gemm on a decode-sized M: run the tensor-core GEMM when it supports the shape.
    if (!tc_gemm_supported(a.M, a.N, a.K, a.group_size)) {
      pl.kernel = kKernelMmaGemm;
      st = plan_mma(a.M, a.N, a.K, &pl);
      if (st != TF_OK) return st;
    } else {
      pl.kernel = kKernelTcGemm;
      pl.tile_m = 16;
      plan_tc(a.M, a.N, a.K, &pl);
    }
  }
  if (pl.kernel == kKernelGemv && !gemv_fits(a.M, a.N, a.K, a.ldx, a.group_size)) {
    pl.kernel = kKernelMmaGemm;
    st = plan_mma(a.M, a.N, a.K, &pl);
    if (st != TF_OK) return st;
  }
  if (a.peers != nullptr) {
    // The fused all-reduce needs the single-launch GEMV plan, every CTA resident at once (peers
    // wait on each other's tiles) and the mailbox capacity.
    const int64_t ctas = static_cast<int64_t>(pl.grid_x) * pl.split_k;
    const int64_t resident = pl.warps_k >= 16 ? kNumSms : 2 * kNumSms;
    if (pl.kernel != kKernelGemv || pl.split_k != pl.cluster || pl.cluster > 2 ||
        ctas > resident || a.M > a.peers->max_m || a.N > a.peers->max_n)
      return TF_ERR_UNSUPPORTED;
  }
  if (pl.workspace > 0 && (a.workspace == nullptr || a.workspace_bytes < pl.workspace))
    return TF_ERR_WORKSPACE;
  if (pl.kernel == kKernelTcGemm) return launch_tc_gemm(pl, a, stream);
  if (pl.kernel == kKernelGemv) return launch_gemv(pl, a, stream);
  return launch_mma_tiles(pl, a, stream);
}

LinearArgs make_args(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, const int32_t* qw,
                     const uint16_t* scales, const int32_t* qzeros, const uint16_t* bias,
                     int64_t N, int32_t G, uint16_t* y, int64_t ldy, void* ws, size_t wsb) {
  LinearArgs a;
  a.peers = nullptr;
  a.x8 = nullptr;
  a.x_scale = nullptr;
  a.x_scale_stride = 0;
  a.norm_w = nullptr;
  a.norm_eps = 0.f;
  a.norm_static = nullptr;
  a.norm_scale_out = nullptr;
  a.silu = 0;
  a.x = x;
  a.M = M;
  a.K = K;
  a.ldx = ldx;
  a.qw = qw;
  a.scales = scales;
  a.qzeros = qzeros;
  a.bias = bias;
  a.N = N;
  a.group_size = G;
  a.y = y;
  a.ldy = ldy;
  a.workspace = ws;
  a.workspace_bytes = wsb;
  return a;
}

// Fixed scratch of tf_w4a16_linear_noalloc. Callers of that entry point own no allocator at the
// call site (an engine that sized all of its device memory up front, or C code without torch), so
// the split-K partials live in this array, which the module loader places in device memory with
// the kernels. 16 MiB covers every decode plan and prefill plans up to a few hundred tokens at
// the benchmark's widths; larger plans are refused, not truncated.
constexpr size_t kNoallocScratchBytes = 16u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device, looked up once per device.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return TF_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      last_cuda_error() = static_cast<int>(e);
      return TF_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return TF_OK;
}

}  // namespace
}  // namespace tfb

static_assert(tfb::kNoallocScratchBytes == TF_NOALLOC_SCRATCH_BYTES,
              "header and library disagree on the fixed scratch size");

extern "C" {

const char* tf_status_string(int status) {
  switch (status) {
    case TF_OK: return "ok";
    case TF_ERR_INVALID_ARG: return "invalid argument";
    case TF_ERR_ALIGNMENT: return "operand not 16-byte aligned";
    case TF_ERR_WORKSPACE: return "workspace missing or too small";
    case TF_ERR_UNSUPPORTED: return "shape not supported by this kernel";
    case TF_ERR_CUDA: return "CUDA runtime error";
    case TF_ERR_NO_DEVICE: return "current device is not sm_100";
    case TF_ERR_TOO_LARGE: return "size exceeds the entry point's fixed capacity";
    default: return "unknown status";
  }
}

int tf_last_cuda_error(void) { return tfb::last_cuda_error(); }

int tf_abi_version(void) { return 1; }

void tf_set_launch_flags(uint32_t flags) { tfb::g_launch_flags = flags; }
uint32_t tf_get_launch_flags(void) { return tfb::g_launch_flags; }

size_t tf_w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t group_size) {
  tfb::LinearPlan pl;
  if (M < 1) return 0;
  if (tfb::plan_linear(M, N, K, group_size, &pl) != TF_OK) return 0;
  // The GEMM entry may fall back to the 64-token MMA kernel; size for the larger of the two.
  tfb::LinearPlan alt = pl;
  size_t ws = pl.workspace;
  if (tfb::plan_mma(M, N, K, &alt) == TF_OK && alt.workspace > ws) ws = alt.workspace;
  if (M <= 8 && tfb::plan_gemv(M, N, K, &alt) == TF_OK && alt.workspace > ws) ws = alt.workspace;
  if (tfb::tc_gemm_supported(M, N, K, group_size)) {
    alt.tile_m = 16;
    tfb::plan_tc(M, N, K, &alt);
    if (alt.workspace > ws) ws = alt.workspace;
  }
  return ws;
}

int tf_launch_plan(int64_t M, int64_t N, int64_t K, int32_t group_size, int32_t* out) {
  if (!out) return TF_ERR_INVALID_ARG;
  tfb::LinearPlan pl;
  const int st = tfb::plan_linear(M, N, K, group_size, &pl);
  if (st != TF_OK) return st;
  out[0] = pl.kernel;
  out[1] = pl.m_bucket;
  out[2] = pl.tile_n;
  out[3] = pl.warps_k;
  out[4] = pl.split_k;
  out[5] = pl.tile_m;
  out[6] = static_cast<int32_t>(pl.grid_x);
  out[7] = static_cast<int32_t>(pl.grid_z);
  out[8] = pl.cluster;
  return TF_OK;
}

int tf_w4a16_gemv(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, const int32_t* qweight_t,
                  const uint16_t* scales, const int32_t* qzeros, const uint16_t* bias, int64_t N,
                  int32_t group_size, uint16_t* y, int64_t ldy, void* workspace,
                  size_t workspace_bytes, void* stream) {
  const auto a = tfb::make_args(x, M, K, ldx, qweight_t, scales, qzeros, bias, N, group_size, y,
                                ldy, workspace, workspace_bytes);
  return tfb::run_linear(a, static_cast<cudaStream_t>(stream), tfb::kKernelGemv);
}

int tf_w4a16_gemm(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, const int32_t* qweight_t,
                  const uint16_t* scales, const int32_t* qzeros, const uint16_t* bias, int64_t N,
                  int32_t group_size, uint16_t* y, int64_t ldy, void* workspace,
                  size_t workspace_bytes, void* stream) {
  const auto a = tfb::make_args(x, M, K, ldx, qweight_t, scales, qzeros, bias, N, group_size, y,
                                ldy, workspace, workspace_bytes);
  return tfb::run_linear(a, static_cast<cudaStream_t>(stream), tfb::kKernelTcGemm);
}

int tf_w4a16_linear(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                    const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                    const uint16_t* bias, int64_t N, int32_t group_size, uint16_t* y, int64_t ldy,
                    void* workspace, size_t workspace_bytes, void* stream) {
  const auto a = tfb::make_args(x, M, K, ldx, qweight_t, scales, qzeros, bias, N, group_size, y,
                                ldy, workspace, workspace_bytes);
  return tfb::run_linear(a, static_cast<cudaStream_t>(stream), -1);
}

size_t tf_peer_mailbox_bytes(int32_t world, int32_t max_m, int32_t max_n) {
  if (world < 2 || world > TF_MAX_PEERS || max_m < 1 || max_m > 8 || max_n < 8) return 0;
  return tfb::peer_layout(world, max_m, max_n).bytes;
}

int tf_peer_mailbox_alloc(size_t bytes, void** mailbox, void* ipc_handle) {
  if (bytes == 0 || !mailbox || !ipc_handle) return TF_ERR_INVALID_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == TF_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    tfb::last_cuda_error() = static_cast<int>(e);
    cudaGetLastError();
    return TF_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *mailbox = p;
  return TF_OK;
}

int tf_peer_mailbox_open(const void* ipc_handle, void** mailbox) {
  if (!ipc_handle || !mailbox) return TF_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(mailbox, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    cudaGetLastError();
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

int tf_peer_mailbox_close(void* peer_mailbox) {
  if (!peer_mailbox) return TF_ERR_INVALID_ARG;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_mailbox);
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    cudaGetLastError();
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

int tf_peer_mailbox_free(void* mailbox) {
  if (!mailbox) return TF_ERR_INVALID_ARG;
  const cudaError_t e = cudaFree(mailbox);
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    cudaGetLastError();
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

int tf_peer_mailbox_error(void* mailbox, int* out_code) {
  if (!mailbox || !out_code) return TF_ERR_INVALID_ARG;
  uint32_t* err = static_cast<uint32_t*>(mailbox) + 2;
  uint32_t v = 0;
  cudaError_t e = cudaMemcpy(&v, err, sizeof(v), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v != 0) e = cudaMemset(err, 0, sizeof(v));
  if (e != cudaSuccess) {
    tfb::last_cuda_error() = static_cast<int>(e);
    cudaGetLastError();
    return TF_ERR_CUDA;
  }
  *out_code = static_cast<int>(v);
  return TF_OK;
}

int tf_w4a16_linear_allreduce(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                              const int32_t* qweight_t, const uint16_t* scales,
                              const int32_t* qzeros, const uint16_t* bias, int64_t N,
                              int32_t group_size, uint16_t* y, int64_t ldy, void* workspace,
                              size_t workspace_bytes, const TfPeerSet* peers, void* stream) {
  if (!peers || peers->world < 2 || peers->world > TF_MAX_PEERS || peers->rank < 0 ||
      peers->rank >= peers->world || peers->max_m < 1 || peers->max_m > 8 || peers->max_n < 8)
    return TF_ERR_INVALID_ARG;
  for (int q = 0; q < peers->world; ++q)
    if (!peers->mailbox[q]) return TF_ERR_INVALID_ARG;
  auto a = tfb::make_args(x, M, K, ldx, qweight_t, scales, qzeros, bias, N, group_size, y, ldy,
                          workspace, workspace_bytes);
  a.peers = peers;
  return tfb::run_linear(a, static_cast<cudaStream_t>(stream), tfb::kKernelGemv);
}

size_t tf_w4a16_fp8_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t group_size) {
  if (M < 1 || K < 1) return 0;
  const size_t lin = tf_w4a16_workspace_bytes(M, N, K, group_size);
  if (M <= 8) return lin;
  const size_t x16 = (static_cast<size_t>(M) * K * 2 + 255) / 256 * 256;
  return x16 + lin;
}

int tf_w4a16_linear_fp8(const uint8_t* xq, const float* x_scale, int64_t scale_stride, int64_t M,
                        int64_t K, int64_t ldx, const int32_t* qweight_t, const uint16_t* scales,
                        const int32_t* qzeros, const uint16_t* bias, int64_t N,
                        int32_t group_size, uint16_t* y, int64_t ldy, void* workspace,
                        size_t workspace_bytes, void* stream_) {
  using namespace tfb;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (scale_stride != 0 && scale_stride != 1) return TF_ERR_INVALID_ARG;
  if (M < 0 || K < 1 || ldx < K) return TF_ERR_INVALID_ARG;
  if (M == 0) return TF_OK;
  if (!xq || !x_scale) return TF_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(xq) % 8 != 0 || ldx % 8 != 0) return TF_ERR_ALIGNMENT;
  LinearPlan pl;
  int st = plan_linear(M, N, K, group_size, &pl);
  if (st != TF_OK) return st;
  if (pl.kernel == kKernelGemv && gemv_fits(M, N, K, K, group_size) && M * ldx < (int64_t(1) << 31)) {
    // Decode: the GEMV stages the codes exactly and scales y in fp32.
    auto a = make_args(reinterpret_cast<const uint16_t*>(xq), M, K, K, qweight_t, scales, qzeros,
                       bias, N, group_size, y, ldy, workspace, workspace_bytes);
    a.ldx = ldx;
    a.x8 = xq;
    a.x_scale = x_scale;
    a.x_scale_stride = scale_stride;
    st = validate_linear(a);
    if (st != TF_OK) return st;
    if (pl.workspace > 0 && (workspace == nullptr || workspace_bytes < pl.workspace))
      return TF_ERR_WORKSPACE;
    return launch_gemv(pl, a, stream);
  }
  // Prefill: x16 = fp16(e4m3 * scale) in the workspace, then the regular launch table.
  const size_t x16_bytes = (static_cast<size_t>(M) * K * 2 + 255) / 256 * 256;
  if (workspace == nullptr || workspace_bytes < x16_bytes) return TF_ERR_WORKSPACE;
  uint16_t* x16 = static_cast<uint16_t*>(workspace);
  st = launch_fp8_to_fp16(xq, M, K, ldx, x_scale, scale_stride, x16, K, stream);
  if (st != TF_OK) return st;
  const auto a = make_args(x16, M, K, K, qweight_t, scales, qzeros, bias, N, group_size, y, ldy,
                           static_cast<char*>(workspace) + x16_bytes,
                           workspace_bytes - x16_bytes);
  return run_linear(a, stream, -1);
}

int tf_rmsnorm_fp8_w4a16_linear(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                                const uint16_t* norm_weight, float eps,
                                const float* static_scale, float* scale_out,
                                const int32_t* qweight_t, const uint16_t* scales,
                                const int32_t* qzeros, const uint16_t* bias, int64_t N,
                                int32_t group_size, uint16_t* y, int64_t ldy, void* workspace,
                                size_t workspace_bytes, void* stream) {
  using namespace tfb;
  if (M < 0 || K < 1) return TF_ERR_INVALID_ARG;
  if (M == 0) return TF_OK;
  if (!norm_weight) return TF_ERR_INVALID_ARG;
  if (M > 8 || K % 8 != 0) return TF_ERR_UNSUPPORTED;
  if (!aligned16(norm_weight)) return TF_ERR_ALIGNMENT;
  auto a = make_args(x, M, K, ldx, qweight_t, scales, qzeros, bias, N, group_size, y, ldy,
                     workspace, workspace_bytes);
  a.norm_w = norm_weight;
  a.norm_eps = eps;
  a.norm_static = static_scale;
  a.norm_scale_out = static_scale ? nullptr : scale_out;
  int st = validate_linear(a);
  if (st != TF_OK) return st;
  LinearPlan pl;
  st = plan_linear(M, N, K, group_size, &pl);
  if (st != TF_OK) return st;
  // One pass: every CTA must hold whole rows (no K split across CTAs).
  if (pl.kernel != kKernelGemv || !gemv_fits(M, N, K, ldx, group_size) || pl.split_k != 1 ||
      pl.cluster != 1)
    return TF_ERR_UNSUPPORTED;
  if (pl.workspace > 0 && (workspace == nullptr || workspace_bytes < pl.workspace))
    return TF_ERR_WORKSPACE;
  return launch_gemv(pl, a, static_cast<cudaStream_t>(stream));
}

int tf_silu_mul_w4a16_linear(const uint16_t* gate_up, int64_t M, int64_t K, int64_t ld,
                             const int32_t* qweight_t, const uint16_t* scales,
                             const int32_t* qzeros, const uint16_t* bias, int64_t N,
                             int32_t group_size, uint16_t* y, int64_t ldy, void* workspace,
                             size_t workspace_bytes, void* stream) {
  using namespace tfb;
  if (M < 0 || K < 1 || ld < 2 * K) return TF_ERR_INVALID_ARG;
  if (M == 0) return TF_OK;
  if (M > 8 || K % 8 != 0) return TF_ERR_UNSUPPORTED;
  auto a = make_args(gate_up, M, K, ld, qweight_t, scales, qzeros, bias, N, group_size, y, ldy,
                     workspace, workspace_bytes);
  a.silu = 1;
  int st = validate_linear(a);
  if (st != TF_OK) return st;
  LinearPlan pl;
  st = plan_linear(M, N, K, group_size, &pl);
  if (st != TF_OK) return st;
  if (pl.kernel != kKernelGemv || !gemv_fits(M, N, K, ld, group_size) || pl.split_k != 1 ||
      pl.cluster != 1 || M * ld >= (int64_t(1) << 31))
    return TF_ERR_UNSUPPORTED;
  if (pl.workspace > 0 && (workspace == nullptr || workspace_bytes < pl.workspace))
    return TF_ERR_WORKSPACE;
  return launch_gemv(pl, a, static_cast<cudaStream_t>(stream));
}

int tf_w4a16_linear_noalloc(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                            const int32_t* qweight_t, const uint16_t* scales,
                            const int32_t* qzeros, const uint16_t* bias, int64_t N,
                            int32_t group_size, uint16_t* y, int64_t ldy, void* stream) {
  auto a = tfb::make_args(x, M, K, ldx, qweight_t, scales, qzeros, bias, N, group_size, y, ldy,
                          nullptr, 0);
  int st = tfb::validate_linear(a);
  if (st != TF_OK || M == 0) return st;
  void* scratch = nullptr;
  st = tfb::noalloc_scratch(&scratch);
  if (st != TF_OK) return st;
  a.workspace = scratch;
  a.workspace_bytes = tfb::kNoallocScratchBytes;
  st = tfb::run_linear(a, static_cast<cudaStream_t>(stream), -1);
  // The scratch is never null here, so a workspace refusal means the plan outgrew it.
  return st == TF_ERR_WORKSPACE ? TF_ERR_TOO_LARGE : st;
}

}  // extern "C"
