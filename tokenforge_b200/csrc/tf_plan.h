// Host-side launch plan shared by the C ABI and the kernels' launchers.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/tokenforge_b200.h"

namespace tfb {

enum LinearKernel : int {
  kKernelGemv = 0,     // decode GEMV (M <= 8): activations in shared memory, warp-level MMA
  kKernelMmaGemm = 1,  // warp-level MMA, 64-token tiles
  kKernelTcGemm = 2,   // tcgen05 + TMEM + TMA tensor-core GEMM
};

struct LinearPlan {
  int kernel;
  int m_bucket;          // smallest launch-table bucket >= M
  int tile_n;            // weight rows per warp tile (mma) or per CTA tile (tcgen05)
  int warps_k;           // warps splitting K inside one CTA (mma kernels)
  int split_k;           // CTAs splitting K (partials reduced in a fixed order)
  int cluster;           // of those, CTAs per thread-block cluster (reduced through DSMEM)
  int tile_m;            // tokens per CTA tile
  int blocks_per_split;  // K blocks per split: 256 wide (GEMV), 128 (MMA tiles), 64 (tcgen05)
  unsigned grid_x, grid_y, grid_z;
  size_t workspace;      // bytes of scratch the launch needs
  int stream_k;          // tcgen05 GEMM: stages dealt evenly over persistent CTAs (split_k 1)
};

// Fills `plan` for y[M, N] = x[M, K] * W[N, K]^T. Returns TF_OK or an error status.
int plan_linear(int64_t M, int64_t N, int64_t K, int group_size, LinearPlan* plan);

// Process-wide launch flags (tf_set_launch_flags).
uint32_t launch_flags();

// Status word of the RMSNorm streaming kernel's bounded waits (rmsnorm_fp8.cu).
int rms_device_error(int* code);
int rms_reset_device_error();

struct LinearArgs {
  const uint16_t* x;
  int64_t M, K, ldx;
  const int32_t* qw;
  const uint16_t* scales;
  const int32_t* qzeros;
  const uint16_t* bias;
  int64_t N;
  int group_size;
  uint16_t* y;
  int64_t ldy;
  void* workspace;
  size_t workspace_bytes;
  const TfPeerSet* peers;  // row-parallel all-reduce through peer mailboxes (null: none)
  // FP8 activations for the decode GEMV (x8 != null replaces x): e4m3 codes, row stride ldx
  // bytes, and the fp32 scale(s) multiplied into y before the bias.
  const uint8_t* x8;
  const float* x_scale;
  int64_t x_scale_stride;
  // Fused RMSNorm + FP8 prologue of the decode GEMV (norm_w != null): x is normalised with
  // norm_w and eps, quantised to e4m3 with the static scale (or per token, written to
  // norm_scale_out when not null), and the GEMV consumes the codes.
  const uint16_t* norm_w;
  float norm_eps;
  const float* norm_static;
  float* norm_scale_out;
  // Fused SiLU product (silu != 0): x is a gate_up output [M, 2K] with row stride ldx, and the
  // GEMV consumes fp16(silu(x[:, :K]) * x[:, K:]).
  int silu;
};

// One rank's mailbox: a 256-byte header (u32 call counter, arrival counter, error word), then
// per (call parity, source rank) a [max_m, max_n] array of 64-bit words, each an fp32 partial
// in the low half and the tag of the call that wrote it in the high half.
struct PeerLayout {
  size_t data_off, bytes;
};
inline PeerLayout peer_layout(int world, int max_m, int max_n) {
  PeerLayout l;
  l.data_off = 256;
  l.bytes = l.data_off + static_cast<size_t>(2) * world * max_m * max_n * 8;
  return l;
}

int launch_gemv(const LinearPlan& plan, const LinearArgs& a, cudaStream_t stream);
int launch_mma_tiles(const LinearPlan& plan, const LinearArgs& a, cudaStream_t stream);
// Row tiles (32 weight rows each) per decode-GEMV CTA for a plan's warps_k: CTAs are 8 warps
// (two per SM) with warps_k <= 8, or one 16-warp CTA per SM with warps_k == 16.
inline int gemv_warps_n(int warps_k) { return warps_k >= 16 ? 1 : 8 / warps_k; }
// Dynamic shared memory of the decode GEMV: M staged activation rows of bps * 128 (+8) fp16.
size_t gemv_smem_bytes(int64_t M, int bps);
int launch_tc_gemm(const LinearPlan& plan, const LinearArgs& a, cudaStream_t stream);
bool tc_gemm_supported(int64_t M, int64_t N, int64_t K, int group_size);
// Fills split_k / blocks_per_split / grid / workspace of a tensor-core plan whose tile_m is set.
void plan_tc(int64_t M, int64_t N, int64_t K, LinearPlan* plan);
// x16[m, k] = fp16(e4m3(xq[m, k]) * scale[m * stride]) (one rounding), row stride ldx16.
int launch_fp8_to_fp16(const uint8_t* xq, int64_t M, int64_t K, int64_t ldq, const float* scale,
                       int64_t stride, uint16_t* x16, int64_t ldx16, cudaStream_t stream);
// y[m, n] = fp16(sum_s partial[s, m, n] + bias[n]), splits summed in order 0..split-1.
int launch_splitk_reduce(const float* partial, int split, int64_t M, int64_t N,
                         const uint16_t* bias, uint16_t* y, int64_t ldy, cudaStream_t stream);

}  // namespace tfb
