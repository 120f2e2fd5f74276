/*
 * tokenforge_b200.h — C ABI of the B200 (sm_100a) quantized-linear backend.
 *
 * These entry points are the native boundary underneath the reference's custom ops
 * (`torch.ops.tokenforge.*`, reference file tokenforge/kernels/ops.py). Every function takes
 * plain device pointers, element counts and a CUDA stream handle (`cudaStream_t` passed as
 * `void*`; NULL is the legacy default stream), enqueues its work on that stream and returns
 * a status code without synchronising. No function reads tensor values on the host, so each
 * one can be recorded into a CUDA graph.
 *
 * Data types on the boundary:
 *   fp16 tensors are `uint16_t` bit patterns (IEEE binary16);
 *   e4m3 tensors are `uint8_t` bit patterns (OCP float8 e4m3fn, the torch.float8_e4m3fn codes);
 *   packed int4 tensors are `int32_t` words, eight 4-bit values per word in the AWQ nibble
 *   interleave (nibble i holds column/row offset (0,2,4,6,1,3,5,7)[i]).
 *
 * Tensor layouts (row-major, innermost dimension last):
 *   AWQ checkpoint  qweight   int32 [K, N/8]     packed along N
 *                   qzeros    int32 [K/G, N/8]   packed along N
 *                   scales    fp16  [K/G, N]
 *   kernel layout   qweight_t int32 [N, K/8]     packed along K, same nibble interleave
 *   activations     x         fp16  [M, K] with row stride ldx (elements), unit stride along K
 *   output          y         fp16  [M, N] with row stride ldy (elements)
 *
 * Alignment contract: every pointer to a 16-byte-vectorised operand (x, qweight_t, y, the
 * rmsnorm rows) must be 16-byte aligned and its row stride a multiple of 8 fp16 elements;
 * otherwise the call returns TF_ERR_ALIGNMENT and enqueues nothing (the Python layer copies
 * misaligned activations to an aligned buffer first).
 */
#ifndef TOKENFORGE_B200_H
#define TOKENFORGE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TF_API __attribute__((visibility("default")))
#else
#define TF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 0 is success; everything else enqueued no work unless stated. */
enum {
  TF_OK = 0,
  TF_ERR_INVALID_ARG = 1,   /* a size, group size or pointer argument is invalid */
  TF_ERR_ALIGNMENT = 2,     /* a vectorised operand is not 16-byte aligned */
  TF_ERR_WORKSPACE = 3,     /* workspace pointer missing or smaller than required */
  TF_ERR_UNSUPPORTED = 4,   /* shape outside what the kernels implement */
  TF_ERR_CUDA = 5,          /* a CUDA runtime call failed (see tf_last_cuda_error) */
  TF_ERR_NO_DEVICE = 6,     /* the current device is not compute capability 10.0 */
  TF_ERR_TOO_LARGE = 7      /* a size exceeds a fixed capacity of the entry point */
};

/* Human-readable text of a status code (static storage). */
TF_API const char* tf_status_string(int status);

/* The last CUDA runtime error seen by this library on the calling thread (cudaError_t value). */
TF_API int tf_last_cuda_error(void);

/* ABI version of this header; bumped on any signature change. */
TF_API int tf_abi_version(void);

/* Process-wide launch flags.
 * TF_LAUNCH_PDL: W4A16 linear kernels and the RMSNorm + FP8 quantizer are launched with
 *   programmatic dependent launch and start reading their weights (qweight_t, scales, qzeros;
 *   the RMSNorm weight) before the preceding kernel on the stream has finished (activations
 *   are read, and outputs written, only after it has). Set it only when no kernel enqueued
 *   directly before such a call on the same stream writes that call's weights. Off by
 *   default. */
#define TF_LAUNCH_PDL 1u
TF_API void tf_set_launch_flags(uint32_t flags);
TF_API uint32_t tf_get_launch_flags(void);

/* ------------------------------------------------------------------------- AWQ repack
 * Replaces repack_awq_to_tf (reference tokenforge/kernels/pack.py:141-143), the load-time
 * conversion inside pack_awq (pack.py:171-181).
 * qweight: int32 [K, N/8] AWQ layout  ->  qweight_t: int32 [N, K/8] kernel layout.
 * Bit-exact: output word (n, j) holds the eight values of column n at rows 8j..8j+7 in the
 * same nibble interleave. Requires K % 8 == 0, N % 8 == 0. */
TF_API int tf_awq_repack(const int32_t* qweight, int64_t K, int64_t N, int32_t* qweight_t,
                  void* stream);

/* Inverse, repack_tf_to_awq (pack.py:146-148): qweight_t [N, K/8] -> qweight [K, N/8]. */
TF_API int tf_awq_unrepack(const int32_t* qweight_t, int64_t N, int64_t K, int32_t* qweight,
                    void* stream);

/* Nibble codec of the AWQ interleave (pack_int4 / unpack_int4, pack.py:42-67).
 * unpack: packed int32 [n_words] -> int32 values [8 * n_words] in [0, 15], value 8w + j taken
 *         from nibble (j % 2) * 4 + j / 2 of word w.
 * pack:   int32 values [8 * n_words] -> packed int32 [n_words]; only the low 4 bits of each
 *         value are used (range checking belongs to the caller, as in pack.py:45-47). */
TF_API int tf_unpack_int4(const int32_t* packed, int64_t n_words, int32_t* values, void* stream);
TF_API int tf_pack_int4(const int32_t* values, int64_t n_words, int32_t* packed, void* stream);

/* ------------------------------------------------------------------------- dequant
 * Replaces the w4a16_dequant op (ops.py:110-120; Triton kernel triton/w4a16.py:118-146;
 * torch rule dequantize_tf pack.py:189-194).
 * out[n, k] = fp16(q[n, k] - z[k/G, n]) * s[k/G, n], one fp16 rounding: bit-exact.
 * out: fp16 [N, K] (nn.Linear.weight layout). group_size in {32, 64, 128}. */
TF_API int tf_w4a16_dequant(const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                     int64_t N, int64_t K, int32_t group_size, uint16_t* out, void* stream);

/* ------------------------------------------------------------------------- W4A16 linear
 * y[m, n] = sum_k x[m, k] * dequant(W)[n, k] (+ bias[n]), fp32 accumulation, fp16 output.
 *
 * tf_w4a16_gemv replaces the planned extension entry `_C.w4a16_gemv(x2, qweight_t, scales,
 * qzeros, bias, group_size)` named at ops.py:86-88 (decode, M = 1..8).
 * tf_w4a16_gemm runs the sm_100a tensor-core kernel at any M (prefill).
 * tf_w4a16_linear is the per-call dispatch of the w4a16_linear op (ops.py:48-94) through the
 * fixed per-M-bucket launch table (replacing autotune.lookup, autotune.py:190-193): the
 * decode GEMV for M <= 8, the 16-token GEMV for M = 9..16 at group size 128, the tensor-core
 * GEMM above.
 *
 * bias may be NULL. Workspace: tf_w4a16_workspace_bytes(M, N, K, group_size) bytes of device
 * memory (may be 0, then workspace may be NULL); contents need not be initialised (the
 * tensor-core GEMM's stream-K plans clear their ticket area with a cudaMemsetAsync on the
 * call's stream before the kernel); it must not be used by another call that runs
 * concurrently. */
TF_API size_t tf_w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t group_size);

TF_API int tf_w4a16_gemv(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                  const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                  const uint16_t* bias, int64_t N, int32_t group_size,
                  uint16_t* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                  void* stream);

TF_API int tf_w4a16_gemm(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                  const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                  const uint16_t* bias, int64_t N, int32_t group_size,
                  uint16_t* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                  void* stream);

TF_API int tf_w4a16_linear(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                    const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                    const uint16_t* bias, int64_t N, int32_t group_size,
                    uint16_t* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                    void* stream);

/* tf_w4a16_linear with no workspace argument: the split-K partials go to a fixed buffer the
 * library holds in device memory (a static __device__ array of TF_NOALLOC_SCRATCH_BYTES per
 * device). No counterpart in the reference. It is for callers that cannot allocate device memory
 * at the call site: a C/C++ engine that plans all its memory before serving and owns no
 * allocator at launch time, or a host without torch to hand out a workspace.
 * - Launches, output and error statuses are those of tf_w4a16_linear (same plan, same kernels).
 * - A shape whose plan needs more than TF_NOALLOC_SCRATCH_BYTES of partials (large prefill M
 *   with split K) returns TF_ERR_TOO_LARGE without launching; use tf_w4a16_linear for it.
 * - The first call on each device (current device) looks the buffer up once
 *   (cudaGetSymbolAddress, which may load the library's kernels); make that first call before
 *   any stream capture. The address is kept for the life of the process: after
 *   cudaDeviceReset (or anything else that destroys and re-creates the device's primary
 *   context) the kept address is stale, so do not call this entry point on that device again
 *   in the same process.
 * - The buffer needs no clearing: each split writes its whole slice before it is read.
 * - One buffer per device: calls that can overlap on the device (several streams, several host
 *   threads) race on it. Issue them on one stream, or use tf_w4a16_linear with a workspace
 *   each. */
#define TF_NOALLOC_SCRATCH_BYTES (16u << 20)
TF_API int tf_w4a16_linear_noalloc(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                    const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                    const uint16_t* bias, int64_t N, int32_t group_size,
                    uint16_t* y, int64_t ldy, void* stream);

/* ------------------------------------------------------------------ FP8 activations
 * W4A16 linear fed by rmsnorm_fp8_quant's output: x[m, k] = e4m3(xq[m, k]) * x_scale[m *
 * scale_stride] (scale_stride 1: the per-token fp32 scales, 0: one static scale), y as
 * tf_w4a16_linear. No reference counterpart: the reference produces e4m3 activations but has no
 * consumer for them (BASELINE config 4's block stack needs one).
 * Sizes the launch table serves with a GEMV (M <= 8; M <= 16 at group size 128): the codes are
 * staged as their exact fp16 values and y is scaled in fp32 before the bias, so the result is
 * as accurate as with fp16 activations x. Larger M: x16 = fp16(e4m3 * scale) (one rounding)
 * is written to the workspace, then the regular launch table runs on it. Workspace: tf_w4a16_fp8_workspace_bytes(M, N, K, group_size).
 * xq must be 8-byte aligned with ldx (bytes) % 8 == 0. */
TF_API size_t tf_w4a16_fp8_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t group_size);
TF_API int tf_w4a16_linear_fp8(const uint8_t* xq, const float* x_scale, int64_t scale_stride,
                    int64_t M, int64_t K, int64_t ldx, const int32_t* qweight_t,
                    const uint16_t* scales, const int32_t* qzeros, const uint16_t* bias, int64_t N,
                    int32_t group_size, uint16_t* y, int64_t ldy, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Fused RMSNorm + FP8 quantization + W4A16 linear for decode (M <= 8): one kernel computes
 *   (q, s) = rmsnorm_fp8_quant(x, norm_weight, eps, static_scale) and y = w4a16_linear_fp8(q, s),
 * with y bit-identical to calling tf_rmsnorm_fp8_quant and then tf_w4a16_linear_fp8. Each CTA
 * normalises and quantises the rows in its shared memory, so neither the codes nor the
 * normalised activations go to HBM and one launch replaces two. No reference counterpart: it is
 * the fused RMSNorm -> quant -> GEMV prologue that the reference's e4m3 output lacks a consumer
 * for. x: fp16 [M, K] (16-byte aligned, ldx % 8 == 0); norm_weight: fp16 [K], 16-byte aligned;
 * static_scale: one fp32 or NULL (dynamic per-token scales, written to scale_out [M] when it is
 * not NULL). Returns TF_ERR_UNSUPPORTED (launching nothing) for M > 8 and for layers whose
 * decode plan splits K across CTAs; the caller then makes the two calls. Workspace as
 * tf_w4a16_linear (none for the plans it accepts). Every CTA normalises all M rows itself, so
 * the fused call pays off at M <= 2; on B200 two calls are faster from M = 4 on. */
TF_API int tf_rmsnorm_fp8_w4a16_linear(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                    const uint16_t* norm_weight, float eps, const float* static_scale,
                    float* scale_out, const int32_t* qweight_t, const uint16_t* scales,
                    const int32_t* qzeros, const uint16_t* bias, int64_t N, int32_t group_size,
                    uint16_t* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                    void* stream);

/* W4A16 linear on the SiLU-gated product of a gate_up output, for decode (M <= 8):
 *   y = w4a16_linear(silu_mul(gate_up), W) in one kernel, bit-identical to tf_silu_mul followed
 * by tf_w4a16_linear. Each CTA computes the products of the K range it stages, so the [M, K]
 * intermediate never goes to HBM and one launch replaces two. No reference counterpart (it
 * serves the MLP of BASELINE config 4's block stack). gate_up: fp16 [M, 2K], 16-byte aligned,
 * row stride ld >= 2K with ld % 8 == 0; K is W's input size. Returns TF_ERR_UNSUPPORTED
 * (launching nothing) for M > 8 and for layers whose decode plan splits K across CTAs. */
TF_API int tf_silu_mul_w4a16_linear(const uint16_t* gate_up, int64_t M, int64_t K, int64_t ld,
                    const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                    const uint16_t* bias, int64_t N, int32_t group_size, uint16_t* y, int64_t ldy,
                    void* workspace, size_t workspace_bytes, void* stream);

/* SiLU-gated product of a fused gate_up projection (BASELINE config 4's block stack; no
 * reference counterpart): out[m, i] = fp16(silu(g) * u), g = gate_up[m, i],
 * u = gate_up[m, I + i], silu(g) = g / (1 + exp(-g)) in fp32. gate_up fp16 [M, 2I] with row
 * stride ld, out fp16 [M, I] with row stride ldo. */
TF_API int tf_silu_mul(const uint16_t* gate_up, int64_t M, int64_t I, int64_t ld, uint16_t* out,
                       int64_t ldo, void* stream);

/* ------------------------------------------------------- row-parallel all-reduce over NVLink
 * Tensor-parallel o / down layers (row-split K) end in a sum of every rank's fp16 partial
 * (NCCL all-reduce after o and down). tf_w4a16_linear_allreduce fuses that
 * sum into the decode GEMV: each rank's GEMV epilogue writes its fp32 partial tile straight into
 * every peer's mailbox (64-bit stores of value + call tag through CUDA IPC mappings over NVLink,
 * no multicast), polls its own mailbox (bounded, 2 s) for the peers' values of the same call and
 * sums the ranks' partials in rank order, so every rank writes the same y. No reference
 * counterpart: the reference has no multi-GPU code.
 *
 * Set-up, once per group (every rank, same order): tf_peer_mailbox_alloc on each rank, share
 * the IPC handles (e.g. an all-gather over the process group), tf_peer_mailbox_open the peers'
 * handles, fill a TfPeerSet. Ranks must be on distinct GPUs. Every rank must then issue the same
 * sequence of tf_w4a16_linear_allreduce calls (the mailbox counts calls on the device, so the
 * calls may be captured in a CUDA graph and replayed). Peers must reach each call within 2 s of
 * each other: a rank whose peer does not arrive in time records an error (read it with
 * tf_peer_mailbox_error) and writes an incomplete sum. */
#define TF_MAX_PEERS 8
#define TF_IPC_HANDLE_BYTES 64

typedef struct TfPeerSet {
  int32_t rank;                    /* this process's rank in [0, world) */
  int32_t world;                   /* 2..TF_MAX_PEERS */
  int32_t max_m;                   /* mailbox capacity: tokens (<= 8) ... */
  int32_t max_n;                   /* ... and output columns */
  void* mailbox[TF_MAX_PEERS];     /* rank q's mailbox mapped in this process; [rank] is local */
} TfPeerSet;

/* Bytes of one rank's mailbox for (world, max_m, max_n). */
TF_API size_t tf_peer_mailbox_bytes(int32_t world, int32_t max_m, int32_t max_n);
/* cudaMalloc + zero fill of `bytes` on the current device; writes the device pointer and the
 * TF_IPC_HANDLE_BYTES-byte IPC handle that peers open. */
TF_API int tf_peer_mailbox_alloc(size_t bytes, void** mailbox, void* ipc_handle);
/* Maps a peer's mailbox (cudaIpcOpenMemHandle) into this process. */
TF_API int tf_peer_mailbox_open(const void* ipc_handle, void** mailbox);
TF_API int tf_peer_mailbox_close(void* peer_mailbox);
TF_API int tf_peer_mailbox_free(void* mailbox);
/* Reads (*out_code: 0 = none) and clears the mailbox's error word (synchronous copy). */
TF_API int tf_peer_mailbox_error(void* mailbox, int* out_code);

/* y = sum over ranks of this rank's tf_w4a16_linear partial (bias given on one rank only).
 * Decode sizes only (the GEMV plan without a second reduce launch); other shapes return
 * TF_ERR_UNSUPPORTED and the caller uses tf_w4a16_linear plus a collective. */
TF_API int tf_w4a16_linear_allreduce(const uint16_t* x, int64_t M, int64_t K, int64_t ldx,
                    const int32_t* qweight_t, const uint16_t* scales, const int32_t* qzeros,
                    const uint16_t* bias, int64_t N, int32_t group_size,
                    uint16_t* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                    const TfPeerSet* peers, void* stream);

/* Tracing of the fused all-reduce (no reference counterpart): from the next call of
 * tf_w4a16_linear_allreduce on, in this process, each 32-row tile's storing warp writes four
 * %globaltimer stamps (ns) to records[4 * tile .. 4 * tile + 3]: entry to the exchange (its
 * partial sums done), its stores to every peer issued, the last peer word arrived, y written.
 * records: device memory of 4 * ceil(N / 32) uint64 on the calling device; NULL turns it off.
 * A launch captured in a CUDA graph keeps the pointer it was captured with. */
TF_API int tf_peer_trace(uint64_t* records);

/* Launch-table introspection (replaces config.default_config / GemmConfig, config.py:23-92).
 * Writes the launch chosen for (M, N, K, G) into out[0..8]:
 *   {kernel (0 = gemv, 1 = mma gemm, 2 = tcgen05 gemm), m_bucket, tile_n, warps_k, split_k,
 *    tile_m, grid_x, grid_z, cluster}. A gemv with tile_m 16 is the 16-token kernel (M 9..16).
 * Returns TF_OK or TF_ERR_INVALID_ARG. */
TF_API int tf_launch_plan(int64_t M, int64_t N, int64_t K, int32_t group_size, int32_t* out);

/* ------------------------------------------------------------------------- RMSNorm + FP8
 * Replaces rmsnorm_fp8_quant (ops.py:130-146; Triton kernel triton/rmsnorm_fp8.py:44-73;
 * torch rule reference.py:35-56).
 * Per row t: y = fp16(x * (1 / sqrt_rn(mean(x^2) + eps))) * weight (fp16 product), then
 *   dynamic (static_scale == NULL): scale[t] = max(amax|y| / 448, 1 / (448 * 512)), written
 *                                   to scale_out[t];
 *   static: scale = *static_scale (device pointer to one fp32), scale_out is not written;
 *   q = e4m3_rne_satfinite(clamp(y / scale, -448, 448)).
 * x: fp16 [T, H] row stride ldx; weight: fp16 [H]; q: e4m3 [T, H] contiguous. */
TF_API int tf_rmsnorm_fp8_quant(const uint16_t* x, int64_t T, int64_t H, int64_t ldx,
                         const uint16_t* weight, float eps, const float* static_scale,
                         uint8_t* q, float* scale_out, void* stream);

/* fp32 -> e4m3 (round to nearest even, saturating to +-448, NaN stays NaN), the exact cast
 * the quantizer uses. Mirrors the probe kernel of the reference's midpoint test
 * (tests/numerics/test_rmsnorm_fp8.py:22-27). */
TF_API int tf_cast_e4m3(const float* in, int64_t n, uint8_t* out, void* stream);

/* The quantization step of tf_rmsnorm_fp8_quant on its own, for activations already
 * normalised: q[r, c] = e4m3_rne_satfinite(clamp(y[r, c] / scale_r, -448, 448)) with the IEEE
 * fp32 division's rounding (reference tokenforge/kernels/reference.py:47-49).
 *   scale != NULL: scale_r = scale[r * scale_stride] (scale_stride 0: one static scale; 1: per
 *                  row); scale_out is not written;
 *   scale == NULL: dynamic, scale_r = max(amax_c |y[r, c]| / 448, 1 / (448 * 512)), written to
 *                  scale_out[r].
 * y: fp16 [R, C] row stride ldy; q: e4m3 [R, C] contiguous. No reference counterpart as a
 * separate op. */
TF_API int tf_e4m3_quant_rows(const uint16_t* y, int64_t R, int64_t C, int64_t ldy,
                              const float* scale, int64_t scale_stride, uint8_t* q,
                              float* scale_out, void* stream);

/* Device-side status word written by kernels whose waits are bounded: 0 = no error; 0x1xx the
 * tcgen05 GEMM (a pipeline wait gave up), 0x301 the RMSNorm + FP8 streaming kernel (a row's
 * bulk copy did not complete in time). Reading it synchronises the current device; resetting
 * writes 0. */
TF_API int tf_device_error(int* out_code);
TF_API int tf_reset_device_error(void);

/* ---------------------------------------------------------------- persistent decode chain
 *
 * A fixed sequence of W4A16 linears at decode sizes run as ONE persistent kernel (one CTA per
 * SM, cooperative launch), so that the weight stream of HBM continues across layer boundaries
 * instead of restarting at every launch. No counterpart in the reference, whose model code calls
 * the linear op once per layer (tokenforge/kernels/ops.py:48); each op of a chain computes what
 * tf_w4a16_linear computes for it, within the same tolerance (the K split, hence the fp32 sum
 * order, differs), and the chain is deterministic.
 *
 * Limits: 1 <= M <= 8 tokens, group size 128, every N a multiple of 32 and K a multiple of 128,
 * 16-byte aligned x / qweight_t / scales / qzeros, row strides multiples of 8 elements.
 *
 * `wait` nonzero: the op reads x only after every earlier op of the chain has finished (use it
 * when x is an earlier op's output). Ops without it must not read what an earlier op writes.
 *
 * tf_decode_chain_create allocates the chain's device tables (tensor maps, the unit schedule,
 * counters and the split-K partials) with cudaMalloc and synchronises the device; it records
 * the x, weight and y addresses, so later runs read and write those same buffers.
 * tf_decode_chain_run enqueues one launch on `stream` (graph-capturable). One chain must not run
 * on two streams at once (its counters are per chain). tf_decode_chain_error reads and clears the
 * chain's error word: nonzero means a bounded wait inside the kernel gave up (0x201: an op's
 * dependency; 0x202: a weight copy) and that run's outputs are undefined.
 */
typedef struct TfChainOp {
  const uint16_t* x;          /* fp16 [M, K], row stride ldx */
  int64_t ldx;
  const int32_t* qweight_t;   /* int32 [N, K/8] */
  const uint16_t* scales;     /* fp16 [K/128, N] */
  const int32_t* qzeros;      /* int32 [K/128, N/8] */
  const uint16_t* bias;       /* fp16 [N] or NULL */
  uint16_t* y;                /* fp16 [M, N], row stride ldy */
  int64_t ldy;
  int64_t N, K;
  int32_t wait;
  int32_t reserved;
} TfChainOp;

typedef struct TfChain TfChain;

TF_API int tf_decode_chain_create(const TfChainOp* ops, int32_t n_ops, int64_t M,
                                  int32_t group_size, TfChain** out);
TF_API int tf_decode_chain_run(TfChain* chain, void* stream);
TF_API int tf_decode_chain_error(TfChain* chain, int* out_code);
TF_API int tf_decode_chain_destroy(TfChain* chain);

/* The unit schedule tf_decode_chain_create would build for these shapes on `num_ctas` SMs
 * (host only, no GPU needed): one record per unit, in per-CTA order. Returns TF_ERR_TOO_LARGE
 * when `capacity` records do not hold them (n_units is set either way). */
typedef struct TfChainUnitInfo {
  int32_t cta, op, tile0, rtiles, c0, c1, piece, pieces, flags;
} TfChainUnitInfo;
TF_API int tf_decode_chain_plan(const int64_t* n, const int64_t* k, int32_t n_ops, int64_t M,
                                int32_t num_ctas, TfChainUnitInfo* out, int32_t capacity,
                                int32_t* n_units);

#ifdef __cplusplus
}
#endif

#endif /* TOKENFORGE_B200_H */
