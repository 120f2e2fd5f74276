// Shared device helpers for the sm_100a quantized-linear kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tokenforge_b200.h"

namespace tfb {

// Host-side record of the last CUDA error (per thread), surfaced by tf_last_cuda_error().
int& last_cuda_error();

inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    last_cuda_error() = static_cast<int>(e);
    return TF_ERR_CUDA;
  }
  return TF_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Offset j (0..7) of a packed word lives in nibble (j % 2) * 4 + j / 2 (the AWQ interleave,
// reference tokenforge/kernels/pack.py:35).
__host__ __device__ __forceinline__ int awq_nibble_of(int j) { return (j & 1) * 4 + (j >> 1); }

// Zero-point of column n from an AWQ-packed qzeros row.
__device__ __forceinline__ uint32_t zero_of(const int32_t* qz_row, int64_t n) {
  const uint32_t w = static_cast<uint32_t>(__ldg(qz_row + (n >> 3)));
  return (w >> (4 * awq_nibble_of(static_cast<int>(n & 7)))) & 0xFu;
}

// Pair j (0..3) of a packed word as fp16x2 (1024 + q[2j], 1024 + q[2j+1]).
// Nibbles j and j+4 carry offsets 2j and 2j+1, so one mask plus the 0x6400 exponent pattern
// turns both into fp16 values without conversion instructions (compiles to one LOP3).
__device__ __forceinline__ uint32_t magic_pair(uint32_t w, int j) {
  return ((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) {
  return *reinterpret_cast<__half2*>(&u);
}

// fp16(q - z) * s with exactly one rounding, two lanes at a time: (1024+q) - (1024+z) is exact
// in fp16 and the product is correctly rounded by HMUL2 (dequant rule, pack.py:189-194).
__device__ __forceinline__ uint32_t dequant_pair(uint32_t magic_q, __half2 zz, __half2 ss) {
  return h2_as_u32(__hmul2(__hsub2(u32_as_h2(magic_q), zz), ss));
}

__device__ __forceinline__ __half2 zero_magic2(uint32_t z) {
  return u32_as_h2(0x64006400u | (z << 16) | z);
}

// Streaming 128-bit global load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// D = A * B + D, m16n8k16, fp16 inputs, fp32 accumulate (warp-synchronous).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Programmatic dependent launch: wait until the preceding grid on the stream has completed and
// its memory is visible (no-op when the kernel was not launched with the PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;");
}

// fp32 pair -> e4m3x2, round-to-nearest-even with saturation to +-448 (NaN stays NaN).
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace tfb
