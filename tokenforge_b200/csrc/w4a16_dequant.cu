// Full-weight dequantization: kernel layout -> fp16 [N, K] (the nn.Linear.weight layout).
//
// Rule (reference tokenforge/kernels/pack.py:189-194, Triton kernel triton/w4a16.py:118-146):
//   out[n, k] = fp16(q[n, k] - z[k/G, n]) * s[k/G, n]
// computed as HMUL2(HSUB2(1024 + q, 1024 + z), s): the subtraction is exact in fp16 and the
// product is rounded once, so the result is bit-identical to the reference for every input,
// including zero, subnormal and non-finite scales.
//
// One thread turns one 16-byte vector of qweight_t (32 values of one row, inside one group
// since G >= 32) into 64 bytes of fp16; consecutive threads walk along K, so both the packed
// reads and the fp16 writes are fully coalesced. HBM-bound: N*K/2 read + N*K*2 written.
#include "tf_common.cuh"

namespace tfb {
namespace {

__global__ void __launch_bounds__(256) w4a16_dequant_kernel(
    const uint4* __restrict__ qw, const __half* __restrict__ scales,
    const int32_t* __restrict__ qzeros, int64_t N, int64_t K, int group_size,
    uint4* __restrict__ out) {
  const int64_t vec_per_row = K / 32;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= N * vec_per_row) return;
  const int64_t n = idx / vec_per_row;
  const int64_t v = idx - n * vec_per_row;
  const int64_t g = (v * 32) / group_size;
  const uint4 w = ldg_stream_v4(qw + idx);
  const __half s = __ldg(scales + g * N + n);
  const uint32_t z = zero_of(qzeros + g * (N / 8), n);
  const __half2 zz = zero_magic2(z);
  const __half2 ss = __halves2half2(s, s);
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  uint4* dst = out + idx * 4;  // 32 fp16 = 4 x uint4
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 o;
    o.x = dequant_pair(magic_pair(words[i], 0), zz, ss);
    o.y = dequant_pair(magic_pair(words[i], 1), zz, ss);
    o.z = dequant_pair(magic_pair(words[i], 2), zz, ss);
    o.w = dequant_pair(magic_pair(words[i], 3), zz, ss);
    dst[i] = o;
  }
}

}  // namespace
}  // namespace tfb

extern "C" int tf_w4a16_dequant(const int32_t* qweight_t, const uint16_t* scales,
                                const int32_t* qzeros, int64_t N, int64_t K, int32_t group_size,
                                uint16_t* out, void* stream) {
  using namespace tfb;
  if (N < 0 || K < 0) return TF_ERR_INVALID_ARG;
  if (group_size != 32 && group_size != 64 && group_size != 128) return TF_ERR_INVALID_ARG;
  if (N % 8 != 0 || K % group_size != 0) return TF_ERR_INVALID_ARG;
  if (N == 0 || K == 0) return TF_OK;
  if (!qweight_t || !scales || !qzeros || !out) return TF_ERR_INVALID_ARG;
  if (!aligned16(qweight_t) || !aligned16(out)) return TF_ERR_ALIGNMENT;
  const int64_t total = N * (K / 32);
  const int threads = 256;
  const int64_t blocks = cdiv(total, threads);
  if (blocks > 0x7fffffffLL) return TF_ERR_UNSUPPORTED;
  w4a16_dequant_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                         static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(qweight_t), reinterpret_cast<const __half*>(scales), qzeros,
      N, K, group_size, reinterpret_cast<uint4*>(out));
  return check_launch();
}
