// AWQ repack: qweight [K, N/8] (packed along N) -> qweight_t [N, K/8] (packed along K).
//
// Semantics follow repack_awq_to_tf (reference tokenforge/kernels/pack.py:141-143): the
// logical int4 matrix is transposed and re-packed with the same nibble interleave
// (nibble i of a word holds offset AWQ_ORDER[i] = (0,2,4,6,1,3,5,7)[i], pack.py:32).
//
// One thread owns an 8x8 block of int4 values per step: eight input words (rows k0..k0+7 of
// one column word) become eight output words (columns 8c..8c+7, one row word k0/8). Because
// both layouts use the same interleave, the block is a plain 8x8 nibble transpose once the
// input words are taken in AWQ_ORDER and the output words are written in AWQ_ORDER:
//   out[8c + ORDER[i]][k0/8] = transpose(in[k0 + ORDER[0..7]][c])[i].
// A thread handles eight consecutive row words (64 values of K), so each output row receives
// a full 32-byte sector written with two 16-byte stores, while the 32 threads of a warp read
// 32 consecutive input words (128 contiguous bytes) per load. HBM-bound: 2 * N * K / 2 bytes.
#include "tf_common.cuh"

namespace tfb {
namespace {

__constant__ int kAwqOrder[8] = {0, 2, 4, 6, 1, 3, 5, 7};

// In-register transpose of an 8x8 matrix of nibbles: element (r, j) is nibble j of w[r].
__device__ __forceinline__ void transpose8x8_nibbles(uint32_t (&w)[8]) {
#pragma unroll
  for (int r = 0; r < 4; ++r) {  // swap 4x4 blocks: 16-bit halves of words r and r+4
    const uint32_t a = w[r], b = w[r + 4];
    w[r] = (a & 0x0000FFFFu) | (b << 16);
    w[r + 4] = (a >> 16) | (b & 0xFFFF0000u);
  }
#pragma unroll
  for (int base = 0; base < 8; base += 4) {  // swap 2x2 blocks: bytes of words r and r+2
#pragma unroll
    for (int r = base; r < base + 2; ++r) {
      const uint32_t a = w[r], b = w[r + 2];
      w[r] = (a & 0x00FF00FFu) | ((b << 8) & 0xFF00FF00u);
      w[r + 2] = ((a >> 8) & 0x00FF00FFu) | (b & 0xFF00FF00u);
    }
  }
#pragma unroll
  for (int r = 0; r < 8; r += 2) {  // swap single nibbles of words r and r+1
    const uint32_t a = w[r], b = w[r + 1];
    w[r] = (a & 0x0F0F0F0Fu) | ((b << 4) & 0xF0F0F0F0u);
    w[r + 1] = ((a >> 4) & 0x0F0F0F0Fu) | (b & 0xF0F0F0F0u);
  }
}

// rows = K (input rows), cols8 = N/8 (input words per row); output is [cols8*8, rows/8].
template <bool kVecStore>
__global__ void __launch_bounds__(128) awq_repack_kernel(const uint32_t* __restrict__ in,
                                                         int64_t rows, int64_t cols8,
                                                         uint32_t* __restrict__ out) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols8) return;
  const int64_t out_words = rows / 8;                 // words per output row
  const int64_t kw0 = static_cast<int64_t>(blockIdx.y) * 8;  // first output word column
  const int64_t left = out_words - kw0;
  const int nblk = left < 8 ? static_cast<int>(left) : 8;

  // Two halves of four row words each: one 16-byte store per output row per half.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t res[8][4];  // res[s][b]: output row 8c + s, word kw0 + 4h + b
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int bb = 4 * h + b;
      if (bb < nblk) {
        uint32_t w[8];
        const int64_t k0 = (kw0 + bb) * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = __ldg(in + (k0 + kAwqOrder[j]) * cols8 + c);
        transpose8x8_nibbles(w);
#pragma unroll
        for (int i = 0; i < 8; ++i) res[kAwqOrder[i]][b] = w[i];
      } else {
#pragma unroll
        for (int s = 0; s < 8; ++s) res[s][b] = 0;
      }
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      uint32_t* dst = out + (8 * c + s) * out_words + kw0 + 4 * h;
      if (kVecStore && nblk >= 4 * h + 4) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(res[s][0], res[s][1], res[s][2], res[s][3]);
      } else {
#pragma unroll
        for (int b = 0; b < 4; ++b)
          if (4 * h + b < nblk) dst[b] = res[s][b];
      }
    }
  }
}

// Tiled variant: a CTA of 128 threads turns 256 input rows x 32 input words into 256 output
// rows x 32 output words (128 contiguous bytes each), staged through shared memory so that both
// the loads (a warp reads 128 bytes of one input row) and the stores (eight threads write one
// 128-byte output row segment) are full lines. Thread (cx, ky) transposes the 8 x 8 nibble
// blocks of column word cx and row words 8ky .. 8ky+7 in registers as above.
constexpr int kTileW = 32;             // input words per tile row = output words per tile row
constexpr int kTileRows = 8 * kTileW;  // input rows per tile = output rows per tile
__global__ void __launch_bounds__(128) awq_repack_tiled_kernel(const uint32_t* __restrict__ in,
                                                               int64_t rows, int64_t cols8,
                                                               uint32_t* __restrict__ out) {
  __shared__ uint32_t tile[kTileRows][kTileW + 1];
  const int cx = threadIdx.x & 31, ky = threadIdx.x >> 5;  // column word, row-word group
  const int64_t c = static_cast<int64_t>(blockIdx.x) * kTileW + cx;
  const int64_t out_words = rows / 8;
  const int64_t kw_base = static_cast<int64_t>(blockIdx.y) * kTileW;
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const int wl = 8 * ky + b;  // output word within the tile
    const int64_t kw = kw_base + wl;
    uint32_t w[8];
    if (c < cols8 && kw < out_words) {
      const int64_t k0 = kw * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = __ldg(in + (k0 + kAwqOrder[j]) * cols8 + c);
      transpose8x8_nibbles(w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = 0;
    }
    // Output row 8cx + s is kept at tile row 32s + cx: with a 33-word pitch the 32 threads of a
    // warp (cx = 0..31) then write 32 different banks.
#pragma unroll
    for (int i = 0; i < 8; ++i) tile[32 * kAwqOrder[i] + cx][wl] = w[i];
  }
  __syncthreads();
  // 256 output rows x 32 words: thread t writes 4 words of row (pass * 16 + t / 8).
  const int sub = threadIdx.x & 7, rsub = threadIdx.x >> 3;
  for (int r = rsub; r < kTileRows; r += 16) {
    const int64_t orow = static_cast<int64_t>(blockIdx.x) * kTileRows + r;  // = 8 * c + s
    if (orow >= cols8 * 8) break;
    const int64_t kw = kw_base + 4 * sub;
    uint32_t* dst = out + orow * out_words + kw;
    const uint32_t* srow = &tile[32 * (r & 7) + (r >> 3)][4 * sub];
    if (kw + 4 <= out_words && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(srow[0], srow[1], srow[2], srow[3]);
    } else {
      for (int e = 0; e < 4 && kw + e < out_words; ++e) dst[e] = srow[e];
    }
  }
}

// AWQ_ORDER as a compile-time function, so that fully unrolled loops index registers.
__device__ __forceinline__ constexpr int awq_order(int j) { return j < 4 ? 2 * j : 2 * j - 7; }

// The same tile, loaded 16 bytes at a time (input row stride a multiple of four words, 16-byte
// aligned): thread (cq, g) takes column words 4cq .. 4cq+3 of row groups g and g + 16 (eight
// input rows each), all sixteen 16-byte loads in flight before the first transpose, so a CTA
// keeps its whole 32 KB input tile in flight (the one-word variant above has 32 B per thread
// outstanding). A warp's load covers four rows x 128 contiguous bytes; the shared-memory writes
// (bank (4cq + cc + g) mod 32) do not conflict; the output phase is the one above.
__global__ void __launch_bounds__(128) awq_repack_tiled_v4_kernel(const uint32_t* __restrict__ in,
                                                                  int64_t rows, int64_t cols8,
                                                                  uint32_t* __restrict__ out) {
  __shared__ uint32_t tile[kTileRows][kTileW + 1];
  const int cq = threadIdx.x & 7, g = threadIdx.x >> 3;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kTileW + 4 * cq;
  const int64_t out_words = rows / 8;
  const int64_t kw_base = static_cast<int64_t>(blockIdx.y) * kTileW;
  const int64_t row_vecs = cols8 / 4;
  uint4 ld[2][8];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t kw = kw_base + g + 16 * h;
    const bool ok = c0 < cols8 && kw < out_words;  // cols8 % 4 == 0: the quad is all in or out
    const uint4* src = reinterpret_cast<const uint4*>(in + kw * 8 * cols8 + c0);
#pragma unroll
    for (int r = 0; r < 8; ++r) ld[h][r] = ok ? ldg_stream_v4(src + r * row_vecs) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = reinterpret_cast<const uint32_t*>(&ld[h][awq_order(j)])[cc];
      transpose8x8_nibbles(w);
#pragma unroll
      for (int i = 0; i < 8; ++i) tile[32 * awq_order(i) + 4 * cq + cc][g + 16 * h] = w[i];
    }
  }
  __syncthreads();
  // Output rows r = 8 * (rsub + 16 * (pass & 1)) + pass / 2: the four rows a warp stores at once
  // (rsub = 4w .. 4w+3) sit in tile rows 32 (r % 8) + r / 8 that differ modulo 32, so their
  // shared-memory reads fall in different banks (rows 32 apart share banks at a 33-word pitch).
  const int sub = threadIdx.x & 7, rsub = threadIdx.x >> 3;
#pragma unroll 4
  for (int pass = 0; pass < 16; ++pass) {
    const int r = 8 * (rsub + 16 * (pass & 1)) + (pass >> 1);
    const int64_t orow = static_cast<int64_t>(blockIdx.x) * kTileRows + r;
    if (orow >= cols8 * 8) continue;
    const int64_t kw = kw_base + 4 * sub;
    uint32_t* dst = out + orow * out_words + kw;
    const uint32_t* srow = &tile[32 * (r & 7) + (r >> 3)][4 * sub];
    if (kw + 4 <= out_words && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(srow[0], srow[1], srow[2], srow[3]);
    } else {
      for (int e = 0; e < 4 && kw + e < out_words; ++e) dst[e] = srow[e];
    }
  }
}

int launch_repack(const int32_t* in, int64_t rows, int64_t cols, int32_t* out,
                  cudaStream_t stream) {
  // rows: the packed-across dimension of the output (K for repack); cols: logical columns.
  if (rows < 0 || cols < 0 || rows % 8 != 0 || cols % 8 != 0) return TF_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return TF_OK;
  if (in == nullptr || out == nullptr) return TF_ERR_INVALID_ARG;
  const int64_t cols8 = cols / 8;
  const int64_t out_words = rows / 8;
  if (out_words >= kTileW && cols8 >= kTileW) {
    const dim3 tgrid(static_cast<unsigned>(cdiv(cols8, kTileW)),
                     static_cast<unsigned>(cdiv(out_words, kTileW)));
    if (tgrid.y <= 65535u && cols8 % 4 == 0 && aligned16(in)) {
      awq_repack_tiled_v4_kernel<<<tgrid, 128, 0, stream>>>(
          reinterpret_cast<const uint32_t*>(in), rows, cols8, reinterpret_cast<uint32_t*>(out));
      return check_launch();
    }
    if (tgrid.y <= 65535u) {
      awq_repack_tiled_kernel<<<tgrid, 128, 0, stream>>>(
          reinterpret_cast<const uint32_t*>(in), rows, cols8, reinterpret_cast<uint32_t*>(out));
      return check_launch();
    }
  }
  const dim3 block(128);
  const dim3 grid(static_cast<unsigned>(cdiv(cols8, 128)), static_cast<unsigned>(cdiv(out_words, 8)));
  if (grid.y > 65535u) return TF_ERR_UNSUPPORTED;
  const bool vec = (out_words % 4 == 0) && aligned16(out);
  if (vec)
    awq_repack_kernel<true><<<grid, block, 0, stream>>>(
        reinterpret_cast<const uint32_t*>(in), rows, cols8, reinterpret_cast<uint32_t*>(out));
  else
    awq_repack_kernel<false><<<grid, block, 0, stream>>>(
        reinterpret_cast<const uint32_t*>(in), rows, cols8, reinterpret_cast<uint32_t*>(out));
  return check_launch();
}

__global__ void unpack_int4_kernel(const uint32_t* __restrict__ packed, int64_t n_words,
                                   uint4* __restrict__ values) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w >= n_words) return;
  const uint32_t v = __ldg(packed + w);
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = (v >> (4 * awq_nibble_of(j))) & 0xFu;
  values[2 * w] = make_uint4(o[0], o[1], o[2], o[3]);
  values[2 * w + 1] = make_uint4(o[4], o[5], o[6], o[7]);
}

__global__ void pack_int4_kernel(const uint4* __restrict__ values, int64_t n_words,
                                 uint32_t* __restrict__ packed) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w >= n_words) return;
  const uint4 a = values[2 * w], b = values[2 * w + 1];
  const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) word |= (v[j] & 0xFu) << (4 * awq_nibble_of(j));
  packed[w] = word;
}

}  // namespace
}  // namespace tfb

extern "C" int tf_unpack_int4(const int32_t* packed, int64_t n_words, int32_t* values,
                              void* stream) {
  using namespace tfb;
  if (n_words < 0) return TF_ERR_INVALID_ARG;
  if (n_words == 0) return TF_OK;
  if (!packed || !values) return TF_ERR_INVALID_ARG;
  if (!aligned16(values)) return TF_ERR_ALIGNMENT;
  unpack_int4_kernel<<<static_cast<unsigned>(cdiv(n_words, 256)), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(packed), n_words, reinterpret_cast<uint4*>(values));
  return check_launch();
}

extern "C" int tf_pack_int4(const int32_t* values, int64_t n_words, int32_t* packed,
                            void* stream) {
  using namespace tfb;
  if (n_words < 0) return TF_ERR_INVALID_ARG;
  if (n_words == 0) return TF_OK;
  if (!packed || !values) return TF_ERR_INVALID_ARG;
  if (!aligned16(values)) return TF_ERR_ALIGNMENT;
  pack_int4_kernel<<<static_cast<unsigned>(cdiv(n_words, 256)), 256, 0,
                     static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(values), n_words, reinterpret_cast<uint32_t*>(packed));
  return check_launch();
}

extern "C" int tf_awq_repack(const int32_t* qweight, int64_t K, int64_t N, int32_t* qweight_t,
                             void* stream) {
  return tfb::launch_repack(qweight, K, N, qweight_t, static_cast<cudaStream_t>(stream));
}

// repack_tf_to_awq (pack.py:146-148) is the same transform with the roles of K and N swapped.
extern "C" int tf_awq_unrepack(const int32_t* qweight_t, int64_t N, int64_t K, int32_t* qweight,
                               void* stream) {
  return tfb::launch_repack(qweight_t, N, K, qweight, static_cast<cudaStream_t>(stream));
}
