// Register-level W4A16 dequant + tensor-core math shared by the decode GEMVs (w4a16_gemv.cu) and
// the persistent decode chain (w4a16_chain.cu): one lane's four weight rows of a 128-wide K block
// (GSlot), the exact (q - z) unpack with LOP3 + magic numbers and sub.rn.f16x2, the m16n8k16 MMAs
// over the staged activations, and the per-block scale fold. Every kernel that uses these
// functions computes the same fp32 block sums for the same inputs.
#pragma once

#include "tf_common.cuh"

namespace tfb {
namespace {

constexpr int kKB = 128;         // K values per block (one quantization group at group size 128)

// One K block of this lane's four rows, in registers from issue to use.
struct GSlot {
  uint4 w[4];   // rows 4q..4q+3: 16 bytes (32 values of k) each
  uint2 s;      // the four rows' scales: (row0 | row1 << 16), (row2 | row3 << 16)
  uint32_t z;   // qzeros word holding the four rows' zero points
};

struct GLane {
  const int32_t* w[4];  // rows r0..r0+3 (the lane's four) + this lane's word offset 4c
  const uint2* s;       // scales row 0, column r0 (4 halves)
  const int32_t* z;     // qzeros row 0, word r0 / 8
  const uint4* xs;      // staged activations: token row q (clamped), + 32c
  int nib[4];           // bit offsets of the four rows' zero points in the qzeros word
  int kb0, b_end;       // this CTA's first block, this warp's end block (exclusive)
  int c;
};

__device__ __forceinline__ uint4 zero4() { return make_uint4(0, 0, 0, 0); }

// PTX forms: one LOP3 per pair, and the fp16 subtract / multiply with explicit .rn so they are
// never contracted into an FMA (which would round once less than the reference).
__device__ __forceinline__ uint32_t lop_mask_or(uint32_t w, uint32_t mask, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(mask), "r"(magic));
  return r;
}
__device__ __forceinline__ uint32_t hsub2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

struct RowConsts {  // per row: fp16x2 (1024 + z) and (s, s)
  uint32_t zz, ss;
};

// Pair j (offsets 2j, 2j+1) of a packed word, dequantized: fp16(q - z) * s, one rounding.
__device__ __forceinline__ uint32_t deq(uint32_t w, int j, const RowConsts& r, uint32_t mask,
                                       uint32_t magic) {
  return hmul2_rn(hsub2_rn(lop_mask_or(w >> (4 * j), mask, magic), r.zz), r.ss);
}

__device__ __forceinline__ void gcompute(float (&acc)[2][2][4], const GSlot& s, int bb,
                                         const GLane& L, uint32_t mask, uint32_t magic) {
  RowConsts rc[4];
  const uint32_t sp[2] = {s.s.x, s.s.y};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t z = (s.z >> L.nib[j]) & 0xFu;
    rc[j].zz = (z * 0x00010001u) | magic;
    rc[j].ss = __byte_perm(sp[j >> 1], sp[j >> 1], (j & 1) ? 0x3232u : 0x1010u);
  }
  const uint4* xp = L.xs + (bb - L.kb0) * (kKB / 8);
  const uint32_t w0[4] = {s.w[0].x, s.w[0].y, s.w[0].z, s.w[0].w};
  const uint32_t w1[4] = {s.w[1].x, s.w[1].y, s.w[1].z, s.w[1].w};
  const uint32_t w2[4] = {s.w[2].x, s.w[2].y, s.w[2].z, s.w[2].w};
  const uint32_t w3[4] = {s.w[3].x, s.w[3].y, s.w[3].z, s.w[3].w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // packed word i: k = 8i .. 8i+7 of the lane's chunk
    const uint4 xv = xp[i];
    // Tile 0: fragment rows q / q+8 <- rows 4q / 4q+1; tile 1 <- rows 4q+2 / 4q+3.
    const uint32_t t0a[4] = {deq(w0[i], 0, rc[0], mask, magic), deq(w1[i], 0, rc[1], mask, magic),
                             deq(w0[i], 1, rc[0], mask, magic), deq(w1[i], 1, rc[1], mask, magic)};
    const uint32_t t0b[4] = {deq(w0[i], 2, rc[0], mask, magic), deq(w1[i], 2, rc[1], mask, magic),
                             deq(w0[i], 3, rc[0], mask, magic), deq(w1[i], 3, rc[1], mask, magic)};
    const uint32_t t1a[4] = {deq(w2[i], 0, rc[2], mask, magic), deq(w3[i], 0, rc[3], mask, magic),
                             deq(w2[i], 1, rc[2], mask, magic), deq(w3[i], 1, rc[3], mask, magic)};
    const uint32_t t1b[4] = {deq(w2[i], 2, rc[2], mask, magic), deq(w3[i], 2, rc[3], mask, magic),
                             deq(w2[i], 3, rc[2], mask, magic), deq(w3[i], 3, rc[3], mask, magic)};
    mma_16816(acc[0][i & 1], t0a, xv.x, xv.y);
    mma_16816(acc[0][i & 1], t0b, xv.z, xv.w);
    mma_16816(acc[1][i & 1], t1a, xv.x, xv.y);
    mma_16816(acc[1][i & 1], t1b, xv.z, xv.w);
  }
}

// mma.m16n8k16 with a zero accumulator input: d = a * b.
__device__ __forceinline__ void mma_16816_zc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// The four rows' zero points of a group-size-128 block as fp16x2 broadcasts: z0[j] = (1024 + z_j)
// twice and z1[j] = (64 + z_j) twice. The rows' zero points sit in nibbles {0, 4, 1, 5} of the
// qzeros word shifted by nib[0] (0 or 8): one LOP3 per row pair places them in the mantissa of
// 0x6400 (1024 + z, unit steps in bits 0-3) or, four bits higher, of 0x5400 (64 + z, unit steps
// in bits 4-7), and a byte permute broadcasts each row's value to both halves. Integer and
// permute instructions only, so the fp16 pipe is left to the per-weight dequant.
__device__ __forceinline__ void zero_points(uint32_t (&z0)[4], uint32_t (&z1)[4], uint32_t zword,
                                            int nib0) {
  const uint32_t zs = zword >> nib0;
  const uint32_t a = lop_mask_or(zs, 0x000F000Fu, 0x64006400u);        // rows 0, 1: 1024 + z
  const uint32_t b = lop_mask_or(zs >> 4, 0x000F000Fu, 0x64006400u);   // rows 2, 3: 1024 + z
  const uint32_t a1 = lop_mask_or(zs << 4, 0x00F000F0u, 0x54005400u);  // rows 0, 1: 64 + z
  const uint32_t b1 = lop_mask_or(zs, 0x00F000F0u, 0x54005400u);       // rows 2, 3: 64 + z
  z0[0] = __byte_perm(a, a, 0x1010u);
  z0[1] = __byte_perm(a, a, 0x3232u);
  z0[2] = __byte_perm(b, b, 0x1010u);
  z0[3] = __byte_perm(b, b, 0x3232u);
  z1[0] = __byte_perm(a1, a1, 0x1010u);
  z1[1] = __byte_perm(a1, a1, 0x3232u);
  z1[2] = __byte_perm(b1, b1, 0x1010u);
  z1[3] = __byte_perm(b1, b1, 0x3232u);
}

// The lane's 4 x 16 dequantized fp16x2 pairs of one word column i of a group-size-128 block, in
// the MMA fragment order: each pair is unpacked to the exact fp16 integers (q - z) (bits 0-3 of
// a half ORed into 0x6400 read as 1024 + q, bits 4-7 ORed into 0x5400 as 64 + q; one LOP3, one
// shift per word for the upper byte, one HSUB2 of (1024 + z) or (64 + z)) and multiplied by the
// row's scale with one HMUL2: w = fp16((q - z) * s), one rounding, the reference's dequantized
// weight (tokenforge/kernels/pack.py:189-194), so the tensor core's fp32 sums are those of the
// reference's fp16 weights and Inf / NaN follow the reference's dequant.
struct W16Frag {
  uint32_t t0a[4], t0b[4], t1a[4], t1b[4];  // tile 0 / 1, k offsets (0..3) / (4..7) of the word
};

__device__ __forceinline__ void dequant_word(W16Frag& f, const uint32_t (&w)[4],
                                             const uint32_t (&z0)[4], const uint32_t (&z1)[4],
                                             const uint32_t (&sc)[4]) {
  const uint32_t m0 = 0x000F000Fu, m1 = 0x00F000F0u;
  const uint32_t g0 = 0x64006400u, g1 = 0x54005400u;
  uint32_t pa[4], pb[4], pc[4], pd[4];  // offsets (0,1), (2,3), (4,5), (6,7) of row j's word
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t h = w[j] >> 8;
    pa[j] = hmul2_rn(hsub2_rn(lop_mask_or(w[j], m0, g0), z0[j]), sc[j]);
    pb[j] = hmul2_rn(hsub2_rn(lop_mask_or(w[j], m1, g1), z1[j]), sc[j]);
    pc[j] = hmul2_rn(hsub2_rn(lop_mask_or(h, m0, g0), z0[j]), sc[j]);
    pd[j] = hmul2_rn(hsub2_rn(lop_mask_or(h, m1, g1), z1[j]), sc[j]);
  }
  // Tile 0: fragment rows q / q+8 <- rows 4q / 4q+1; tile 1 <- rows 4q+2 / 4q+3.
  f.t0a[0] = pa[0]; f.t0a[1] = pa[1]; f.t0a[2] = pb[0]; f.t0a[3] = pb[1];
  f.t0b[0] = pc[0]; f.t0b[1] = pc[1]; f.t0b[2] = pd[0]; f.t0b[3] = pd[1];
  f.t1a[0] = pa[2]; f.t1a[1] = pa[3]; f.t1a[2] = pb[2]; f.t1a[3] = pb[3];
  f.t1b[0] = pc[2]; f.t1b[1] = pc[3]; f.t1b[2] = pd[2]; f.t1b[3] = pd[3];
}

// (s, s) broadcasts of the lane's four rows' scales.
__device__ __forceinline__ void scale_pairs(uint32_t (&sc)[4], const GSlot& s) {
  sc[0] = __byte_perm(s.s.x, s.s.x, 0x1010u);
  sc[1] = __byte_perm(s.s.x, s.s.x, 0x3232u);
  sc[2] = __byte_perm(s.s.y, s.s.y, 0x1010u);
  sc[3] = __byte_perm(s.s.y, s.s.y, 0x3232u);
}

// acc += x * w over one group-size-128 block bb, w dequantized per weight as the reference
// does (dequant_word); acc[t][i % 2] are two independent accumulator chains per row tile.
__device__ __forceinline__ void gcompute_w16(float (&acc)[2][2][4], const GSlot& s, int bb,
                                             const GLane& L) {
  uint32_t z0[4], z1[4], sc[4];
  zero_points(z0, z1, s.z, L.nib[0]);
  scale_pairs(sc, s);
  const uint4* xp = L.xs + (bb - L.kb0) * (kKB / 8);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 xv = xp[i];
    const uint32_t w[4] = {(&s.w[0].x)[i], (&s.w[1].x)[i], (&s.w[2].x)[i], (&s.w[3].x)[i]};
    W16Frag f;
    dequant_word(f, w, z0, z1, sc);
    mma_16816(acc[0][i & 1], f.t0a, xv.x, xv.y);
    mma_16816(acc[1][i & 1], f.t1a, xv.x, xv.y);
    mma_16816(acc[0][i & 1], f.t0b, xv.z, xv.w);
    mma_16816(acc[1][i & 1], f.t1b, xv.z, xv.w);
  }
}

}  // namespace
}  // namespace tfb
