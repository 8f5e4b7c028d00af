// Splitting bf16 activations into e2m1 terms for the block-scaled tensor-core
// MMA (tcgen05.mma.kind::mxf4), whose two operands are both e2m1 with an e8m0
// scale per 32 elements.  A 32-element block x is written as
//   x = sum_{t < kTerms} 2^{e_t} * q_t,   q_t in e2m1,
// greedily: each term takes the block maximum of the remaining residual, picks
// e_t = ceil(log2(max / 6)) so the largest residual maps onto e2m1's largest
// magnitude, rounds to nearest even (hardware cvt) and subtracts.  Bf16 blocks
// need up to 4-5 terms to become exact; with five, the residual stays below
// 2^-15 of the block maximum (Gaussian rows: dot products off by ~1e-6
// relative, far under half a bf16 ulp).
#pragma once
#include "common.cuh"

namespace flyai {

// Two floats -> one e2m1x2 byte (round to nearest even, saturating): lo in the
// low nibble (even K), hi in the high nibble.
__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
      "mov.b16 %0, {t, 0};\n\t}"
      : "=h"(r)
      : "f"(hi), "f"(lo));
  return r & 0xFFu;
}
__device__ __forceinline__ float2 e2m1x2_to_f32x2(uint32_t byte) {
  uint32_t h2;
  asm("{\n\t.reg .b8 t, z;\n\t"
      "mov.b16 {t, z}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(h2)
      : "h"(static_cast<uint16_t>(byte)));
  const __half2 h = *reinterpret_cast<const __half2*>(&h2);
  return __half22float2(h);
}

// Row layouts of the split activations (K = row length, multiple of 32):
//   terms  [K/32 blocks][kTerms][16 bytes]  -- the kTerms e2m1 rows of one
//          32-element block are adjacent (96 bytes), so one row's terms over the
//          whole K are one contiguous run that a bulk copy moves as-is; the MMA
//          reads it as 8-row core matrices (terms 0..7, slots past kTerms see the
//          next block and are ignored) with a 96-byte K stride;
//   scales [K/128 groups of 4 blocks][8 term slots][16 bytes] -- e8m0 of
//          (term, block) in the first 4 bytes of slot t (the 4 blocks of one
//          128-element group: the word the tensor-memory scale layout wants per
//          (row, group)); the other 12 bytes are padding.  A token's 128 bytes
//          of one group are 8 consecutive rows of tcgen05.cp's 32x128b scale
//          chunk, so a chunk's B scales are assembled by 128-byte bulk copies.
constexpr int kTermSlots = 8;
static_assert(kTerms <= kTermSlots, "terms must fit the 8-row core matrix of a token");
__host__ __device__ __forceinline__ size_t term_row_bytes(int K) {
  return static_cast<size_t>(K / 32) * kTerms * 16;
}
constexpr int kTermSfGroupBytes = kTermSlots * 16;   // one token's scales of one 128-K group
__host__ __device__ __forceinline__ size_t term_sf_row_bytes(int K) {
  return static_cast<size_t>((K + 127) / 128) * kTermSfGroupBytes;
}
__host__ __device__ __forceinline__ size_t term_sf_offset(int block, int term) {
  return static_cast<size_t>(block / 4) * kTermSfGroupBytes + term * 16 + block % 4;
}

// One 32-element block held as 8 consecutive values by each of 4 adjacent
// lanes (quarter = lane & 3); all 32 lanes of the warp must call (shuffles).
// With store, writes this lane's 4 packed bytes of term t at tb + t*16 +
// quarter*4 and, from quarter 0, the block's e8m0 scale of term t at sb + t*16
// (tb, sb: the block's place in the row layouts above).
__device__ __forceinline__ void decompose_block(float (&v)[8], int quarter, uint8_t* tb,
                                                uint8_t* sb, bool store) {
#pragma unroll 1
  for (int t = 0; t < kTerms; ++t) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    int e = -127;
    if (amax > 0.f && isfinite(amax)) {
      int E;
      const float f = frexpf(amax * (1.0f / 6.0f), &E);   // amax/6 = f * 2^E, f in [0.5, 1)
      e = (f == 0.5f) ? E - 1 : E;                           // ceil(log2(amax / 6))
      e = max(-126, min(126, e));
    }
    const float inv = (e == -127) ? 0.f : exp2i(-e);
    const float scale = (e == -127) ? 0.f : exp2i(e);
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const uint32_t b = f32x2_to_e2m1x2(v[i] * inv, v[i + 1] * inv);
      const float2 q = e2m1x2_to_f32x2(b);
      v[i] = __fsub_rn(v[i], __fmul_rn(q.x, scale));
      v[i + 1] = __fsub_rn(v[i + 1], __fmul_rn(q.y, scale));
      word |= b << (4 * i);
    }
    if (store) {
      *reinterpret_cast<uint32_t*>(tb + t * 16 + quarter * 4) = word;
      if (quarter == 0) sb[t * 16] = static_cast<uint8_t>(e + 127);
    }
  }
}

// The threads of a block split bf16 rows [row0, row0 + nrows) of src (ld
// elements per row, K columns, K multiple of 32) into the term and scale row
// layouts above (rows of term_row_bytes / term_sf_row_bytes, starting at terms
// and sf for row0).  blockDim.x must be a multiple of 32.
__device__ __forceinline__ void decompose_rows(const uint16_t* src, int ld, int K, int row0,
                                               int nrows, uint8_t* terms, uint8_t* sf) {
  const int blocks = K / 32;
  const size_t trb = term_row_bytes(K), srb = term_sf_row_bytes(K);
  const int units = nrows * blocks * 4;
  for (int u0 = 0; u0 < units; u0 += blockDim.x) {
    const int u = u0 + threadIdx.x;
    const bool live = u < units;
    const int q = u & 3, blk = (u >> 2) % blocks, r = live ? (u >> 2) / blocks : 0;
    float v[8];
    if (live) {
      const uint4 w =
          *reinterpret_cast<const uint4*>(src + static_cast<size_t>(row0 + r) * ld + blk * 32 + q * 8);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(ws[i] << 16);
        v[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    decompose_block(v, q, terms + r * trb + static_cast<size_t>(blk) * kTerms * 16,
                    sf + r * srb + term_sf_offset(blk, 0), live);
  }
  // scale slots no MMA column uses (terms past kTerms, blocks past K): neutral
  const int groups = (K + 127) / 128;
  for (int i = threadIdx.x; i < nrows * groups * kTermSlots * 4; i += blockDim.x) {
    const int r = i / (groups * kTermSlots * 4), rem = i % (groups * kTermSlots * 4);
    const int g = rem / (kTermSlots * 4), t = (rem / 4) % kTermSlots, b = g * 4 + rem % 4;
    if (t >= kTerms || b >= blocks) sf[r * srb + g * kTermSfGroupBytes + t * 16 + b % 4] = 127;
  }
}

}  // namespace flyai
