// DeepSeek-V4-style W4A8 MoE layer (FLYAI_FMT_FP4_W4A8): bank and block layouts
// shared by the launcher and the kernels of v4_moe.cu.
//
// Routed experts hold e2m1 weights with one e8m0 scale per 32 along K (the V4
// checkpoint's float4_e2m1fn_x2 + float8_e8m0fnu pair, model.py:133-139); the
// shared expert holds e4m3 weights with one e8m0 scale per 128x128 block
// (dtype "fp8", scale_dtype "fp8").  Activations are e4m3 with one power-of-two
// scale per 1x128 block (act_quant with scale_fmt "ue8m0").
#pragma once
#include "act_quant.cuh"
#include "common.cuh"
#include "fp8_moe.cuh"

namespace flyai {

constexpr int kV4Chunk = 16;                             // tokens of one expert per chunk = MMA N
constexpr int kV4Fp4Tile = 128 * 64;                     // 8 KB: 128 rows x 128 K of packed e2m1
constexpr int kV4Sf = 512;                               // one tcgen05.cp chunk: 128 rows x 4 e8m0
constexpr int kV4RawTile = kV4Fp4Tile + kV4Sf;           // 8704: routed-expert tile in the bank
constexpr int kV4F8Tile = 128 * 128;                     // 16 KB: 128 rows x 128 K of e4m3
constexpr int kV4XTile = kV4F8Tile + kV4Sf;              // 16896: e4m3 tile + its scale chunk
constexpr int kV4BTile = kV4Chunk * 128;                 // 2 KB: 16 token rows x 128 K of e4m3
constexpr int kV4BBytes = kV4BTile + kV4Sf;              // + the tokens' scale chunk
constexpr int kV4BOff = 2 * kV4XTile;                    // 33792: B block inside a stage
constexpr int kV4Stage = kV4BOff + kV4BBytes;            // 36352: one 128-wide K block of an item

// Bank of one projection.  Routed expert e (local index < El): per 128-row
// output block, per 128-wide K block one "raw block" of `tiles` raw tiles (W13:
// the w1 tile then the w3 tile of the same rows; W2: one w2 tile).  A raw tile
// is 8 KB of e2m1 -- 16 K (8 bytes) of row r, K-chunk c at c*1024 + (r/8)*64 +
// (r%8)*8, i.e. half the offset its e4m3 expansion takes in the canonical
// K-major tcgen05 operand (16 bytes at c*2048 + (r/8)*128 + (r%8)*16) -- then
// the tile's 512-byte scale chunk (row m, 32-block j at (m%32)*16 + (m/32)*4 + j:
// the bytes tcgen05.cp 32x128b.warpx4 moves into tensor memory).  The shared
// expert(s) follow at shared_off in the same order with e4m3 tiles in the
// canonical layout, each followed by a scale chunk holding its block's e8m0.
struct V4Bank {
  int tiles;          // tiles per block: 2 (W13) or 1 (W2)
  int RB, KB;         // 128-row output blocks, 128-wide K blocks
  size_t fp4_block;   // bytes per routed raw block
  size_t fp4_expert;  // bytes per routed expert
  size_t f8_block;    // bytes per shared-expert block
  size_t f8_expert;   // bytes per shared expert
  size_t shared_off;  // first byte of the shared expert(s)
};
__host__ __device__ inline V4Bank v4_bank(const flyai_moe_desc& d, int proj) {
  V4Bank b;
  b.tiles = proj == FLYAI_PROJ_W13 ? 2 : 1;
  b.RB = (proj == FLYAI_PROJ_W13 ? d.inter : d.hidden) / 128;
  b.KB = (proj == FLYAI_PROJ_W13 ? d.hidden : d.inter) / 128;
  b.fp4_block = static_cast<size_t>(b.tiles) * kV4RawTile;
  b.fp4_expert = b.fp4_block * b.RB * b.KB;
  b.f8_block = static_cast<size_t>(b.tiles) * kV4XTile;
  b.f8_expert = b.f8_block * b.RB * b.KB;
  b.shared_off = b.fp4_expert * static_cast<size_t>(d.expert_end - d.expert_begin);
  return b;
}

__host__ __device__ inline bool is_v4(const flyai_moe_desc& d) { return d.format == FLYAI_FMT_FP4_W4A8; }

// e2m1 nibbles -> e4m3 bytes, exact (every e2m1 value is an e4m3 value): the 8
// packed elements of w (low nibble first) become the 8 bytes of (lo, hi).  The
// magnitude codes index a byte table with prmt; the sign bits pick 0x00 / 0x80.
__device__ __forceinline__ void e2m1x8_to_e4m3(uint32_t w, uint32_t& lo, uint32_t& hi) {
  constexpr uint32_t kMagLo = 0x3C383000u;   // codes 0..3: 0, 0.5, 1, 1.5
  constexpr uint32_t kMagHi = 0x4C484440u;   // codes 4..7: 2, 3, 4, 6
  const uint32_t m = w & 0x77777777u, s = (w >> 3) & 0x11111111u;
  lo = __byte_perm(kMagLo, kMagHi, m & 0xFFFFu) | __byte_perm(0x8000u, 0u, s & 0xFFFFu);
  hi = __byte_perm(kMagLo, kMagHi, m >> 16) | __byte_perm(0x8000u, 0u, s >> 16);
}

}  // namespace flyai
