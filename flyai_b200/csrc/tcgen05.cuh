// tcgen05 (5th-generation tensor core) building blocks for sm_100a: TMEM
// allocation, shared-memory matrix descriptors, block-scaled MMA issue, scale
// factor copies into TMEM, TMEM loads and commit-to-mbarrier.  Encodings
// follow the sm100 UMMA descriptor bit fields (the same fields CUTLASS's
// cute/arch/mma_sm100_desc.hpp names).
#pragma once
#include "common.cuh"

namespace flyai {
namespace tc {

// ---- TMEM allocation (one full warp executes each) --------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// ---- shared-memory matrix descriptor ----------------------------------------
// K-major, no swizzle: in 16-byte units the operand is
// ((8 rows, n groups), 2 K-chunks) : ((1, SBO), LBO) -- a core matrix is 8 rows
// x 16 bytes stored contiguously (128 B), row groups are SBO bytes apart and the
// two 16-byte K chunks one MMA consumes are LBO bytes apart.
__device__ __forceinline__ uint64_t smem_desc_kmajor(const void* smem_ptr, uint32_t lbo_bytes,
                                                     uint32_t sbo_bytes) {
  const uint32_t addr = smem_u32(smem_ptr);
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);             // start address   [0,14)
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;  // leading offset  [16,30)
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;  // stride offset   [32,46)
  d |= 1ull << 46;                                               // descriptor version 1
  return d;                                                      // no swizzle, base offset 0
}

// K-major with the 128-byte swizzle: row r of the operand is one 128-byte line
// (64 16-bit elements of K) at r * 128, its 16-byte chunk q stored at chunk
// position q ^ (r % 8), 8-row groups 1024 bytes apart (SBO); the leading offset
// field is 1 (adjacent chunks).  The operand must start on a 1024-byte boundary;
// the K = 16 step j of an MMA starts 32 * j bytes into the line (the hardware
// applies the XOR on the address bits, so the start address moves by plain
// offsets).  The same layout in global memory, copied with a bulk copy to a
// 1024-aligned destination, keeps its swizzle.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* smem_ptr) {
  const uint32_t addr = smem_u32(smem_ptr);
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);   // start address   [0,14)
  d |= 1ull << 16;                                     // leading offset  [16,30) = 16 B
  d |= static_cast<uint64_t>(1024 >> 4) << 32;         // stride offset   [32,46)
  d |= 1ull << 46;                                     // descriptor version 1
  d |= 2ull << 61;                                     // layout: 128-byte swizzle
  return d;
}
__host__ __device__ __forceinline__ int sw128_offset(int r, int q) {
  return r * 128 + ((q ^ (r & 7)) << 4);
}

// ---- instruction descriptor: block-scaled e2m1 x e2m1 (kind::mxf4) ------------
// M = 128, N multiple of 8 in [16, 256], both operands K-major, ue8m0 scales per
// 32 elements, dense K = 64 per instruction.  The scale-factor ids select the
// byte pair inside each 32-bit TMEM scale word (0: blocks 0-1, 2: blocks 2-3)
// and must agree with bits 31:30 of the scale TMEM addresses passed to the MMA.
__host__ __device__ __forceinline__ uint32_t idesc_mxf4(int N, int a_sf_id, int b_sf_id) {
  uint32_t d = 0;
  d |= static_cast<uint32_t>(b_sf_id & 3) << 4;   // B scale factor id
  d |= 1u << 7;                                   // A format: e2m1
  d |= 1u << 10;                                  // B format: e2m1
  d |= static_cast<uint32_t>((N >> 3) & 0x3F) << 17;
  d |= 1u << 23;                                  // scale format: ue8m0
  d |= static_cast<uint32_t>(128 >> 4) << 24;     // M = 128
  d |= static_cast<uint32_t>(a_sf_id & 3) << 29;  // A scale factor id
  return d;
}

// ---- instruction descriptor: NVFP4 (kind::mxf4nvf4, block16) --------------------
// Same fields as idesc_mxf4 with ue4m3 scales (scale format 0) and one 32-bit
// TMEM scale word (4 blocks of 16) per row and K=64 step, so both scale ids are 0.
__host__ __device__ __forceinline__ uint32_t idesc_nvf4(int N) {
  uint32_t d = 0;
  d |= 1u << 7;                                   // A format: e2m1
  d |= 1u << 10;                                  // B format: e2m1
  d |= static_cast<uint32_t>((N >> 3) & 0x3F) << 17;
  d |= static_cast<uint32_t>(128 >> 4) << 24;     // M = 128
  return d;
}

// D(tmem) (+)= A(smem) x B(smem)^T, e2m1 operands with ue4m3 scales per 16 elements.
__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(sfa_tmem),
      "r"(sfb_tmem)
      : "memory");
}

// D(tmem) (+)= A(smem) x B(smem)^T with per-32 block scales read from TMEM.
__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(sfa_tmem),
      "r"(sfb_tmem)
      : "memory");
}

// ---- instruction descriptor: e4m3 x e4m3 -> fp32 (kind::f8f6f4) --------------
// M = 128, N multiple of 16 in [16, 256], both operands K-major, dense K = 32
// per instruction, no block scaling (the caller rescales per K block).
__host__ __device__ __forceinline__ uint32_t idesc_f8_e4m3(int N) {
  uint32_t d = 0;
  d |= 1u << 4;                                   // D format: f32
  // A and B format e4m3 = 0 (bits 7-9, 10-12), both K-major (bits 15, 16 = 0)
  d |= static_cast<uint32_t>((N >> 3) & 0x3F) << 17;
  d |= static_cast<uint32_t>(128 >> 4) << 24;     // M = 128
  return d;
}

// D(tmem) (+)= A(smem) x B(smem)^T, e4m3 operands, fp32 accumulate.
__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// ---- instruction descriptor: bf16 x bf16 -> fp32 (kind::f16) --------------------
// M = 128, N multiple of 16 in [16, 256], both operands K-major, K = 16 per instruction.
__host__ __device__ __forceinline__ uint32_t idesc_bf16(int N) {
  uint32_t d = 0;
  d |= 1u << 4;                                   // D format: f32
  d |= 1u << 7;                                   // A format: bf16
  d |= 1u << 10;                                  // B format: bf16
  d |= static_cast<uint32_t>((N >> 3) & 0x3F) << 17;
  d |= static_cast<uint32_t>(128 >> 4) << 24;     // M = 128
  return d;
}

// Same with f16 operands (A and B format 0).
__host__ __device__ __forceinline__ uint32_t idesc_f16(int N) {
  uint32_t d = 0;
  d |= 1u << 4;                                   // D format: f32
  d |= static_cast<uint32_t>((N >> 3) & 0x3F) << 17;
  d |= static_cast<uint32_t>(128 >> 4) << 24;     // M = 128
  return d;
}

// D(tmem) (+)= A(smem) x B(smem)^T, 16-bit operands (idesc_bf16 / idesc_f16), fp32 accumulate.
__device__ __forceinline__ void mma_kf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 op of this thread completed.
__device__ __forceinline__ void commit_to(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Copy a 32-row x 16-byte scale-factor chunk (512 contiguous bytes in shared
// memory) into TMEM columns [taddr, taddr+4) of all four 32-lane quadrants:
// lane l of every quadrant receives chunk row l % 32.
__device__ __forceinline__ void copy_sf_chunk(uint32_t taddr, const void* smem_chunk) {
  const uint64_t desc = smem_desc_kmajor(smem_chunk, 0, 128);
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n" ::"r"(taddr), "l"(desc)
               : "memory");
}

// Same copy from a prebuilt descriptor (smem_desc_kmajor(chunk, 0, 128)); a
// descriptor for a chunk `off` bytes further is desc + (off >> 4).
__device__ __forceinline__ void copy_sf_chunk_desc(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n" ::"r"(taddr), "l"(desc)
               : "memory");
}

// Each thread of a warp reads 8 consecutive 32-bit TMEM columns of its lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
}
// Each thread of a warp reads 16 consecutive 32-bit TMEM columns of its lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// Byte offset of scale (row m, 32-block kb) inside a 512-byte chunk covering
// 128 rows x 4 blocks: 32 rows of 16 bytes; row (m % 32) holds, for each
// quadrant q = m / 32, four bytes (one per block).
__host__ __device__ __forceinline__ int sf_chunk_offset(int m, int kb) {
  return (m & 31) * 16 + (m >> 5) * 4 + kb;
}

// Byte offset of the 16-byte K-chunk c of row r inside a canonical K-major
// operand of `rows` rows (rows multiple of 8): chunk-major, then 8-row groups.
__host__ __device__ __forceinline__ int kmajor_offset(int r, int c, int rows) {
  return c * rows * 16 + (r >> 3) * 128 + (r & 7) * 16;
}

}  // namespace tc
}  // namespace flyai
