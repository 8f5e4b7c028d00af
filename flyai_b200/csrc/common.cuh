// Shared device helpers for the sm_100a MoE kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/flyai_moe.h"

namespace flyai {

// Library-wide launch counter (host side), read through flyai_moe_launch_count().
void note_launch(int n = 1);

constexpr int kMaxTopK = 8;
constexpr int kMaxTopKExternal = 16;   // FLYAI_GATE_EXTERNAL (Kimi-K3) layers

// ---- bf16 arithmetic with the reference's rounding points -------------------
// The reference materialises every elementwise result in bf16 (torch CPU ops on
// bf16 tensors compute in fp32 and round once, round-to-nearest-even).  These
// helpers use the _rn intrinsics so nvcc never contracts a*b+c into one FMA.
__device__ __forceinline__ float bf16r(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t float_to_bf16_bits(float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&h);
}

// e8m0 scale byte -> 2^(s-127) as fp32 (s=0 is the subnormal 2^-127, s=255 NaN).
__device__ __forceinline__ float e8m0_to_float(uint32_t s) {
  s &= 0xFFu;
  if (s == 0u) return __uint_as_float(0x00400000u);
  if (s == 255u) return __uint_as_float(0x7FC00000u);
  return __uint_as_float(s << 23);
}

// 2^p as fp32 for p in [-126, 127].
__device__ __forceinline__ float exp2i(int p) {
  return __uint_as_float(static_cast<uint32_t>(p + 127) << 23);
}

// Four e2m1x2 bytes of a word -> four f16x2 registers (hardware cvt, exact).
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t& r0, uint32_t& r1,
                                                 uint32_t& r2, uint32_t& r3) {
  asm("{\n\t.reg .b8 q0, q1, q2, q3;\n\t"
      "mov.b32 {q0, q1, q2, q3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, q0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, q1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, q2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, q3;\n\t}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_nc_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];\n" : "=r"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- mbarrier / bulk copy / programmatic dependent launch -------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Raise the transaction count of the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait on an mbarrier phase: gives up after ~limit_ns (returns false).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on bar.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// L2 cache policy for data read once (weights streamed by the expert kernels):
// its lines are the first candidates for eviction.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
// bulk_g2s with an L2 cache policy (l2_policy_evict_first).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;\n" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Generic-proxy global writes seen so far become visible to later bulk copies.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;\n" ::: "memory");
}
// Bounded wait until a global counter reaches target (acquire): false after ~limit_ns.
__device__ __forceinline__ bool wait_counter_geq(const int32_t* c, int target,
                                                 uint64_t limit_ns = 2000000000ull) {
  if (ld_acquire_gpu(c) >= target) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 64; ++i) {
      if (ld_acquire_gpu(c) >= target) return true;
      __nanosleep(32);
    }
    if (global_ns() - t0 > limit_ns) return false;
  }
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
// One lane of the (fully active) warp gets true.  Issue paths that run the whole
// warp through the loop and predicate only the tcgen05 / bulk-copy instruction on
// this keep their operands warp-uniform.
__device__ __forceinline__ bool elect_one() {
  uint32_t is_leader;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(is_leader));
  return is_leader != 0;
}
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ uint4 lds128(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
__device__ __forceinline__ uint32_t lds32(const void* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// Error bits a kernel can leave in the workspace (read back with flyai_moe_read_error).
constexpr int32_t kErrWaitTimeout = 1;
constexpr int32_t kErrBadIndex = 2;   // an expert id or table entry out of range (read as 0)

// Expert-parallel mailbox (flyai_moe_ep_alloc): kEpFlagBytes of flag words, then
// the pair-row buffers.  Word r = the last epoch rank r finished; word
// kEpFailWord + r = the last epoch whose expert kernel on rank r gave up on a
// bounded wait (its rows are incomplete).
constexpr int kEpFlagBytes = 256;
constexpr int kEpFailWord = 16;

constexpr int kTcChunk = 4;      // tokens of one expert per chunk, tcgen05 verify kernel
constexpr int kTcPfChunk = 128;   // pairs per chunk, tcgen05 prefill kernel (the MMA's N)
constexpr int kTcPrefillMinTokens = 65;   // batches this large take the prefill kernel
constexpr int kTcPfK = 64;          // K elements per bf16 row slice of the prefill kernel
constexpr int kTcPfBlk = kTcPfChunk * kTcPfK * 2;   // 16 KB: one slice of a full chunk
constexpr int kChunkRowStride = 16;   // token-row slots per chunk descriptor (verify chunks)
// Pairs per chunk of the tcgen05 kernels for a batch of M tokens.
__host__ __device__ inline int tc_chunk_tokens(int M) {
  return M >= kTcPrefillMinTokens ? kTcPfChunk : kTcChunk;
}
// Upper bound on the prefill chunks of P pairs over El experts: every non-empty
// expert has one partial chunk at most.
__host__ __device__ inline int tc_pf_max_chunks(size_t P, size_t El) {
  return static_cast<int>((El < P ? El : P) + P / kTcPfChunk + 1);
}
constexpr int kTerms = 6;        // e2m1 terms an activation row is split into for kind::mxf4
constexpr int kNpLogitSlices = 8;   // K slices of the prefill router logits (fp64 partial sums)

// ---- workspace layout -------------------------------------------------------
// Words of the route ticket region (the first 512 bytes of the workspace in
// every format; the FP8/NVFP4 layout uses words 0..65 only).
constexpr int kTicketEp = 65;            // expert-parallel CTA count, failure word
constexpr int kTicketGridBarrier = 67;   // fused layer's grid barrier: arrivals, generation

// All regions 256-byte aligned, carved in this order from the caller's buffer.
struct Workspace {
  float* logits;       // [M, E] fp32 holding bf16 values
  int32_t* ids;        // [M*k]
  float* wts;          // [M*k] fp32 holding bf16 values
  int32_t* counts;     // [E_local]
  int32_t* offsets;    // [E_local + 1]
  int32_t* active;     // [E_local]  local expert index of each non-empty expert
  int32_t* n_active;   // [1]
  int32_t* perm;       // [M*k] flat pair index at each permuted position
  uint16_t* pair_out;  // [M*k, H] bf16 weighted expert outputs, flat pair order
  int32_t* err;        // [1] error bits set by kernels (kErr*)
  int32_t* dbg;        // [8] first failure details of the self-checking build
  int32_t* route_ticket; // [1 + 64 + 2 + 2] at offset 0: tokens the fused route kernel
                         //     finished, per token its logit CTAs that finished, then
                         //     CTAs of the expert-parallel expert kernel that finished
                         //     and whether one of them gave up on a wait, then the fused
                         //     layer's grid barrier (arrivals, generation); must be 0
                         //     before first use, restored to 0 by every call (the
                         //     generation word excepted: any value serves)
  int32_t* fold_ticket;  // [M * H/16] contributions per (token, 16-row output tile);
                         //     cleared by the route step of every call
  int32_t* n_chunks;   // [1] number of chunks (tc_chunk_tokens pairs each) over all non-empty experts
  int32_t* chunk_slot; // [max_chunks] active-list slot of each chunk
  int32_t* chunk_c0;   // [max_chunks] first token (within the expert) of each chunk
  uint8_t* x_terms;    // [M][H/32][kTerms][16] e2m1 terms of every token row (tensor-core path)
  uint8_t* x_sf;       // [M][H/128][8][16] their e8m0 scales (4 used bytes per 16)
  uint8_t* h_terms;    // [M*k][I/32][kTerms][16] terms of the SwiGLU rows, permuted order
  uint8_t* h_sf;       // [M*k][I/128][8][16]
  uint8_t* pxb;        // prefill only: [pf_max_chunks][H/64][kTcPfBlk] bf16 token rows by chunk
  uint8_t* phb;        // prefill only: [pf_max_chunks][I/64][kTcPfBlk] bf16 SwiGLU rows by chunk
  int32_t* pcf;        // prefill only: [pf_max_chunks][kTcPfChunk] flat pair index per chunk slot
  float* pcw;          // prefill only: [pf_max_chunks][kTcPfChunk] routing weight per chunk slot
  double* plog;        // prefill only: [kNpLogitSlices][M, E] fp64 partial router logits
  float* pxm;          // prefill only: [kNpLogitSlices][M] partial row maxima of |x| (unused)
  int pf_max_chunks;
  int4* chunk_info;    // [max_chunks] (local expert, first permuted position, tokens, 0)
  int32_t* chunk_rows; // [max_chunks][kChunkRowStride] token row of each of the chunk's tokens
  int32_t* chunk_done; // [max_chunks] gate/up tiles of the chunk finished (cleared by route)
  int max_chunks;
  size_t total;
};

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline Workspace carve_workspace(const flyai_moe_desc& d, int M, void* base) {
  Workspace w{};
  const size_t E = d.num_experts, El = d.expert_end - d.expert_begin, k = d.top_k;
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = base ? static_cast<char*>(base) + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  const size_t P = static_cast<size_t>(M) * k;
  // The route ticket sits at offset 0 whatever the descriptor, so a workspace
  // (or the no-allocation scratch array) reused with another descriptor still
  // finds it where the previous call restored it to zero.
  w.route_ticket = reinterpret_cast<int32_t*>(take(4 * (kTicketGridBarrier + 2)));
  w.logits = reinterpret_cast<float*>(take(static_cast<size_t>(M) * E * 4));
  w.ids = reinterpret_cast<int32_t*>(take(P * 4));
  w.wts = reinterpret_cast<float*>(take(P * 4));
  w.counts = reinterpret_cast<int32_t*>(take(El * 4));
  w.offsets = reinterpret_cast<int32_t*>(take((El + 1) * 4));
  w.active = reinterpret_cast<int32_t*>(take(El * 4));
  w.n_active = reinterpret_cast<int32_t*>(take(4));
  w.perm = reinterpret_cast<int32_t*>(take(P * 4));
  w.pair_out = reinterpret_cast<uint16_t*>(take(P * static_cast<size_t>(d.hidden) * 2));
  w.err = reinterpret_cast<int32_t*>(take(4));
  w.dbg = reinterpret_cast<int32_t*>(take(32));
  w.fold_ticket = reinterpret_cast<int32_t*>(take(static_cast<size_t>(M) * (d.hidden / 16) * 4));
  w.n_chunks = reinterpret_cast<int32_t*>(take(4));
  w.max_chunks = static_cast<int>(El + (P + kTcChunk - 1) / kTcChunk + 1);   // smallest chunk size
  w.chunk_slot = reinterpret_cast<int32_t*>(take(static_cast<size_t>(w.max_chunks) * 4));
  w.chunk_c0 = reinterpret_cast<int32_t*>(take(static_cast<size_t>(w.max_chunks) * 4));
  // term scale rows: per 128-K group 8 term slots of 16 bytes (terms.cuh)
  const size_t sfh = static_cast<size_t>((d.hidden + 127) / 128) * 128;
  const size_t sfi = static_cast<size_t>((d.inter + 127) / 128) * 128;
  // the verify kernel's e2m1 term rows (calls of up to kTcPrefillMinTokens - 1 tokens)
  const size_t mv = M < kTcPrefillMinTokens ? M : kTcPrefillMinTokens - 1;
  w.x_terms = reinterpret_cast<uint8_t*>(take(mv * kTerms * (d.hidden / 2)));
  w.x_sf = reinterpret_cast<uint8_t*>(take(mv * sfh));
  w.h_terms = reinterpret_cast<uint8_t*>(take(mv * k * kTerms * (d.inter / 2)));
  w.h_sf = reinterpret_cast<uint8_t*>(take(mv * k * sfi));
  if (M >= kTcPrefillMinTokens) {   // the prefill kernel's bf16 row slices
    w.pf_max_chunks = tc_pf_max_chunks(P, El);
    w.pxb = reinterpret_cast<uint8_t*>(
        take(static_cast<size_t>(w.pf_max_chunks) * (d.hidden / kTcPfK) * kTcPfBlk));
    w.phb = reinterpret_cast<uint8_t*>(
        take(static_cast<size_t>(w.pf_max_chunks) * (d.inter / kTcPfK) * kTcPfBlk));
    w.pcf = reinterpret_cast<int32_t*>(take(static_cast<size_t>(w.pf_max_chunks) * kTcPfChunk * 4));
    w.pcw = reinterpret_cast<float*>(take(static_cast<size_t>(w.pf_max_chunks) * kTcPfChunk * 4));
    w.plog = reinterpret_cast<double*>(take(static_cast<size_t>(kNpLogitSlices) * M * E * 8));
    w.pxm = reinterpret_cast<float*>(take(static_cast<size_t>(kNpLogitSlices) * M * 4));
  }
  w.chunk_info = reinterpret_cast<int4*>(take(static_cast<size_t>(w.max_chunks) * 16));
  w.chunk_rows = reinterpret_cast<int32_t*>(take(static_cast<size_t>(w.max_chunks) * kChunkRowStride * 4));
  w.chunk_done = reinterpret_cast<int32_t*>(take(static_cast<size_t>(w.max_chunks) * 4));
  w.total = off;
  return w;
}

}  // namespace flyai
