// MXFP4 (GPT-OSS) expert projections for prefill-size batches on tcgen05.
//
// Same arithmetic as tc_experts.cu -- the reference's bf16 chain of
// transformers modeling_gpt_oss.py:69-114 -- arranged for many tokens per
// expert.  At verify sizes the layer streams weights and the activations go
// through the e2m1 MMA as six terms; with hundreds of tokens per expert the MMA
// work dominates and a 16-bit form is cheaper: an MXFP4 weight (e2m1 x 2^(e-127))
// is exact in bf16, and so is every bf16 activation, so the weights are expanded
// to bf16 in shared memory and multiplied on tcgen05 kind::f16 (exact products,
// fp32 accumulation) against the token rows as they are.  (The tensor core adds
// each K = 16 group into the accumulator with a truncation, so results differ
// from an IEEE fp32 dot product in the last bits of the accumulator.)
//
// Launches (after the route and its plan of kTcPfChunk-pair chunks):
// gp_scatter_kernel writes each chunk's bf16 token rows per 64-wide K slice in
// the 128-byte-swizzled K-major operand layout, plus the chunk's flat pair
// indices and routing weights; gp_moe_kernel runs gate/up + SwiGLU + down (one
// persistent CTA per SM, items dealt strided so concurrent CTAs share a chunk's
// rows and an expert's weights in L2); combine_kernel folds the pair rows.
//
// gp_moe_kernel, 736 threads:
//   warp 0      weight producer: per 128-wide K step of an item, bulk copies of
//               its bank tiles (e2m1 data + e8m0 scale chunk) into a ring of 4;
//   warps 1, 23 MMA issuers, one per tile of an item: 4 kind::f16 MMAs (K = 16)
//               per tile and slice into one of two 256-column TMEM slots (tile t
//               at +128 t); two issuers double the instruction rate that bounds
//               the small-N MMAs of partly filled chunks;
//   warps 2..5  epilogue: gate/up -> bias, clamp, SwiGLU in bf16 straight into
//               the chunk's down operand (chunk_done counts the items); down ->
//               bias, routing weight, bf16 pair rows by flat pair index;
//   warps 6..21 expansion: weight step -> two bf16 slices of the weight operand
//               (one group of 8 warps per 64-wide K half, one A slot each);
//   warp 22     row producer: per 64-wide K slice, the chunk's token rows (or
//               SwiGLU rows) into a ring of 5.
// A gate/up item is two consecutive 128-row tiles of the interleaved W13 (even
// rows gate, odd rows up): 128 SwiGLU features; the epilogue pairs TMEM lanes
// 2j, 2j+1.  A down item is two consecutive 128-row tiles of W2 (the last item
// of a projection may hold one).  Both operands use the
// 128-byte swizzle (tc::smem_desc_sw128).  Every wait is bounded (~2 s) and
// records kErrWaitTimeout.
#include <cuda_bf16.h>

#include "common.cuh"
#include "route.cuh"
#include "tc_bank.cuh"
#include "tcgen05.cuh"

namespace flyai {

namespace {
constexpr int kGpK = kTcPfK;                      // K elements per slice / MMA stage
constexpr int kGpN = kTcPfChunk;                  // pairs per chunk (MMA N <= 128)
constexpr int kGpBlk = kTcPfBlk;                  // 16 KB: one slice of a full chunk, bf16
constexpr int kGpRaw = 4;                         // weight ring (128-wide K steps)
constexpr int kGpRawTile = 8192 + 512;            // one tile's step: e2m1 data + scale chunk
constexpr int kGpRawBytes = 2 * kGpRawTile;
constexpr int kGpAStages = 2;                     // expanded slices, one per expansion group
constexpr int kGpATile = 128 * kGpK * 2;          // 16 KB: 128 rows x 64 K, bf16
constexpr int kGpAStage = 2 * kGpATile;
constexpr int kGpBStages = 5;
constexpr int kGpDqWarps = 16;
constexpr int kGpDqThreads = kGpDqWarps * 32;
constexpr int kGpRowWarp = 6 + kGpDqWarps;        // the row producer
constexpr int kGpMmaWarp2 = kGpRowWarp + 1;       // the second MMA issuer (an item's tile 1)
constexpr int kGpThreads = (kGpMmaWarp2 + 1) * 32;
constexpr int kGpSlotCols = 256;
constexpr int kGpOffA = kGpRaw * kGpRawBytes;
constexpr int kGpOffB = kGpOffA + kGpAStages * kGpAStage;
constexpr int kGpOffBar = kGpOffB + kGpBStages * kGpBlk;
static_assert(kGpOffA % 1024 == 0 && kGpOffB % 1024 == 0, "swizzled operands start on 1024 B");
static_assert(kGpATile % 1024 == 0 && kGpBlk % 1024 == 0, "swizzled operands start on 1024 B");
static_assert(kGpDqThreads == 2 * 2 * 128, "two groups x (row, 32-weight chunk) per thread");
static_assert(2 * kGpSlotCols <= 512, "tensor memory budget");
static_assert(kGpN <= 128 && kGpK * 2 == 128, "two tiles of N columns per slot; one 128-B line per row");
}  // namespace

// (1 KB of slack: the kernel rounds its dynamic shared memory base up to 1024 B)
__host__ __device__ inline size_t gp_smem_bytes() {
  return 1024 + kGpOffBar + (2 * kGpRaw + 2 * kGpAStages + 2 * kGpBStages + 2 * 2 + 1) * 8 + 16;
}

// ---------------------------------------------------------------------------
// Token rows -> each chunk's 64-wide K slices in the swizzled operand layout
// (token slot i is the 128-byte line i; slots from the chunk's count up to np =
// count rounded up to 16 are zero), and the chunk's flat pair indices and
// routing weights (column 0 of the grid).  CTA (group of 8 slices, chunk).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gp_scatter_kernel(const uint16_t* __restrict__ x,
                                                         const int32_t* __restrict__ perm,
                                                         const float* __restrict__ wts,
                                                         const int32_t* __restrict__ n_chunks,
                                                         const int4* __restrict__ chunk_info,
                                                         uint8_t* __restrict__ xb, int32_t* __restrict__ cf,
                                                         float* __restrict__ cw, int H, int k) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.y;
  if (c >= *n_chunks) return;
  const int4 ci = chunk_info[c];
  const int nt = ci.z, np = (nt + 15) & ~15, KS = H / kGpK, ks0 = blockIdx.x * 8;
  if (blockIdx.x == 0 && threadIdx.x < kGpN) {
    const int i = threadIdx.x;
    const int flat = i < nt ? __ldg(&perm[ci.y + i]) : 0;
    cf[static_cast<size_t>(c) * kGpN + i] = flat;
    cw[static_cast<size_t>(c) * kGpN + i] = i < nt ? __ldg(&wts[flat]) : 0.f;
  }
  const int units = 8 * np * 8;   // (slice, token slot, 16-byte unit)
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int q = u & 7, i = (u >> 3) % np, ks = ks0 + (u >> 3) / np;
    if (ks >= KS) continue;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (i < nt) {
      const int tok = __ldg(&perm[ci.y + i]) / k;
      v = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(tok) * H + ks * kGpK + q * 8));
    }
    *reinterpret_cast<uint4*>(xb + (static_cast<size_t>(c) * KS + ks) * kGpBlk + tc::sw128_offset(i, q)) = v;
  }
}

// ---------------------------------------------------------------------------
// The expert kernel
// ---------------------------------------------------------------------------
struct GpParams {
  TcProj gu, dn;          // banks, layouts, fp32 biases (act_* unused)
  const int32_t* n_chunks;
  const int4* chunk_info;  // (local expert, first position, pairs, 0)
  int32_t* chunk_done;
  const int32_t* cf;       // [chunks][kGpN] flat pair index per slot
  const float* cw;         // [chunks][kGpN] routing weight per slot
  const uint8_t* xb;       // [chunks][H/64][kGpBlk] token rows
  uint8_t* hb;             // [chunks][I/64][kGpBlk] SwiGLU rows
  uint16_t* pair_out;
  int hidden, inter;
  float limit, alpha;
  int32_t* err;
};

// The walk over an item's 128-wide K steps: K-tile kt of the bank, step s inside
// it, step width kw (128, or 64 for the tail of a K extent that is an odd
// multiple of 64).
struct GpSteps {
  int kt, s, kw, nkt, K;
  __device__ __forceinline__ void start(int K_) {
    K = K_;
    nkt = (K + kKT - 1) / kKT;
    kt = 0;
    s = 0;
    set_kw();
  }
  __device__ __forceinline__ int kt_len() const { return K - kt * kKT < kKT ? K - kt * kKT : kKT; }
  __device__ __forceinline__ void set_kw() {
    const int rem = kt_len() - s * 128;
    kw = rem < 128 ? rem : 128;
  }
  __device__ __forceinline__ bool valid() const { return kt < nkt; }
  __device__ __forceinline__ void next() {
    if ((s + 1) * 128 < kt_len()) {
      ++s;
    } else {
      ++kt;
      s = 0;
    }
    if (kt < nkt) set_kw();
  }
};

// 2^(e-127) * 2^112 as a bf16 pair (biased exponent e + 112; e <= 142).
__device__ __forceinline__ uint32_t gp_scale_pair(uint32_t e) {
  const uint32_t b = (e + 112u) << 7;
  return b | (b << 16);
}

// One 32-weight chunk (16 bytes of e2m1, low nibble = even K) with e8m0 scale e
// -> 16-byte units q0..q0+3 (8 weights each) of row `row` of a swizzled tile,
// exact.  An f16 e2m1 value shifted right by 3 is the bf16 of that value times
// 2^-112 (zeros stay zero); the bf16 product with 2^(e-15) is then exact.
// Scales above 2^15 (e > 142) take the product in fp32 instead.
__device__ __forceinline__ void gp_expand32(uint4 q, uint32_t e, uint8_t* tile, int row, int q0) {
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
  if (e <= 142u) {
    const uint32_t sc = gp_scale_pair(e);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t f[4], o[4];
      e2m1x8_to_f16x8(words[j], f[0], f[1], f[2], f[3]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t b = ((f[i] >> 3) & 0x0FFF0FFFu) | (f[i] & 0x80008000u);
        __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&b),
                                   *reinterpret_cast<const __nv_bfloat162*>(&sc));
        o[i] = *reinterpret_cast<uint32_t*>(&r);
      }
      *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, q0 + j)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    const float s = e8m0_to_float(e);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t f[4], o[4];
      e2m1x8_to_f16x8(words[j], f[0], f[1], f[2], f[3]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&f[i]));
        o[i] = static_cast<uint32_t>(float_to_bf16_bits(__fmul_rn(v.x, s))) |
               (static_cast<uint32_t>(float_to_bf16_bits(__fmul_rn(v.y, s))) << 16);
      }
      *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, q0 + j)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// The GPT-OSS gate/up chain for one (gate, up) accumulator pair.
__device__ __forceinline__ float gp_swiglu(float gate, float up, bool bias, float bg, float bu, float limit,
                                           float alpha) {
  gate = bf16r(gate);
  up = bf16r(up);
  if (bias) {
    gate = bf16r(__fadd_rn(gate, bg));
    up = bf16r(__fadd_rn(up, bu));
  }
  gate = gate > limit ? limit : gate;
  up = up > limit ? limit : (up < -limit ? -limit : up);
  const float ta = bf16r(__fmul_rn(gate, alpha));
  const float sg = bf16r(__frcp_rn(__fadd_rn(1.f, expf(-ta))));
  const float glu = bf16r(__fmul_rn(gate, sg));
  const float up1 = bf16r(__fadd_rn(up, 1.f));
  return bf16r(__fmul_rn(up1, glu));
}

__global__ void __launch_bounds__(kGpThreads, 1) gp_moe_kernel(const __grid_constant__ GpParams p) {
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  uint8_t* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);   // swizzle atoms need 1024 B
  constexpr int SA = kGpAStages, SB = kGpBStages, R = kGpRaw;
  uint8_t* raw = sm;
  uint8_t* sa = sm + kGpOffA;
  uint8_t* sb = sm + kGpOffB;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(sm + kGpOffBar);
  uint64_t* raw_empty = raw_full + R;   // the expansion warps are done with the step
  uint64_t* a_full = raw_empty + R;     // an expansion group wrote its slice
  uint64_t* a_empty = a_full + SA;      // the slice's MMAs completed
  uint64_t* b_full = a_empty + SA;      // the producer's bytes landed
  uint64_t* b_empty = b_full + SB;      // the slice's MMAs completed
  uint64_t* acc_full = b_empty + SB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* epi_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int r = 0; r < R; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], kGpDqWarps);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], kGpDqWarps / 2);   // the slot's expansion group
      mbar_init(&a_empty[s], 2);               // both issuers' MMAs of the slice
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 2);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 2);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(epi_done, 4);
    mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tmem_slot;
  pdl_wait();   // plan, token rows and cleared counters are visible
  pdl_launch_dependents();

  const TcLayout& L13 = p.gu.L;
  const TcLayout& L2 = p.dn.L;
  const int NI = (L13.MT + 1) / 2, NT = (L2.MT + 1) / 2;   // items of two tiles
  const int KS1 = p.hidden / kGpK, KS2 = p.inter / kGpK;
  TcStridedCursor cur;   // concurrent CTAs share a chunk's rows and an expert's weights in L2
  cur.start(blockIdx.x, gridDim.x, *p.n_chunks, NI, NT);
  if (!cur.valid()) {
    if (warp == 1) tc::tmem_dealloc(tbase, 512);
    return;
  }

  if (warp == 0) {
    // ---------------- weight producer ----------------
    bool ok = true;
    uint32_t rr = 0;
    for (; cur.valid(); cur.next()) {
      if (lane == 0 && ok) {
        const TcItem t = cur.t;
        const int e = __ldg(&p.chunk_info[t.chunk].x);
        const TcLayout& L = t.gu ? L13 : L2;
        const int mt0 = 2 * t.mt;
        const int tiles = min(2, L.MT - mt0);
        const uint8_t* ebase = (t.gu ? p.gu.bank : p.dn.bank) + static_cast<size_t>(e) * L.expert_bytes;
        GpSteps st;
        for (st.start(L.K); st.valid(); st.next(), ++rr) {
          const uint32_t r = rr % R;
          if (rr >= R && !mbar_wait_bounded(&raw_empty[r], ((rr / R) - 1) & 1)) {
            ok = false;
            break;
          }
          uint32_t abytes = 0;
          for (int tt = 0; tt < tiles; ++tt)
            abytes += static_cast<uint32_t>(tc_rows(L, mt0 + tt) * st.kw / 2 + 512);
          mbar_expect_tx(&raw_full[r], abytes);
          for (int tt = 0; tt < tiles; ++tt) {
            const int rows = tc_rows(L, mt0 + tt);
            const uint8_t* tile = ebase + tc_tile_offset(L, mt0 + tt, st.kt);
            uint8_t* dst = raw + r * kGpRawBytes + tt * kGpRawTile;
            bulk_g2s(dst, tile + static_cast<size_t>(st.s) * 4 * rows * 16,
                     static_cast<uint32_t>(rows * st.kw / 2), &raw_full[r]);
            bulk_g2s(dst + 8192, tile + static_cast<size_t>(rows) * (st.kt_len() / 2) + st.s * 512, 512,
                     &raw_full[r]);
          }
        }
      }
      __syncwarp();
    }
    if (lane == 0) {   // copies in flight land before exit
      for (uint32_t r = 0; r < R && r < rr; ++r) {
        const uint32_t last = ((rr - 1 - r) / R) * R + r;
        if (!mbar_wait_bounded(&raw_full[r], (last / R) & 1)) ok = false;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
  } else if (warp == kGpRowWarp) {
    // ---------------- row producer ----------------
    bool ok = true;
    uint32_t ks = 0;
    for (; cur.valid(); cur.next()) {
      if (lane == 0 && ok) {
        const TcItem t = cur.t;
        const int np = (__ldg(&p.chunk_info[t.chunk].z) + 15) & ~15;
        const uint8_t* b = (t.gu ? p.xb : p.hb) + static_cast<size_t>(t.chunk) * (t.gu ? KS1 : KS2) * kGpBlk;
        const uint32_t bbytes = static_cast<uint32_t>(np) * 128u;
        const int nsl = (t.gu ? p.hidden : p.inter) / kGpK;
        if (!t.gu) {   // the chunk's SwiGLU rows come from its gate/up items
          if (!wait_counter_geq(&p.chunk_done[t.chunk], NI)) ok = false;
          fence_proxy_async_global();
        }
        for (int sl = 0; ok && sl < nsl; ++sl, ++ks) {
          const uint32_t s = ks % SB;
          if (ks >= SB && !mbar_wait_bounded(&b_empty[s], ((ks / SB) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&b_full[s], bbytes);
          bulk_g2s(sb + s * kGpBlk, b + static_cast<size_t>(sl) * kGpBlk, bbytes, &b_full[s]);
        }
      }
      __syncwarp();
    }
    if (lane == 0) {
      for (uint32_t s = 0; s < SB && s < ks; ++s) {
        const uint32_t last = ((ks - 1 - s) / SB) * SB + s;
        if (!mbar_wait_bounded(&b_full[s], (last / SB) & 1)) ok = false;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
  } else if (warp == 1 || warp == kGpMmaWarp2) {
    // ---------------- MMA issuers ----------------
    // Issuer `me` multiplies tile `me` of every item (an item with one tile
    // leaves the second issuer only its commits).  The whole warp walks the
    // items and waits (operands stay warp-uniform); one elected lane issues the
    // tcgen05 instructions.
    const int me = warp == 1 ? 0 : 1;
    bool ok = true;
    uint32_t ks = 0, item = 0, ause[2] = {0u, 0u};
    const uint64_t a0 = tc::smem_desc_sw128(sa), b0 = tc::smem_desc_sw128(sb);
    for (; ok && cur.valid(); cur.next(), ++item) {
      const TcItem t = cur.t;
      const int np = (__ldg(&p.chunk_info[t.chunk].z) + 15) & ~15;
      const uint32_t idesc = tc::idesc_bf16(np);
      const TcLayout& L = t.gu ? L13 : L2;
      const bool mine = me < min(2, L.MT - 2 * t.mt);
      const uint32_t slot = item & 1u;
      if (item >= 2) ok = mbar_wait_bounded(&acc_empty[slot], ((item >> 1) - 1) & 1);
      ok = __all_sync(0xffffffffu, ok);
      tc::fence_after_sync();
      const uint32_t d = tbase + slot * kGpSlotCols;
      bool first = true;
      GpSteps st;
      for (st.start(L.K); ok && st.valid(); st.next()) {
        for (int h = 0; ok && h < st.kw / kGpK; ++h, ++ks) {
          const uint32_t u = ks % SB;
          ok = mbar_wait_bounded(&a_full[h], ause[h] & 1) && mbar_wait_bounded(&b_full[u], (ks / SB) & 1);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc::fence_after_sync();
          const uint64_t as = a0 + ((h * kGpAStage) >> 4), bs = b0 + ((u * kGpBlk) >> 4);
          if (elect_one()) {
            if (mine) {
#pragma unroll
              for (int i = 0; i < 4; ++i)   // K = 16 per MMA: 32 bytes into each 128-byte line
                tc::mma_kf16(d + me * 128, as + ((me * kGpATile + i * 32) >> 4), bs + i * 2, idesc,
                             !first || i > 0);
            }
            tc::commit_to(&a_empty[h]);
            tc::commit_to(&b_empty[u]);
          }
          __syncwarp();
          ++ause[h];
          first = false;
        }
      }
      if (ok && elect_one()) tc::commit_to(&acc_full[slot]);
      __syncwarp();
    }
    if (lane == 0) {
      if (!mbar_wait_bounded(epi_done, 0)) ok = false;   // last accumulator read
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
    if (me == 0) {
      tc::fence_after_sync();
      tc::tmem_dealloc(tbase, 512);
    }
  } else if (warp < 6) {
    // ---------------- epilogue (TMEM lane quadrant = warp % 4) ----------------
    const int q = warp & 3, m = 32 * q + lane;   // row of the 128-row tile
    const int par = lane & 1;                    // even lane: gate row, odd lane: up row
    bool ok = true;
    uint32_t item = 0;
    for (; cur.valid(); cur.next(), ++item) {
      const TcItem t = cur.t;
      const int4 ci = __ldg(&p.chunk_info[t.chunk]);
      const int e = ci.x, nt = ci.z, np = (nt + 15) & ~15;
      const uint32_t slot = item & 1u;
      if (ok && !mbar_wait_bounded(&acc_full[slot], (item >> 1) & 1)) ok = false;
      tc::fence_after_sync();
      const uint32_t ta = tbase + slot * kGpSlotCols + ((32u * q) << 16);
      if (t.gu) {
        const int tiles = min(2, L13.MT - 2 * t.mt);
        for (int tt = 0; tt < tiles; ++tt) {
          const int mtile = 2 * t.mt + tt;   // W13 tile: rows mtile*128 + m (2 inter rows = 128 per tile)
          const int row = mtile * 128 + m;
          const float bias_v = p.gu.bias ? __ldg(p.gu.bias + static_cast<size_t>(e) * L13.R + row) : 0.f;
          const float bias_o = __shfl_xor_sync(0xffffffffu, bias_v, 1);
          const float bg = par ? bias_o : bias_v, bu = par ? bias_v : bias_o;
          // feature m/2 -> slice mtile of the down operand, K element (m/2) % 64 there
          const int kk = m >> 1;
          uint8_t* hs = p.hb + (static_cast<size_t>(t.chunk) * KS2 + mtile) * kGpBlk + (kk & 7) * 2;
          for (int c0 = 0; c0 < np; c0 += 16) {
            uint32_t v[16];
            tc::tmem_ld16(ta + tt * 128 + c0, v);
            tc::tmem_wait_ld();
            // both lanes of a (gate, up) pair work: this lane takes the columns of
            // its parity, receiving the partner row's accumulator for them
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              const float a0v = ok ? __uint_as_float(v[2 * jj]) : 0.f;
              const float a1v = ok ? __uint_as_float(v[2 * jj + 1]) : 0.f;
              const float mine = par ? a1v : a0v, give = par ? a0v : a1v;
              const float got = __shfl_xor_sync(0xffffffffu, give, 1);
              const int i = c0 + 2 * jj + par;   // token slot
              const float h = i < nt ? gp_swiglu(par ? got : mine, par ? mine : got, p.gu.bias != nullptr, bg,
                                                 bu, p.limit, p.alpha)
                                     : 0.f;
              *reinterpret_cast<uint16_t*>(hs + tc::sw128_offset(i, kk >> 3)) = float_to_bf16_bits(h);
            }
          }
        }
      } else {
        const int32_t* cfl = p.cf + static_cast<size_t>(t.chunk) * kGpN;
        const float* cwt = p.cw + static_cast<size_t>(t.chunk) * kGpN;
        const int tiles = min(2, L2.MT - 2 * t.mt);
        for (int tt = 0; tt < tiles; ++tt) {
        const int row = (2 * t.mt + tt) * 128 + m;   // output column of the pair rows
        const bool live_row = row < L2.R;
        const float bias_v =
            (p.dn.bias && live_row) ? __ldg(p.dn.bias + static_cast<size_t>(e) * L2.R + row) : 0.f;
        for (int c0 = 0; c0 < np; c0 += 16) {
          uint32_t v[16];
          tc::tmem_ld16(ta + tt * 128 + c0, v);
          int fl[16];
          float wt[16];
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            const int4 a = __ldg(reinterpret_cast<const int4*>(cfl + c0 + j));
            const float4 b = __ldg(reinterpret_cast<const float4*>(cwt + c0 + j));
            fl[j] = a.x, fl[j + 1] = a.y, fl[j + 2] = a.z, fl[j + 3] = a.w;
            wt[j] = b.x, wt[j + 1] = b.y, wt[j + 2] = b.z, wt[j + 3] = b.w;
          }
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c0 + j < nt && live_row) {   // rows by flat pair index
              float o = bf16r(ok ? __uint_as_float(v[j]) : 0.f);
              if (p.dn.bias) o = bf16r(__fadd_rn(o, bias_v));
              o = bf16r(__fmul_rn(o, wt[j]));
              p.pair_out[static_cast<size_t>(fl[j]) * p.hidden + row] = float_to_bf16_bits(o);
            }
          }
        }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[slot]);
      if (t.gu) {   // release the item's SwiGLU rows to the chunk's down items
        fence_proxy_async_global();
        __threadfence();
        named_barrier_sync(1, 128);
        if (m == 0) atomicAdd(&p.chunk_done[t.chunk], 1);
      }
    }
    if (!ok) atomicOr(p.err, kErrWaitTimeout);
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(epi_done);
  } else {
    // ---------------- weight expansion ----------------
    // Two groups of 8 warps, one per 64-wide K half of a weight step: group g
    // writes the step's slice g, always into A slot g.  A thread expands the
    // 32-weight chunk cc of its row in its half, for each tile of the item.  A
    // 64-wide step (the tail of an odd K extent) has no second half: group 1
    // only releases it.
    static_assert(kGpAStages == 2, "one A slot per expansion group");
    const int et = threadIdx.x - 6 * 32;   // 0..kGpDqThreads-1
    const int grp = et >> 8, row = et & 127, cc = (et >> 7) & 1;
    bool ok = true;
    uint32_t rr = 0, ause = 0;
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const TcLayout& L = t.gu ? L13 : L2;
      const int mt0 = 2 * t.mt;
      const int tiles = min(2, L.MT - mt0);
      GpSteps st;
      for (st.start(L.K); st.valid(); st.next(), ++rr) {
        const uint32_t r = rr % R;
        const bool mine = grp * kGpK < st.kw;
        if (ok && !mbar_wait_bounded(&raw_full[r], (rr / R) & 1)) ok = false;
        // slot grp's previous use was this group's slice of an earlier step
        if (ok && mine && ause >= 1 && !mbar_wait_bounded(&a_empty[grp], (ause - 1) & 1)) ok = false;
        if (ok && mine) {
          const uint8_t* src = raw + r * kGpRawBytes;
          uint8_t* dst = sa + grp * kGpAStage;
          const int c = 2 * grp + cc;   // 32-weight chunk of the step
          for (int tt = 0; tt < tiles; ++tt) {
            const int rows = tc_rows(L, mt0 + tt);
            if (row < rows) {
              const uint8_t* tile = src + tt * kGpRawTile;
              const uint4 qd = lds128(tile + c * rows * 16 + (row >> 3) * 128 + (row & 7) * 16);
              const uint32_t e8 = tile[8192 + (row & 31) * 16 + (row >> 5) * 4 + c];
              gp_expand32(qd, e8, dst + tt * kGpATile, row, cc * 4);
            }
          }
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        }
        __syncwarp();
        if (ok && lane == 0) {
          if (mine) mbar_arrive(&a_full[grp]);
          mbar_arrive(&raw_empty[r]);
        }
        if (mine) ++ause;
      }
    }
    if (!ok && lane == 0) atomicOr(p.err, kErrWaitTimeout);
  }
}

int launch_tc_prefill(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                      uint16_t* pair_out, const Workspace& ws, cudaStream_t stream) {
  if (M == 0) return FLYAI_OK;
  if (!ws.pxb || d.hidden % kGpK || d.inter % kGpK) return FLYAI_ERR_UNSUPPORTED;
  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem = gp_smem_bytes();
  if (smem > static_cast<size_t>(max_smem)) return FLYAI_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(gp_moe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.stream = stream;
  cfg.gridDim = dim3((d.hidden / kGpK + 7) / 8, ws.pf_max_chunks);
  cfg.blockDim = dim3(256);
  if (cudaLaunchKernelEx(&cfg, gp_scatter_kernel, static_cast<const uint16_t*>(x),
                         static_cast<const int32_t*>(ws.perm), static_cast<const float*>(ws.wts),
                         static_cast<const int32_t*>(ws.n_chunks), static_cast<const int4*>(ws.chunk_info),
                         ws.pxb, ws.pcf, ws.pcw, d.hidden, d.top_k) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  GpParams prm{};
  prm.gu = TcProj{static_cast<const uint8_t*>(w.w13), tc_layout(d, FLYAI_PROJ_W13),
                  static_cast<const float*>(w.w13_bias), nullptr, nullptr};
  prm.dn = TcProj{static_cast<const uint8_t*>(w.w2), tc_layout(d, FLYAI_PROJ_W2),
                  static_cast<const float*>(w.w2_bias), nullptr, nullptr};
  prm.n_chunks = ws.n_chunks;
  prm.chunk_info = ws.chunk_info;
  prm.chunk_done = ws.chunk_done;
  prm.cf = ws.pcf;
  prm.cw = ws.pcw;
  prm.xb = ws.pxb;
  prm.hb = ws.phb;
  prm.pair_out = pair_out;
  prm.hidden = d.hidden;
  prm.inter = d.inter;
  prm.limit = d.swiglu_limit;
  prm.alpha = d.swiglu_alpha;
  prm.err = ws.err;
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kGpThreads);
  cfg.dynamicSmemBytes = smem;
  if (cudaLaunchKernelEx(&cfg, gp_moe_kernel, prm) != cudaSuccess) return FLYAI_ERR_CUDA;
  note_launch();
  return FLYAI_OK;
}

}  // namespace flyai
