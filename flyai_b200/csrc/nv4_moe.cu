// MiniMax-M2.5-style NVFP4 MoE layer on sm_100a (FLYAI_FMT_NVFP4 with
// FLYAI_GATE_SIGMOID_BF16 and FLYAI_ACT_SILU_BF16).
//
// Reference arithmetic (HF transformers' MiniMaxM2 modules, which the M2.5
// stage's vLLM FusedMoE configuration mirrors: engines/minimax_m25/m25_stage.py:
// 288-311, 412-416): weights are NVFP4-dequantised (e2m1 x e4m3 block-16 scale x
// fp32 global scale); gate/up = F.linear(x, W13) in bf16, chunk into halves,
// h = silu(gate) * up (bf16), down = F.linear(h, W2) (bf16), times the routing
// weight (fp32) to bf16, and bf16 index_add over experts in ascending id.
//
// Kernels (after f8_route_kernel<true>, which also splits the token rows into
// e2m1 terms): nv4_scatter_kernel gathers each chunk's term rows into B blocks,
// nv4_moe_kernel runs gate/up and down on tcgen05 kind::mxf4nvf4.block16 (one
// persistent CTA per SM), the combine folds the pair rows.  The pipeline is the
// FP8 layer's (one 128-wide K block per stage) with the block-scaled MMA: the
// weights' e4m3 scales and the terms' power-of-two ue4m3 scales go to TMEM with
// tcgen05.cp per stage.  A gate/up item accumulates its whole K in one TMEM
// buffer and the epilogue adds a token's 6 term columns times the row factor
// R once; a down item folds one buffer per K block, times that block's SwiGLU
// factor.  Every wait is bounded (~2 s).
#include <math.h>

#include "common.cuh"
#include "fp8_moe.cuh"
#include "nv4.cuh"
#include "tc_bank.cuh"
#include "tcgen05.cuh"

namespace flyai {

template <typename Kern, typename... Args>
static cudaError_t nv_launch(Kern kernel, dim3 grid, int block, size_t smem, cudaStream_t s,
                             bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------------------
// Bank packing
// ---------------------------------------------------------------------------
static size_t nv_global_offset(const flyai_moe_desc& d, int proj) {
  const size_t nexp = d.expert_end - d.expert_begin + d.n_shared;
  return nv_bank(d.hidden, d.inter, proj).expert * nexp;
}

size_t nv4_packed_bytes(const flyai_moe_desc& d, int proj) {
  const size_t nexp = d.expert_end - d.expert_begin + d.n_shared;
  return align_up(nv_global_offset(d, proj) + nexp * nv_bank(d.hidden, d.inter, proj).nglobal * 4, 256);
}

// One thread per 16-byte unit of a tile: data units c*128 + r (K-chunk c of row
// r, canonical K-major position), then the two scale chunks (32 lines each;
// line l holds rows l, l+32, l+64, l+96, four block-16 scales apiece).
// Scales come linear ([R, K/16] per expert) or, with swz, in the block-scale
// layout of the CUTLASS / FlashInfer NVFP4 kernels that vLLM swizzles a loaded
// layer's scales into (vllm/model_executor/layers/quantization/utils/
// nvfp4_utils.py swizzle_blockscale): per expert the [R, C = K/16] matrix padded
// to [roundup(R, 128), roundup(C, 4)], element (r, c) at
// ((r / 128 * (C' / 4) + c / 4) * 32 + r % 32) * 16 + (r % 128) / 32 * 4 + c % 4.
__global__ void nv4_pack_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                                uint8_t* __restrict__ packed, int nexp, int R, int K, NvBank b, int swz) {
  constexpr int kUnits = kNvTileBytes / 16;   // 576
  const size_t total = static_cast<size_t>(nexp) * b.RB * b.KB * b.tiles * kUnits;
  const int half_rows = b.tiles == 2 ? R / 2 : 0;
  for (size_t u = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; u < total;
       u += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t tile_id = u / kUnits;   // (e, rb, kb, tt)
    const int v = static_cast<int>(u % kUnits);
    const int tt = static_cast<int>(tile_id % b.tiles);
    const size_t blk = tile_id / b.tiles;
    const int kb = static_cast<int>(blk % b.KB);
    const int rb = static_cast<int>((blk / b.KB) % b.RB);
    const int e = static_cast<int>(blk / (static_cast<size_t>(b.KB) * b.RB));
    const size_t row0 = static_cast<size_t>(e) * R + tt * half_rows + rb * 128;
    uint4 out;
    if (v < kNvTile / 16) {
      const int c = v / 128, r = v % 128;
      out = *reinterpret_cast<const uint4*>(blocks + (row0 + r) * (K / 2) + kb * 64 + c * 16);
    } else {
      const int w = v - kNvTile / 16, j = w / 32, l = w % 32;
      const int C = K / 16, c0 = kb * 8 + j * 4;
      const size_t Rp = (static_cast<size_t>(R) + 127) / 128 * 128, Cp = (static_cast<size_t>(C) + 3) / 4 * 4;
      uint32_t word[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const size_t rl = static_cast<size_t>(tt) * half_rows + rb * 128 + 32 * q + l;   // row in the expert
        const uint8_t* s =
            swz ? scales + static_cast<size_t>(e) * Rp * Cp +
                      ((rl / 128 * (Cp / 4) + c0 / 4) * 32 + rl % 32) * 16 + (rl % 128) / 32 * 4
                : scales + (row0 + 32 * q + l) * C + c0;
        word[q] = static_cast<uint32_t>(s[0]) | (static_cast<uint32_t>(s[1]) << 8) |
                  (static_cast<uint32_t>(s[2]) << 16) | (static_cast<uint32_t>(s[3]) << 24);
      }
      out = make_uint4(word[0], word[1], word[2], word[3]);
    }
    *reinterpret_cast<uint4*>(packed + blk * b.block + static_cast<size_t>(tt) * kNvTileBytes +
                              static_cast<size_t>(v) * 16) = out;
  }
}

int launch_nv4_pack(const flyai_moe_desc& d, int proj, const void* blocks, const void* scales,
                    const void* global_scale, void* packed, cudaStream_t stream, bool swizzled) {
  const int nexp = d.expert_end - d.expert_begin + d.n_shared;
  if (nexp == 0) return FLYAI_OK;
  const NvBank b = nv_bank(d.hidden, d.inter, proj);
  const int R = proj == FLYAI_PROJ_W13 ? 2 * d.inter : d.hidden;
  const int K = proj == FLYAI_PROJ_W13 ? d.hidden : d.inter;
  nv4_pack_kernel<<<2368, 256, 0, stream>>>(static_cast<const uint8_t*>(blocks),
                                            static_cast<const uint8_t*>(scales),
                                            static_cast<uint8_t*>(packed), nexp, R, K, b, swizzled ? 1 : 0);
  note_launch();
  if (cudaGetLastError() != cudaSuccess) return FLYAI_ERR_CUDA;
  if (cudaMemcpyAsync(static_cast<uint8_t*>(packed) + nv_global_offset(d, proj), global_scale,
                      static_cast<size_t>(nexp) * b.nglobal * 4, cudaMemcpyDeviceToDevice,
                      stream) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  return FLYAI_OK;
}

// ---------------------------------------------------------------------------
// Token term rows -> each chunk's B blocks
// ---------------------------------------------------------------------------
struct NvScatterParams {
  const uint8_t* xq;    // [M][KB][kNvRowBytes]
  const uint8_t* xsf;   // [M][KB][kNvRowSf]
  const float* xr;      // [M][KB]
  const int32_t* perm;
  const int32_t* n_chunks;
  const int4* chunk_info;
  uint8_t* xb;
  int KB, k, P;
};

// CTA (group of 8 K blocks, chunk).  Token slots past the chunk's count are
// left as they are: they only feed MMA columns nobody reads.
__global__ void __launch_bounds__(256) nv4_scatter_kernel(const __grid_constant__ NvScatterParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.y;
  if (c >= *p.n_chunks) return;
  const int4 ci = p.chunk_info[c];
  const int kb0 = blockIdx.x * 8, nt = ci.z;
  constexpr int kPieces = kNvRowBytes / 16 + kTermSlots * 2 / 4 + 1;   // 24 data + 4 sf + 1 R
  for (int u = threadIdx.x; u < nt * 8 * kPieces; u += blockDim.x) {
    const int i = u / (8 * kPieces), rem = u % (8 * kPieces);
    const int kb = kb0 + rem / kPieces, pc = rem % kPieces;
    if (kb >= p.KB) continue;
    const int pos = ci.y + i;
    const int t = pos < p.P ? __ldg(&p.perm[pos]) / p.k : pos - p.P;
    const size_t src = static_cast<size_t>(t) * p.KB + kb;
    uint8_t* blk = p.xb + (static_cast<size_t>(c) * p.KB + kb) * kNvBBytes;
    if (pc < kNvRowBytes / 16) {
      *reinterpret_cast<uint4*>(blk + i * kNvRowBytes + pc * 16) =
          __ldg(reinterpret_cast<const uint4*>(p.xq + src * kNvRowBytes + pc * 16));
    } else if (pc < kPieces - 1) {
      // four scale words: step j = w / 2, slots (w % 2) * 4 .. +3
      const int w = pc - kNvRowBytes / 16, j = w >> 1, s0 = (w & 1) * 4;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.xsf + src * kNvRowSf + j * 32 + s0 * 4));
      uint8_t* dst = blk + kNvBData + j * kNvSfChunk + (8 * i + s0) * 16;
      *reinterpret_cast<uint32_t*>(dst) = v.x;
      *reinterpret_cast<uint32_t*>(dst + 16) = v.y;
      *reinterpret_cast<uint32_t*>(dst + 32) = v.z;
      *reinterpret_cast<uint32_t*>(dst + 48) = v.w;
    } else {
      reinterpret_cast<float*>(blk + kNvBData + 2 * kNvSfChunk)[i] = __ldg(&p.xr[src]);
    }
  }
}

// ---------------------------------------------------------------------------
// The expert kernel
// ---------------------------------------------------------------------------
// Items and their order are the FP8 kernel's: (chunk, 128-row block) of
// gate/up (w1 tile + w3 tile of the same rows, K = H) then of down (K = I);
// a chunk's down items wait for its I/128 gate/up items (chunk_done), whose
// epilogue splits the chunk's SwiGLU block into terms straight into hb.
// One thread issues tcgen05 ops at ~65 cycles each, and a gate/up stage takes 12
// of them (6 scale copies, 4 MMAs, commits) for 21 KB of data -- a single issuer
// caps a CTA near 37 GB/s.  Two issuer warps take alternate K blocks (by the
// global K-block count ks): each accumulates into its own half of the slot and
// the epilogue adds the halves.
// Accumulator slots (TMEM columns [0, 256)): slot u % 2 holds either one gate/up
// item (issuer p: gate at p*64, up at p*64 + 32) or a group of up to kNvDnGroup
// consecutive down K blocks (K block g at g*32).  acc_full counts both issuers.
constexpr int kNvStages = 8;
constexpr int kNvSlots = 2;
constexpr int kNvSlotCols = 128;
constexpr int kNvDnGroup = 4;
constexpr int kNvABytes = 2 * kNvTileBytes;  // 18432
constexpr int kNvStage = kNvABytes + kNvBBytes;
constexpr int kNvSfCols = 24;                // per stage: A 2 tiles x 2 chunks x 4, B 2 x 4
constexpr int kNvSfBase = kNvSlots * kNvSlotCols;
constexpr int kNvThreads = 224;              // warp 0 producer, 1 and 6 MMA issuers, 2..5 epilogue
static_assert(kNvStage % 16 == 0, "stage alignment");
static_assert(kNvSfBase + kNvStages * kNvSfCols <= 512, "tensor memory budget");
// Each issuer waits only for the stages of its own K blocks (ks parity), by
// phase parity.  With an even stage count stage s = ks % S always carries K
// blocks of one parity, so an issuer waits for every use of its stages in order.
// With an odd count consecutive uses of a stage alternate between the issuers:
// an issuer then waits for use k+2 of a stage whose use k+1 (the other
// issuer's) may not have landed, and phase k+2 has the parity of phase k, which
// it already saw complete -- the wait passes early, the MMAs read a stage in
// mid-copy and the ring's phases fall out of step.
static_assert(kNvStages % 2 == 0, "stage s must carry K blocks of one issuer parity");
static_assert(kNvDnGroup * kNvN <= kNvSlotCols && 4 * kNvN <= kNvSlotCols, "slot layout");

struct NvParams {
  const uint8_t* w13;
  const uint8_t* w2;
  NvBank b13, b2;
  const float* g13;   // [E', 2] global scales of w1, w3
  const float* g2;    // [E']
  const int32_t* n_chunks;
  const int4* chunk_info;
  int32_t* chunk_done;
  const int32_t* perm;
  const float* wts;
  const uint8_t* xb;
  uint8_t* hb;
  uint16_t* rows;
  const float* xr;    // [M][H/128] token row factors R (one value per row)
  int H, P, k;
  int32_t* err;
};

__host__ __device__ inline size_t nv_smem_bytes() {
  return static_cast<size_t>(kNvStages) * kNvStage + align_up(kNvBBytes, 128) + 4 * kNvChunk * 4 +
         (2 * kNvStages + 2 * kNvSlots + 1) * 8 + 16;
}

__global__ void __launch_bounds__(kNvThreads, 1) nv4_moe_kernel(const __grid_constant__ NvParams p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  constexpr int S = kNvStages;
  uint8_t* ring = sm;
  uint8_t* hst = sm + S * kNvStage;                                      // h B block staging
  float* red = reinterpret_cast<float*>(hst + align_up(kNvBBytes, 128)); // [4 warps][4 tokens]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 4 * kNvChunk);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + kNvSlots;
  uint64_t* epi_done = acc_empty + kNvSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      // the stage's MMAs completed + 4: the epilogue warps read a down stage's
      // SwiGLU factors (the MMA thread stands in for them on gate/up stages)
      mbar_init(&empty[s], 1 + 4);
    }
    for (int b = 0; b < kNvSlots; ++b) {
      mbar_init(&acc_full[b], 2);    // both issuers committed
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
  pdl_wait();   // plan, B blocks and cleared counters are visible
  pdl_launch_dependents();

  const int NI = p.b13.RB, NT = p.b2.RB, KB1 = p.b13.KB, KB2 = p.b2.KB;
  TcCursor cur;
  {
    const long long nch = *p.n_chunks, G = gridDim.x, b = blockIdx.x;
    const long long n_gu = nch * NI, n_dn = nch * NT;
    const long long g0 = n_gu * b / G, d0 = n_dn * b / G;
    cur.start(g0, n_gu * (b + 1) / G - g0, d0, n_dn * (b + 1) / G - d0, NI, NT);
  }
  if (!cur.valid()) {
    if (warp == 1) tc::tmem_dealloc(tbase, 512);
    return;
  }

  if (warp == 0) {
    // ---------------- producer ----------------
    // weights are read once: evict-first L2 policy (they recycle each other's
    // lines instead of evicting what else the L2 holds)
    const uint64_t wpol = l2_policy_evict_first();
    bool ok = true;
    uint32_t ks = 0;
    for (; cur.valid(); cur.next()) {
      if (lane == 0 && ok) {
        const TcItem t = cur.t;
        const int e = __ldg(&p.chunk_info[t.chunk].x);
        const NvBank& B = t.gu ? p.b13 : p.b2;
        const uint8_t* a = (t.gu ? p.w13 : p.w2) + static_cast<size_t>(e) * B.expert +
                           static_cast<size_t>(t.mt) * B.KB * B.block;
        const uint8_t* b = (t.gu ? p.xb : p.hb) + static_cast<size_t>(t.chunk) * B.KB * kNvBBytes;
        const uint32_t abytes = static_cast<uint32_t>(B.block);
        int kb = 0;
        if (!t.gu) {
          // A down item's weights do not depend on the chunk's gate/up tiles: its
          // first stages are requested before the wait, only the B blocks after it
          const int npre = B.KB < S ? B.KB : S;
          for (; kb < npre; ++kb) {
            const uint32_t s = (ks + kb) % S, use = (ks + kb) / S;
            if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&full[s], abytes + kNvBBytes);
            bulk_g2s_hint(ring + s * kNvStage, a + static_cast<size_t>(kb) * abytes, abytes, &full[s], wpol);
          }
          if (!wait_counter_geq(&p.chunk_done[t.chunk], NI)) ok = false;
          fence_proxy_async_global();
          for (int j = 0; j < kb; ++j) {   // (issued also after a failed wait: the phases complete)
            const uint32_t s = (ks + j) % S;
            bulk_g2s(ring + s * kNvStage + kNvABytes, b + static_cast<size_t>(j) * kNvBBytes, kNvBBytes, &full[s]);
          }
          ks += kb;
        }
        for (; ok && kb < B.KB; ++kb, ++ks) {
          const uint32_t s = ks % S, use = ks / S;
          if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], abytes + kNvBBytes);
          bulk_g2s_hint(ring + s * kNvStage, a + static_cast<size_t>(kb) * abytes, abytes, &full[s], wpol);
          bulk_g2s(ring + s * kNvStage + kNvABytes, b + static_cast<size_t>(kb) * kNvBBytes,
                   kNvBBytes, &full[s]);
        }
      }
      __syncwarp();
    }
    if (lane == 0) {
      for (uint32_t s = 0; s < S && s < ks; ++s) {   // copies in flight land before exit
        const uint32_t last = ((ks - 1 - s) / S) * S + s;
        if (!mbar_wait_bounded(&full[s], (last / S) & 1)) ok = false;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 6) {
    // ---------------- MMA issuers (K blocks with ks % 2 == par) ----------------
    const uint32_t par = warp == 6;
    bool ok = true;
    uint32_t ks = 0, su = 0;
    const uint32_t idesc = tc::idesc_nvf4(kNvN);
    const uint64_t a0 = tc::smem_desc_kmajor(ring, 2048, 128);
    const uint64_t b0 = tc::smem_desc_kmajor(ring + kNvABytes, kTcBlockBytes, kNvRowBytes);
    const uint64_t cp0 = tc::smem_desc_kmajor(ring, 0, 128);
    // the whole warp walks the items and waits (operands stay warp-uniform); one
    // elected lane issues the tcgen05 ops
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const int nk = t.gu ? KB1 : KB2, tiles = t.gu ? 2 : 1;
      const int gsize = t.gu ? nk : kNvDnGroup;   // K blocks per slot use
      bool fresh = true;                          // next MMA starts this issuer's accumulator
      for (int kb = 0; kb < nk; ++kb, ++ks) {
        const uint32_t slot = su % kNvSlots;
        const int g = kb % gsize;
        if (g == 0 && ok && su >= kNvSlots)
          ok = __all_sync(0xffffffffu, mbar_wait_bounded(&acc_empty[slot], ((su / kNvSlots) - 1) & 1));
        if (g == 0) fresh = true;
        if ((ks & 1u) == par && ok) {
          const uint32_t s = ks % S;
          ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (ks / S) & 1));
          if (ok) {
            tc::fence_after_sync();
            const uint32_t st16 = static_cast<uint32_t>((s * kNvStage) >> 4);
            const uint32_t sf = tbase + kNvSfBase + s * kNvSfCols;
            // gate/up: this issuer's half; down: K block g's columns
            const uint32_t d = tbase + slot * kNvSlotCols + (t.gu ? par * 2 * kNvN : g * kNvN);
            const bool acc0 = t.gu ? !fresh : false;
            if (elect_one()) {
              // scales to TMEM: A tile tt step j at sf + tt*8 + j*4, B step j at sf + 16 + j*4
              for (int tt = 0; tt < tiles; ++tt)
#pragma unroll
                for (int j = 0; j < 2; ++j)
                  tc::copy_sf_chunk_desc(sf + tt * 8 + j * 4,
                                         cp0 + st16 + ((tt * kNvTileBytes + kNvTile + j * kNvSfChunk) >> 4));
#pragma unroll
              for (int j = 0; j < 2; ++j)
                tc::copy_sf_chunk_desc(sf + 16 + j * 4,
                                       cp0 + st16 + ((kNvABytes + kNvBData + j * kNvSfChunk) >> 4));
              for (int tt = 0; tt < tiles; ++tt)
#pragma unroll
                for (int j = 0; j < 2; ++j)   // K = 64 per MMA: K-chunks 2j, 2j+1
                  tc::mma_nvf4(d + tt * kNvN, a0 + st16 + ((tt * kNvTileBytes + j * 4096) >> 4),
                               b0 + st16 + ((j * 2 * kTcBlockBytes) >> 4), idesc, sf + tt * 8 + j * 4,
                               sf + 16 + j * 4, acc0 || j > 0);
              tc::commit_to(&empty[s]);
              if (t.gu) mbar_arrive_cnt(&empty[s], 4);   // gate/up stages have no epilogue reader
            }
            __syncwarp();
            fresh = false;
          }
        }
        if (g == gsize - 1 || kb == nk - 1) {   // slot use complete: this issuer's part
          if (elect_one()) tc::commit_to(&acc_full[slot]);
          __syncwarp();
          ++su;
        }
      }
    }
    if (lane == 0) {
      if (!mbar_wait_bounded(epi_done, 0)) ok = false;
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
    if (warp == 1) {
      tc::fence_after_sync();
      tc::tmem_dealloc(tbase, 512);
    }
  } else {
    // ---------------- epilogue (TMEM lane quadrant = warp % 4) ----------------
    const int q = warp & 3;
    const int r = 32 * q + lane;   // row of the 128-row block
    bool ok = true;
    uint32_t su = 0, ks = 0;
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const int4 ci = __ldg(&p.chunk_info[t.chunk]);
      const int e = ci.x, pos0 = ci.y, nt = ci.z;
      float accg[kNvChunk], accu[kNvChunk];
#pragma unroll
      for (int i = 0; i < kNvChunk; ++i) accg[i] = accu[i] = 0.f;
      if (t.gu) {
        // one slot, both issuers' halves (a single K block: only its issuer's)
        const uint32_t ks0 = ks;
        ks += KB1;   // gate/up stages are released by the issuers alone
        const uint32_t slot = su % kNvSlots;
        float R[kNvChunk];   // token row factors (the route kernel's split)
#pragma unroll
        for (int i = 0; i < kNvChunk; ++i) {
          const int pos = pos0 + (i < nt ? i : 0);
          const int tok = pos < p.P ? __ldg(&p.perm[pos]) / p.k : pos - p.P;
          R[i] = __ldg(&p.xr[static_cast<size_t>(tok) * KB1]);
        }
        if (ok && !mbar_wait_bounded(&acc_full[slot], (su / kNvSlots) & 1)) ok = false;
        tc::fence_after_sync();
        const uint32_t ta = tbase + slot * kNvSlotCols + ((32u * q) << 16);
        const int h0 = KB1 > 1 ? 0 : static_cast<int>(ks0 & 1u), h1 = KB1 > 1 ? 2 : h0 + 1;
        for (int hf = h0; hf < h1; ++hf) {
          uint32_t g0[16], g1[16], u0[16], u1[16];
          tc::tmem_ld16(ta + hf * 2 * kNvN, g0);
          tc::tmem_ld16(ta + hf * 2 * kNvN + 16, g1);
          tc::tmem_ld16(ta + hf * 2 * kNvN + kNvN, u0);
          tc::tmem_ld16(ta + hf * 2 * kNvN + kNvN + 16, u1);
          tc::tmem_wait_ld();
          // token i's term columns are 8i .. 8i+5
#pragma unroll
          for (int i = 0; i < kNvChunk; ++i) {
            float sg = 0.f, su2 = 0.f;
#pragma unroll
            for (int tt = 0; tt < kNvTerms; ++tt) {
              const int col = 8 * i + tt;
              sg = __fadd_rn(sg, __uint_as_float(col < 16 ? g0[col & 15] : g1[col & 15]));
              su2 = __fadd_rn(su2, __uint_as_float(col < 16 ? u0[col & 15] : u1[col & 15]));
            }
            accg[i] = fmaf(sg, R[i], accg[i]);
            accu[i] = fmaf(su2, R[i], accu[i]);
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[slot]);
        ++su;
      } else {
        for (int kb0 = 0; kb0 < KB2; kb0 += kNvDnGroup) {
          const int ng = min(kNvDnGroup, KB2 - kb0);
          const uint32_t slot = su % kNvSlots;
          float R[kNvDnGroup][kNvChunk];   // the group's SwiGLU factors, from the stages' B blocks
#pragma unroll
          for (int g = 0; g < kNvDnGroup; ++g) {
            if (g < ng) {
              const uint32_t s = ks % S;
              if (ok && !mbar_wait_bounded(&full[s], (ks / S) & 1)) ok = false;
              const float4 rf = *reinterpret_cast<const float4*>(ring + s * kNvStage + kNvABytes +
                                                                 kNvBData + 2 * kNvSfChunk);
              R[g][0] = rf.x, R[g][1] = rf.y, R[g][2] = rf.z, R[g][3] = rf.w;
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[s]);
              ++ks;
            }
          }
          if (ok && !mbar_wait_bounded(&acc_full[slot], (su / kNvSlots) & 1)) ok = false;
          tc::fence_after_sync();
          const uint32_t ta = tbase + slot * kNvSlotCols + ((32u * q) << 16);
#pragma unroll
          for (int g = 0; g < kNvDnGroup; ++g) {
            if (g < ng) {
              uint32_t g0[16], g1[16];
              tc::tmem_ld16(ta + g * kNvN, g0);
              tc::tmem_ld16(ta + g * kNvN + 16, g1);
              tc::tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < kNvChunk; ++i) {
                float sg = 0.f;
#pragma unroll
                for (int tt = 0; tt < kNvTerms; ++tt) {
                  const int col = 8 * i + tt;
                  sg = __fadd_rn(sg, __uint_as_float(col < 16 ? g0[col & 15] : g1[col & 15]));
                }
                accg[i] = fmaf(sg, R[g][i], accg[i]);
              }
            }
          }
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[slot]);
          ++su;
        }
      }
      // (after a failed wait the item still runs through the named barriers,
      // which every epilogue warp must reach equally often; its data is void)
      if (t.gu) {
        const float g1 = __ldg(&p.g13[2 * e]), g3 = __ldg(&p.g13[2 * e + 1]);
        float h[kNvChunk];
#pragma unroll
        for (int i = 0; i < kNvChunk; ++i) {
          const float gate = bf16r(__fmul_rn(accg[i], g1)), up = bf16r(__fmul_rn(accu[i], g3));
          const float sg = bf16r(__fdiv_rn(gate, __fadd_rn(1.f, expf(-gate))));
          h[i] = i < nt ? bf16r(__fmul_rn(sg, up)) : 0.f;
        }
        // split the chunk's 128-element SwiGLU block (row r = K element r) into terms
#pragma unroll
        for (int i = 0; i < kNvChunk; ++i) {
          const float a = warp_max(fabsf(h[i]));
          if (lane == 0) red[q * kNvChunk + i] = a;
        }
        named_barrier_sync(1, 128);
        float hn[kNvChunk];
        int rexp[kNvChunk];
#pragma unroll
        for (int i = 0; i < kNvChunk; ++i) {
          const float m = fmaxf(fmaxf(red[i], red[kNvChunk + i]),
                                fmaxf(red[2 * kNvChunk + i], red[3 * kNvChunk + i]));
          rexp[i] = nv_block_exp(m);
          hn[i] = __fmul_rn(h[i], exp2i(-rexp[i]));
        }
        const int chunk32 = r >> 5, in32 = r & 31, blk16 = (r & 63) >> 4, step = r >> 6;
#pragma unroll 1
        for (int tt = 0; tt < kNvTerms; ++tt) {
#pragma unroll
          for (int i = 0; i < kNvChunk; ++i) {
            float bm = fabsf(hn[i]);
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
            const int ex = nv_term_exp(bm);
            uint32_t code = 0;
            if (ex != -127) {
              code = f32x2_to_e2m1x2(__fmul_rn(hn[i], exp2i(-ex)), 0.f) & 0xFu;
              const float qv = e2m1x2_to_f32x2(code).x;
              hn[i] = __fsub_rn(hn[i], __fmul_rn(qv, exp2i(ex)));
            }
            const uint32_t other = __shfl_xor_sync(0xffffffffu, code, 1);
            if ((r & 1) == 0)
              hst[i * kNvRowBytes + chunk32 * (kNvTerms * 16) + tt * 16 + (in32 >> 1)] =
                  static_cast<uint8_t>(code | (other << 4));
            if ((r & 15) == 0)
              hst[kNvBData + step * kNvSfChunk + (8 * i + tt) * 16 + blk16] =
                  static_cast<uint8_t>(ex == -127 ? 0u : ue4m3_pow2(ex));
          }
        }
        if (r < 2 * kNvChunk * (kTermSlots - kNvTerms)) {   // zero scales of the unused slots
          const int j = r & 1, i = (r >> 1) % kNvChunk, sl = kNvTerms + (r >> 1) / kNvChunk;
          *reinterpret_cast<uint32_t*>(hst + kNvBData + j * kNvSfChunk + (8 * i + sl) * 16) = 0u;
        }
#pragma unroll
        for (int i = 0; i < kNvChunk; ++i)
          if (r == i) reinterpret_cast<float*>(hst + kNvBData + 2 * kNvSfChunk)[i] = exp2i(rexp[i]);
        named_barrier_sync(1, 128);
        uint8_t* blk = p.hb + (static_cast<size_t>(t.chunk) * KB2 + t.mt) * kNvBBytes;
        for (int u = r; u < kNvBBytes / 16; u += 128)
          *reinterpret_cast<uint4*>(blk + u * 16) = *reinterpret_cast<const uint4*>(hst + u * 16);
        fence_proxy_async_global();
        __threadfence();
        named_barrier_sync(1, 128);
        if (r == 0) atomicAdd(&p.chunk_done[t.chunk], 1);
      } else {
        const float g2 = __ldg(&p.g2[e]);
        const int col = t.mt * 128 + r;
#pragma unroll
        for (int i = 0; i < kNvChunk; ++i) {
          if (i < nt) {
            const float o = bf16r(__fmul_rn(accg[i], g2));
            const int flat = __ldg(&p.perm[pos0 + i]);   // rows by flat pair index
            p.rows[static_cast<size_t>(flat) * p.H + col] = float_to_bf16_bits(__fmul_rn(o, __ldg(&p.wts[flat])));
          }
        }
      }
    }
    if (!ok) atomicOr(p.err, kErrWaitTimeout);
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(epi_done);
  }
}

int launch_nv4_experts(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                       void* y, uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream,
                       cudaEvent_t ev0, cudaEvent_t ev1) {
  (void)x;   // the route kernel split the token rows into ws.xq / ws.xsf / ws.xs
  if (M == 0) return FLYAI_OK;
  const int P = M * d.top_k, KB = d.hidden / 128;
  NvScatterParams sp{ws.xq, ws.xsf, ws.xs, ws.perm, ws.n_chunks, ws.chunk_info, ws.xb, KB, d.top_k, P};
  if (nv_launch(nv4_scatter_kernel, dim3((KB + 7) / 8, f8_max_chunks(d, M)), 256, 0, stream, true,
                sp) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();

  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem = nv_smem_bytes();
  if (smem > static_cast<size_t>(max_smem)) return FLYAI_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(nv4_moe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  NvParams prm{};
  prm.w13 = static_cast<const uint8_t*>(w.w13);
  prm.w2 = static_cast<const uint8_t*>(w.w2);
  prm.b13 = nv_bank(d.hidden, d.inter, FLYAI_PROJ_W13);
  prm.b2 = nv_bank(d.hidden, d.inter, FLYAI_PROJ_W2);
  prm.g13 = reinterpret_cast<const float*>(prm.w13 + nv_global_offset(d, FLYAI_PROJ_W13));
  prm.g2 = reinterpret_cast<const float*>(prm.w2 + nv_global_offset(d, FLYAI_PROJ_W2));
  prm.n_chunks = ws.n_chunks;
  prm.chunk_info = ws.chunk_info;
  prm.chunk_done = ws.chunk_done;
  prm.perm = ws.perm;
  prm.wts = ws.wts;
  prm.xb = ws.xb;
  prm.hb = ws.hb;
  prm.rows = rows;
  prm.xr = ws.xs;
  prm.H = d.hidden;
  prm.P = P;
  prm.k = d.top_k;
  prm.err = ws.err;
  if (ev0 && ev1 && cudaEventRecord(ev0, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  if (nv_launch(nv4_moe_kernel, dim3(sms), kNvThreads, smem, stream, true, prm) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  if (ev0 && ev1 && cudaEventRecord(ev1, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  return y ? launch_fp8_combine(d, M, rows, y, ws, stream, true) : FLYAI_OK;
}

}  // namespace flyai
