// MXFP4 expert projections on the 5th-generation tensor cores (tcgen05).
//
// Reference arithmetic (transformers/models/gpt_oss/modeling_gpt_oss.py:69-114,
// dequant transformers/integrations/mxfp4.py:279-330) and rounding chain are the
// same as in mxfp4.cu; here the dot products run on the block-scaled MMA
// `tcgen05.mma.kind::mxf4.block_scale.block32`, which consumes the packed e2m1
// weights and their e8m0 per-32 scales directly -- no dequantisation
// instructions.  Both operands of that MMA are e2m1, so every bf16 activation
// row is split once into kTerms e2m1 rows with their own scales (terms.cuh); the
// terms are extra MMA columns (N = kTcChunk tokens x 8 term slots) and the
// epilogue adds a token's term columns in fp32.
//
// tc_moe_kernel runs gate/up and down of one layer call in a single launch, one
// persistent CTA per SM, warp-specialised (see the role comments in the kernel):
// a bulk-copy producer, two MMA-issuing warps, four epilogue warps and a stager
// of the B operand.  The combine into y is a separate PDL-chained kernel.
// Every wait is bounded (~2 s) and records kErrWaitTimeout.
#include <cstdlib>

#include "common.cuh"
#include "route.cuh"
#include "route_dev.cuh"
#include "tc_bank.cuh"
#include "tcgen05.cuh"
#include "terms.cuh"

namespace flyai {

bool tc_supported(const flyai_moe_desc& d) {
  return d.hidden % 64 == 0 && d.inter % 64 == 0 && d.hidden <= kTcMaxK && d.inter <= kTcMaxK;
}

size_t tc_packed_bytes(const flyai_moe_desc& d, int proj) {
  return tc_layout(d, proj).expert_bytes * static_cast<size_t>(d.expert_end - d.expert_begin);
}

// Bank row -> source row.  The W13 bank interleaves gate and up rows (gate j at
// 2j, up j at 2j+1: GPT-OSS's gate_up_proj order); a source holding w1's rows then
// w3's (split = inter) is interleaved on the way.
__device__ __forceinline__ int tc_src_row(int row, int split) {
  return split ? ((row & 1) ? split + (row >> 1) : (row >> 1)) : row;
}

// One thread per 16-byte chunk (one 32-element scale group of one row).
__global__ void tc_pack_data_kernel(const uint8_t* __restrict__ blocks,
                                    uint8_t* __restrict__ packed, int E, TcLayout L, int split) {
  const size_t per_expert = static_cast<size_t>(L.R) * L.G;
  const size_t total = per_expert * E;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(i / per_expert);
    const int rem = static_cast<int>(i % per_expert);
    const int row = rem / L.G, g = rem % L.G;
    const int mt = row / 128, r = row % 128, kt = (g * 32) / kKT, c = g - kt * (kKT / 32);
    const int rows_t = tc_rows(L, mt);
    uint8_t* dst = packed + static_cast<size_t>(e) * L.expert_bytes + tc_tile_offset(L, mt, kt) +
                   static_cast<size_t>(c) * rows_t * 16 + (r >> 3) * 128 + (r & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(
        blocks + ((static_cast<size_t>(e) * L.R + tc_src_row(row, split)) * L.G + g) * 16);
  }
}

// One thread per scale slot of every tile's chunks (rows padded to 128).
__global__ void tc_pack_scale_kernel(const uint8_t* __restrict__ scales,
                                     uint8_t* __restrict__ packed, int E, TcLayout L, int split) {
  const int chunks_full = kKT / 128;
  const size_t per_mtile = static_cast<size_t>(L.NKT) * chunks_full * 512;
  const size_t total = per_mtile * L.MT * E;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(i / (per_mtile * L.MT));
    size_t rem = i % (per_mtile * L.MT);
    const int mt = static_cast<int>(rem / per_mtile);
    rem %= per_mtile;
    const int kt = static_cast<int>(rem / (chunks_full * 512));
    const int off = static_cast<int>(rem % (chunks_full * 512));
    const int kt_len = tc_kt_len(L, kt);
    if (off / 512 >= (kt_len + 127) / 128) continue;
    const int b = off % 512;
    const int r = b / 16 + 32 * ((b % 16) / 4);          // inverse of the chunk layout
    const int g = kt * (kKT / 32) + (off / 512) * 4 + b % 4;
    const int rows_t = tc_rows(L, mt);
    uint8_t v = 127;                                      // neutral scale for padding
    if (r < rows_t && g < L.G)
      v = scales[(static_cast<size_t>(e) * L.R + tc_src_row(mt * 128 + r, split)) * L.G + g];
    packed[static_cast<size_t>(e) * L.expert_bytes + tc_tile_offset(L, mt, kt) +
           static_cast<size_t>(rows_t) * (kt_len / 2) + off] = v;
  }
}

int launch_tc_pack(const flyai_moe_desc& d, int proj, const void* blocks, const void* scales,
                   void* packed, cudaStream_t stream) {
  const TcLayout L = tc_layout(d, proj);
  const int El = d.expert_end - d.expert_begin;
  if (El == 0) return FLYAI_OK;
  // FLYAI_ACT_SITU W13 sources are [w1; w3]
  const int split = (d.activation == FLYAI_ACT_SITU && proj == FLYAI_PROJ_W13) ? d.inter : 0;
  tc_pack_data_kernel<<<2368, 256, 0, stream>>>(static_cast<const uint8_t*>(blocks),
                                                static_cast<uint8_t*>(packed), El, L, split);
  note_launch();
  tc_pack_scale_kernel<<<1184, 256, 0, stream>>>(static_cast<const uint8_t*>(scales),
                                                 static_cast<uint8_t*>(packed), El, L, split);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// The fused expert kernel
// ---------------------------------------------------------------------------
// Work items: (chunk, 128-row tile) of the gate/up projection and of the down
// projection, dealt to the CTAs round-robin in runs of kTcRun, gate/up first.  A chunk is up to
// kTcChunk tokens of one expert; its down tiles wait until all of its gate/up
// tiles (on any CTA) have written the SwiGLU rows, counted in chunk_done.
// Gate/up items never wait on anything and come first in every CTA, so the
// waits resolve; a chunk's gate/up tiles are dealt within one or two rounds,
// so they are long done when its down tiles come up.
constexpr int kTcN = kTcChunk * kTermSlots;                // 32: MMA N, column token*8 + term
constexpr int kTcAcc = 4;                                  // accumulator buffers
constexpr int kTcAccCols = 2 * kTcN;                       // even / odd K-tile halves
// The ring's stages are split between the two MMA issuers (issuer p: stages p,
// p + 2, ...; K-tile kt goes to issuer kt & 1), so every use of a stage is
// waited for by the one issuer that consumes it, in order.  (A stage shared by
// the issuers would let one of them wait for a use two phases after the last
// one it saw, which a parity wait cannot tell from that last phase.)
constexpr int kTcStages = 4;
constexpr int kTcHalfStages = kTcStages / 2;
static_assert(kTcStages % 2 == 0, "the ring splits evenly between the two issuers");
constexpr int kTcRun = 3;                                  // items per dealt run (TcRunCursor)
constexpr int kTcSfaCol = kTcAcc * kTcAccCols;             // A scales: 16 columns per ring stage
constexpr int kTcSfbCol = kTcSfaCol + 16 * kTcStages;      // B scales: 2 buffers x 4 per K group
static_assert(kTcSfbCol + 2 * 4 * (kTcMaxK / 128) <= 512, "tensor memory budget");
// warps: 0 producer, 1 and 7 MMA issuers (even / odd K-tiles), 2..5 epilogue, 6 B stager
constexpr int kTcThreads = 256;


struct TcParams {
  TcProj gu, dn;
  const int32_t* n_chunks;
  const int4* chunk_info;     // (local expert, first position, tokens, 0)
  const int32_t* chunk_rows;  // token row of each chunk token (gate/up activation rows)
  int32_t* chunk_done;
  const int32_t* perm;
  const float* wts;
  uint8_t* h_terms;           // SwiGLU rows as terms, by position (down activation rows)
  uint8_t* h_sf;
  uint16_t* pair_out;         // [P, H] weighted expert rows, flat pair order
  int hidden, inter, kmax;
  float limit, alpha;         // GPT-OSS clamp and alpha; situ: linear_beta (0 = none) and beta
  int situ;                   // FLYAI_ACT_SITU: Kimi-K3 activation, unweighted pair rows
  int32_t* err;
  // expert parallel over peer memory (ep_world > 0): pair rows go to every
  // rank's mailbox instead of pair_out, then this rank's flag is raised in each
  int ep_world, ep_rank;
  uint32_t ep_epoch;
  uint16_t* ep_rows[FLYAI_MOE_EP_MAX_RANKS];
  uint32_t* ep_flags[FLYAI_MOE_EP_MAX_RANKS];
  int32_t* ep_ticket;         // [0] CTAs that finished, [1] set when a wait gave up
                              // (workspace, self-resetting)
  // fused verify layer (tc_moe_kernel<true>): routing in the prologue, fold in
  // the down epilogue
  struct Route {
    const uint16_t* x;
    const uint16_t* wr;
    const uint16_t* br;
    int M, E, k;
    int e_begin, e_end;                     // this GPU's experts (expert parallel: a shard)
    float* logits;                          // [M, E] workspace
    int32_t* ids_ws;                        // [M*k] workspace copies of the routing
    float* wts_ws;
    int32_t* ids_out;                       // caller's top-k ids (int32) and weights (bf16)
    uint16_t* wts_out;
    int32_t* bar;                           // [2] grid barrier: arrivals, generation
    int32_t* fold_cnt;                      // [M][down row tiles] pair rows stored per
                                            // (token, 128-column slice of y)
    uint16_t* y;
    int clear_chunks;                       // chunk_done entries a call may use
  } rt;
};

// Fused layer: at most this many (token, slot) pairs, so the plan fits in shared
// memory next to the pipeline buffers.
constexpr int kTcFusedMaxPairs = 256;
// Plan kept in shared memory for the whole fused call: ids, weights, the
// permutation, each token's slots in ascending expert id, chunk descriptors (a
// chunk holds >= 1 pair, so <= P of them) and four words (chunk count, fold
// mask, barrier status).
constexpr size_t kTcPlanBytes = 4 * kTcFusedMaxPairs * 4 + kTcFusedMaxPairs * 16 + 16;
// Per-warp top-k scratch of the fused prologue: E (value, index) pairs, E
// logits, the tie path's working memory (16-byte multiple).
__host__ __device__ inline size_t tc_topk_scratch(int E) {
  return (static_cast<size_t>(E) * 12 + kTopkWarpScratch + 15) / 16 * 16;
}

// A bounded wait gave up: the error word gets kErrWaitTimeout and, under expert
// parallelism, the call is marked failed so its peers do not fold partial rows.
__device__ __forceinline__ void tc_record_timeout(const TcParams& p) {
  atomicOr(p.err, kErrWaitTimeout);
  if (p.ep_world) atomicExch(p.ep_ticket + 1, 1);
}

// The last CTA of this rank's expert kernel raises this rank's flag to the
// call's epoch in every rank's mailbox.  Ordering: each CTA's peer row stores
// reach its issuer through the epilogue's mbarrier arrive (release) and wait
// (acquire); a GPU-scope fence orders them before the CTA's ticket; the last
// CTA's ticket observes every other CTA's, and its system-scope fence, which is
// cumulative over all of them, orders every row before the flag's system-scope
// release -- one system fence per call, not one per CTA.  When any CTA of the
// call gave up on a wait it first raises this rank's failure word to the epoch,
// which the peers' combine turns into an error instead of a fold.
__device__ __forceinline__ void tc_ep_signal(const TcParams& p) {
  __threadfence();
  if (atomicAdd(p.ep_ticket, 1) != static_cast<int>(gridDim.x) - 1) return;
  *p.ep_ticket = 0;
  __threadfence();
  const bool failed = atomicExch(p.ep_ticket + 1, 0) != 0;
  // one system-scope fence, then relaxed system-scope stores: the fence makes
  // each store a release (a release store per flag would fence once per rank)
  __threadfence_system();
  if (failed)
    for (int r = 0; r < p.ep_world; ++r)
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;\n" ::"l"(p.ep_flags[r] + kEpFailWord + p.ep_rank),
                   "r"(p.ep_epoch)
                   : "memory");
  if (failed) __threadfence_system();   // the failure word lands before the flag
  for (int r = 0; r < p.ep_world; ++r)
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;\n" ::"l"(p.ep_flags[r] + p.ep_rank), "r"(p.ep_epoch)
                 : "memory");
}

// Shared memory: weight ring, two B buffers (kTcChunk term rows each), one
// B-scale gather buffer, the SwiGLU hand-off and the mbarriers.
struct TcSmem {
  size_t b, b_bytes, sfb, hs, bars, plan, total;
};
__host__ __device__ inline TcSmem tc_smem_layout(int kmax, size_t tile_full, bool fused) {
  TcSmem m{};
  m.b = kTcStages * tile_full;
  m.b_bytes = (kTcChunk * term_row_bytes(kmax) + 32 + 127) / 128 * 128;
  m.sfb = m.b + 2 * m.b_bytes;
  m.hs = m.sfb + static_cast<size_t>((kmax + 127) / 128) * 512;
  m.bars = m.hs + 2 * kTcChunk * 64 * 4;
  m.plan = m.bars + (2 * kTcStages + 2 * kTcAcc + 8) * 8 + 16;
  m.total = m.plan + (fused ? kTcPlanBytes : 0);
  return m;
}


// Kimi-K3 `situ` of one (gate, up) pair of bf16 Linear outputs, in fp32 as
// SituAndMul.forward computes it (vendor/kimi_k3_ref/modeling_kimi_linear.py:75-80):
// beta*tanh(g/beta) * sigmoid(g) * (lb*tanh(u/lb), or u when lb is 0), to bf16.
__device__ __forceinline__ float tc_situ(float g, float u, float beta, float lb) {
  const float sg = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-g)));
  const float a = __fmul_rn(__fmul_rn(beta, tanhf(__fdiv_rn(g, beta))), sg);
  const float uu = lb > 0.f ? __fmul_rn(lb, tanhf(__fdiv_rn(u, lb))) : u;
  return bf16r(__fmul_rn(a, uu));
}

// Down epilogue: weighted pair rows (flat pair order; situ layers: the bf16 w2
// outputs unweighted); the combine kernel folds each token's k rows afterwards.
__device__ __forceinline__ void tc_epilogue_down(const TcParams& p, const float (&val)[kTcChunk],
                                                 int nt, int pos0, int mt, int q, int lane,
                                                 float bias_v, const int32_t* perm,
                                                 const float* wts) {
  const int o = mt * 128 + 32 * q + lane;
  if (o >= p.dn.L.R) return;
  for (int i = 0; i < nt; ++i) {
    const int flat = perm[pos0 + i];
    float v = bf16r(val[i]);
    if (p.dn.bias) v = bf16r(__fadd_rn(v, bias_v));
    if (!p.situ) v = bf16r(__fmul_rn(v, wts[flat]));   // situ rows: the combine weighs them
    const uint16_t b = float_to_bf16_bits(v);
    const size_t at = static_cast<size_t>(flat) * p.hidden + o;
    if (p.ep_world == 0) {
      p.pair_out[at] = b;
    } else {
      for (int r = 0; r < p.ep_world; ++r) p.ep_rows[r][at] = b;   // NVLink stores to peers
    }
  }
}

// ---------------------------------------------------------------------------
// Fused verify layer: the prologue of tc_moe_kernel<true>
// ---------------------------------------------------------------------------
// A layer call at verify size is one launch.  Every CTA first takes units of
// routing work -- the e2m1 split of one token row, or one expert's logits for
// every token (router row held in registers, the same fp64 summation order as
// logit_warp, so the logits equal the route kernel's bit for bit) -- then the
// grid meets at one barrier (the grid is co-resident: a cooperative launch of
// one CTA per SM).  After it every CTA reads all logits from L2, selects each
// token's top-k (select_softmax_token: torch's order and bf16 softmax) and
// builds the plan in its own shared memory; CTA 0 also writes the routing to
// the workspace and the caller's outputs.  Identical inputs give identical
// plans in every CTA, so no second grid-wide step is needed.

// Sense-reversing grid barrier on two workspace words: the last CTA to arrive
// restores the arrival count to zero and advances the generation the others
// wait on (bounded, ~2 s).  One thread per CTA calls it.
__device__ __forceinline__ bool tc_grid_barrier(int32_t* bar, int G) {
  const int gen = ld_acquire_gpu(bar + 1);
  __threadfence();
  if (atomicAdd(bar, 1) == G - 1) {
    // nothing touches the count again in this launch: a plain store, then the
    // release of the generation (no round trip waited on)
    asm volatile("st.relaxed.gpu.global.b32 [%0], %1;\n" ::"l"(bar), "r"(0) : "memory");
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;\n" ::"l"(bar + 1), "r"(1) : "memory");
    return true;
  }
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (ld_acquire_gpu(bar + 1) != gen) return true;
    if (global_ns() - t0 > 2000000000ull) return false;
    __nanosleep(256);
  }
}

// Logits of expert e for every token: x . W_r[e] + b_r[e] rounded once to bf16
// (bf16 products exact in fp32, summed in fp64 in logit_warp's order).  Warp w
// takes tokens w, w + 8, ...; the router row stays in registers.
__device__ __forceinline__ void tc_route_logits(const TcParams::Route& r, int e, int H) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kV = kTcMaxK / 256;
  const uint16_t* w = r.wr + static_cast<size_t>(e) * H;
  uint4 wv[kV];
#pragma unroll
  for (int i = 0; i < kV; ++i) {
    const int k0 = lane * 8 + 256 * i;
    wv[i] = k0 < H ? ldg_nc_v4(w + k0) : make_uint4(0, 0, 0, 0);
  }
  const double b = r.br ? static_cast<double>(bf16_bits_to_float(r.br[e])) : 0.0;
  for (int m = warp; m < r.M; m += kTcThreads / 32) {
    const uint16_t* xr = r.x + static_cast<size_t>(m) * H;
    uint4 xv[kV];
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int k0 = lane * 8 + 256 * i;
      xv[i] = k0 < H ? *reinterpret_cast<const uint4*>(xr + k0) : make_uint4(0, 0, 0, 0);
    }
    double acc = 0.0;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      if (lane * 8 + 256 * i >= H) break;
      const uint32_t xs[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
      const uint32_t ws[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x0 = __uint_as_float(xs[j] << 16), x1 = __uint_as_float(xs[j] & 0xFFFF0000u);
        const float w0 = __uint_as_float(ws[j] << 16), w1 = __uint_as_float(ws[j] & 0xFFFF0000u);
        acc += static_cast<double>(__fmul_rn(x0, w0));
        acc += static_cast<double>(__fmul_rn(x1, w1));
      }
    }
    acc = warp_sum_f64(acc);
    if (lane == 0) r.logits[static_cast<size_t>(m) * r.E + e] = bf16r(__double2float_rn(acc + b));
  }
}

// The plan of route_plan_small (route.cu) built by the whole CTA in shared
// memory, one thread per (token, slot) pair p (P <= kTcThreads), over the pairs
// routed to this GPU's experts [e_begin, e_end): p's place in the stable
// permutation is (local pairs of lower experts) + (earlier pairs of its own
// expert); a pair whose rank inside its expert is a multiple of kTcChunk opens a
// chunk, numbered after the chunks of the lower experts.  Chunk descriptors
// carry the local expert index (the bank holds the local experts only).  Two
// passes over the P ids in shared memory, no serial scan over the experts.
// Returns the number of chunks; every thread of the CTA must call.
__device__ __forceinline__ int tc_fused_plan(const int32_t* ids_s, int P, int e_begin, int e_end,
                                             int32_t* perm_s, int32_t* rin_s, int4* cinfo_s) {
  const int tid = threadIdx.x;
  int e = 0, less = 0, rin = 0, cnt = 0;
  const bool local = tid < P && ids_s[tid] >= e_begin && ids_s[tid] < e_end;
  if (local) {
    e = ids_s[tid];
#pragma unroll 4
    for (int q = 0; q < P; ++q) {
      const int eq = ids_s[q];
      less += (eq < e) & (eq >= e_begin);
      rin += (eq == e) & (q < tid);
      cnt += eq == e;
    }
    perm_s[less + rin] = tid;
  }
  if (tid < P) rin_s[tid] = local ? rin : 1;   // non-local pairs open nothing
  const bool opens = local && rin % kTcChunk == 0;
  const int nch = __syncthreads_count(opens);
  if (opens) {
    int before = 0;
#pragma unroll 4
    for (int q = 0; q < P; ++q)
      before += (ids_s[q] < e) & (ids_s[q] >= e_begin) & (rin_s[q] % kTcChunk == 0);
    cinfo_s[before + rin / kTcChunk] = make_int4(e - e_begin, less + rin, min(kTcChunk, cnt - rin), 0);
  }
  return nch;
}

// Column o of y for token m: the bf16 fold of the token's k weighted pair rows
// in ascending expert id (combine_kernel's arithmetic); order_s holds each
// token's slots in that order.  Called once the last of the token's k pair rows
// of o's 128-column slice is stored.
__device__ __forceinline__ void tc_fold_token(const TcParams& p, int m, int o,
                                              const int32_t* order_s) {
  const int k = p.rt.k, H = p.hidden;
  uint16_t v[kMaxTopK];
#pragma unroll
  for (int s = 0; s < kMaxTopK; ++s)
    if (s < k) v[s] = __ldcg(p.pair_out + (static_cast<size_t>(m) * k + order_s[m * k + s]) * H + o);
  float a = 0.f;
#pragma unroll
  for (int s = 0; s < kMaxTopK; ++s)
    if (s < k) a = bf16r(__fadd_rn(a, bf16_bits_to_float(v[s])));
  p.rt.y[static_cast<size_t>(m) * H + o] = float_to_bf16_bits(a);
}

template <bool kFused>
__global__ void __launch_bounds__(kTcThreads, 1) tc_moe_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t tsm[];
  constexpr int S = kTcStages;
  const size_t tile_full = p.gu.L.tile_full;
  const TcSmem m = tc_smem_layout(p.kmax, tile_full, kFused);
  uint8_t* ring = tsm;
  uint8_t* bsm = tsm + m.b;            // buffer j at bsm + j * m.b_bytes
  uint8_t* sfbsm = tsm + m.sfb;
  float* hs = reinterpret_cast<float*>(tsm + m.hs);
  uint64_t* full = reinterpret_cast<uint64_t*>(tsm + m.bars);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + kTcAcc;
  uint64_t* b_full = acc_empty + kTcAcc;   // [2]
  uint64_t* b_empty = b_full + 2;          // [2]
  uint64_t* sfb_done = b_empty + 2;        // issuer 0 copied the gathered B scales to TMEM
  uint64_t* iss_done = sfb_done + 1;       // [2] every MMA of an issuer completed
  uint64_t* epi_done = iss_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Set-up before the routing plan is visible (overlaps the route kernel's tail).
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kTcAcc; ++b) {
      mbar_init(&acc_full[b], 2);
      mbar_init(&acc_empty[b], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&b_full[b], 1);
      mbar_init(&b_empty[b], 2);
      mbar_init(&iss_done[b], 1);
    }
    mbar_init(sfb_done, 1);
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
  pdl_wait();   // routing plan, x terms and cleared counters are visible (x alone when fused)
  // the plan: workspace arrays written by the route kernel, or (fused) this
  // CTA's own copy in shared memory
  const int4* cinfo = p.chunk_info;
  const int32_t* perm = p.perm;
  const float* wts = p.wts;
  const int32_t* plan_order = nullptr;
  int32_t* plan_words = nullptr;   // fused: [1] fold mask, [2] barrier passed
  long long nch;
  if constexpr (kFused) {
    const TcParams::Route& r = p.rt;
    const int H = p.hidden, P = r.M * r.k;
    uint8_t* pl = tsm + m.plan;
    int32_t* ids_s = reinterpret_cast<int32_t*>(pl);
    float* wts_s = reinterpret_cast<float*>(pl + kTcFusedMaxPairs * 4);
    int32_t* perm_s = reinterpret_cast<int32_t*>(pl + 2 * kTcFusedMaxPairs * 4);
    int32_t* order_s = reinterpret_cast<int32_t*>(pl + 3 * kTcFusedMaxPairs * 4);
    int4* cinfo_s = reinterpret_cast<int4*>(pl + 4 * kTcFusedMaxPairs * 4);
    plan_words = reinterpret_cast<int32_t*>(pl + 4 * kTcFusedMaxPairs * 4 + kTcFusedMaxPairs * 16);
    // units: token rows to e2m1 terms, then one expert's logits each
    for (int u = blockIdx.x; u < r.M + r.E; u += gridDim.x) {
      if (u < r.M)
        decompose_rows(r.x, H, H, u, 1, const_cast<uint8_t*>(p.gu.act_terms) + u * term_row_bytes(H),
                       const_cast<uint8_t*>(p.gu.act_sf) + u * term_sf_row_bytes(H));
      else
        tc_route_logits(r, u - r.M, H);
    }
    if (blockIdx.x == 0) {   // counters the call's items advance start at zero
      for (int i = threadIdx.x; i < r.clear_chunks; i += kTcThreads) p.chunk_done[i] = 0;
      for (int i = threadIdx.x; i < r.M * p.dn.L.MT; i += kTcThreads) r.fold_cnt[i] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) plan_words[2] = tc_grid_barrier(r.bar, gridDim.x);
    __syncthreads();
    if (!plan_words[2]) {   // the grid never met: nothing of this call is valid
      if (threadIdx.x == 0) {
        tc_record_timeout(p);
        if (p.ep_world) tc_ep_signal(p);   // peers see the failure word, not a silence
      }
      if (warp == 1) tc::tmem_dealloc(tbase, 512);
      return;
    }
    // every token's top-k from the logits in L2 (scratch: the weight ring; per
    // warp E (value, index) pairs, E logits and the tie path's scratch)
    uint8_t* wsc = tsm + static_cast<size_t>(warp) * tc_topk_scratch(r.E);
    KV* kv = reinterpret_cast<KV*>(wsc);
    float* lrow = reinterpret_cast<float*>(wsc + r.E * sizeof(KV));
    for (int mm = warp; mm < r.M; mm += kTcThreads / 32) {
      for (int j = lane; j < r.E; j += 32) lrow[j] = __ldcg(r.logits + static_cast<size_t>(mm) * r.E + j);
      __syncwarp();
      select_softmax_token(lrow, kv, mm, r.E, r.k, ids_s, wts_s, nullptr, nullptr,
                           wsc + r.E * (sizeof(KV) + 4));
      __syncwarp();
    }
    __syncthreads();
    const int n_plan = tc_fused_plan(
        ids_s, P, r.e_begin, r.e_end, perm_s,
        reinterpret_cast<int32_t*>(tsm + static_cast<size_t>(kTcThreads / 32) * tc_topk_scratch(r.E)),
        cinfo_s);
    if (threadIdx.x < P) {   // slot order of each token by expert id (ids of a token differ)
      const int tok = threadIdx.x / r.k, e = ids_s[threadIdx.x];
      int rank = 0;
      for (int s2 = 0; s2 < r.k; ++s2) rank += ids_s[tok * r.k + s2] < e;
      order_s[tok * r.k + rank] = threadIdx.x - tok * r.k;
    }
    if (blockIdx.x == 0) {
      for (int i = threadIdx.x; i < P; i += kTcThreads) {
        r.ids_ws[i] = ids_s[i];
        r.wts_ws[i] = wts_s[i];
        if (r.ids_out) r.ids_out[i] = ids_s[i];
        if (r.wts_out) r.wts_out[i] = float_to_bf16_bits(wts_s[i]);
      }
    }
    // the ring's generic-proxy scratch writes come before its bulk-copy writes,
    // and other CTAs' token terms (generic stores before the barrier) before the
    // bulk copies that read them
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    fence_proxy_async_global();
    __syncthreads();
    cinfo = cinfo_s;
    perm = perm_s;
    wts = wts_s;
    plan_order = order_s;
    nch = n_plan;
  } else {
    nch = *p.n_chunks;
  }
  pdl_launch_dependents();
  const int mtg = p.gu.L.MT, mtd = p.dn.L.MT;
  // Runs of kTcRun items dealt round-robin, gate/up then down (TcRunCursor);
  // runs of one when the gate/up items would not give every CTA a few runs.
  TcRunCursor cur;
  cur.start(blockIdx.x, gridDim.x, nch, mtg, mtd,
            nch * mtg >= 4LL * gridDim.x ? kTcRun : 1);
  if (!cur.valid()) {   // nothing for this CTA
    if (warp == 1) tc::tmem_dealloc(tbase, 512);
    if (threadIdx.x == 0 && p.ep_world) tc_ep_signal(p);
    return;
  }
  // token row of slot i of a gate/up chunk
  auto chunk_row = [&](int chunk, int pos0, int i) -> int {
    if constexpr (kFused) return perm[pos0 + i] / p.rt.k;
    else return __ldg(&p.chunk_rows[chunk * kChunkRowStride + i]);
  };

  if (warp == 0) {
    // ---------------- producer: weight tiles into the ring ----------------
    // Weight tiles are read once: their copies carry an evict-first L2 policy,
    // so they recycle each other's L2 lines instead of evicting (and writing
    // back) whatever else the L2 holds.
    bool ok = true;
    uint32_t nuse[2] = {0u, 0u};   // tiles put into each issuer's half of the ring
    const uint64_t stream_policy = l2_policy_evict_first();
    for (; cur.valid(); cur.next()) {
      if (lane == 0 && ok) {
        const TcItem t = cur.t;
        const TcProj& P = t.gu ? p.gu : p.dn;
        const int e = cinfo[t.chunk].x;
        const int rows_t = tc_rows(P.L, t.mt);
        const uint8_t* src =
            P.bank + static_cast<size_t>(e) * P.L.expert_bytes + static_cast<size_t>(t.mt) * P.L.mtile_full;
        for (int kt = 0; kt < P.L.NKT; ++kt) {
          const uint32_t par = kt & 1, k = nuse[par]++;
          const uint32_t s = par + 2 * (k % kTcHalfStages), use = k / kTcHalfStages;
          if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1)) {
            ok = false;
            break;
          }
          const uint32_t bytes = static_cast<uint32_t>(tc_tile_bytes(rows_t, tc_kt_len(P.L, kt)));
          mbar_expect_tx(&full[s], bytes);
          bulk_g2s_hint(ring + s * tile_full, src, bytes, &full[s], stream_policy);
          src += bytes;
        }
      }
      __syncwarp();
    }
    if (lane == 0) {
      for (uint32_t par = 0; par < 2; ++par)   // copies in flight land before exit
        for (uint32_t j = 0; j < kTcHalfStages && j < nuse[par]; ++j) {
          const uint32_t last = ((nuse[par] - 1 - j) / kTcHalfStages) * kTcHalfStages + j;
          if (!mbar_wait_bounded(&full[par + 2 * j], (last / kTcHalfStages) & 1)) ok = false;
        }
      if (!ok) tc_record_timeout(p);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 7) {
    // ---------------- MMA issuers ----------------
    // Two warps issue: one the even K-tiles of every item, the other the odd
    // ones, each into its own half of the item's accumulator (the epilogue adds
    // the halves).  The whole warp walks the items and waits, so descriptors and
    // loop state stay warp-uniform; one elected lane issues the tcgen05 ops.
    // Descriptors are built once and advanced by adding the 16-byte-unit offset
    // to their address field (smem addresses < 256 KB never carry out of it).
    const int odd = warp == 7;
    bool ok = true;
    uint32_t nuse = 0, item_no = 0, bc = 0;   // nuse: tiles of this issuer so far
    TcItem prev{-1, -1, -1};
    const uint32_t idesc[2] = {tc::idesc_mxf4(kTcN, 0, 0), tc::idesc_mxf4(kTcN, 2, 2)};
    const uint64_t cp_ring = tc::smem_desc_kmajor(ring, 0, 128);
    // B scales: token-major rows (srb bytes each), one 8-row core matrix per token
    const uint64_t cp_sfb_gu = tc::smem_desc_kmajor(sfbsm, 0, static_cast<uint32_t>(term_sf_row_bytes(p.gu.L.K)));
    const uint64_t cp_sfb_dn = tc::smem_desc_kmajor(sfbsm, 0, static_cast<uint32_t>(term_sf_row_bytes(p.dn.L.K)));
    const uint64_t b_gu = tc::smem_desc_kmajor(bsm, kTcBlockBytes, term_row_bytes(p.gu.L.K));
    const uint64_t b_dn = tc::smem_desc_kmajor(bsm, kTcBlockBytes, term_row_bytes(p.dn.L.K));
    const uint32_t b_step = static_cast<uint32_t>(m.b_bytes >> 4);
    const int ngk = (p.kmax + 127) / 128;
    uint32_t sfb_col = 0;
    uint64_t b_base = 0;
    for (; ok && cur.valid(); cur.next(), ++item_no) {
      const TcItem t = cur.t;
      const TcProj& P = t.gu ? p.gu : p.dn;
      const int rows_t = tc_rows(P.L, t.mt);
      if (!tc_same_b(t, prev)) {
        // B buffer bc%2 was filled by the stager (after the MMAs of chunk bc-2
        // completed); issuer 0 copies its scales to TMEM for both issuers
        const uint32_t j = bc & 1;
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&b_full[j], (bc >> 1) & 1));
        tc::fence_after_sync();
        sfb_col = tbase + kTcSfbCol + j * 4 * ngk;
        if (!odd) {
          const int ng = (P.L.K + 127) / 128;
          if (elect_one()) {
            const uint64_t cp_sfb = t.gu ? cp_sfb_gu : cp_sfb_dn;
            for (int g = 0; g < ng; ++g)
              tc::copy_sf_chunk_desc(sfb_col + 4 * g, cp_sfb + (kTermSfGroupBytes >> 4) * g);
            tc::commit_to(sfb_done);
          }
          __syncwarp();
        } else if (ok) {
          ok = __all_sync(0xffffffffu, mbar_wait_bounded(sfb_done, bc & 1));
        }
        b_base = (t.gu ? b_gu : b_dn) + j * b_step;
        ++bc;
        prev = t;
      }
      const uint32_t buf = item_no % kTcAcc, use = item_no / kTcAcc;
      if (ok && use > 0) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&acc_empty[buf], (use - 1) & 1));
      if (!ok) break;
      tc::fence_after_sync();
      const uint32_t d_tmem = tbase + buf * kTcAccCols + odd * kTcN;
      const uint64_t a_base = tc::smem_desc_kmajor(ring, rows_t * 16, 128);
      const uint32_t a_step = static_cast<uint32_t>(rows_t) * 2;   // two 16-byte K chunks
      for (int kt = 0; kt < P.L.NKT; ++kt) {
        if ((kt & 1) != odd) continue;
        const uint32_t k = nuse++;
        const uint32_t s = odd + 2 * (k % kTcHalfStages);
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (k / kTcHalfStages) & 1));
        if (!ok) break;
        tc::fence_after_sync();
        const int kt_len = tc_kt_len(P.L, kt);
        const uint32_t st16 = static_cast<uint32_t>((s * tile_full) >> 4);
        const uint64_t cp_s = cp_ring + st16 + static_cast<uint32_t>(rows_t) * (kt_len / 32);
        const uint32_t sfa_col = tbase + kTcSfaCol + 16 * s;
        const int nsf = (kt_len + 127) / 128, nmma = kt_len / 64;
        const uint64_t a_s = a_base + st16;
        const uint64_t b_s = b_base + static_cast<uint32_t>(kt * (kKT / 32) * kTcBlockBytes / 16);
        const uint32_t sfb_s = sfb_col + 4 * (kKT / 128) * kt;
        if (elect_one()) {
#pragma unroll
          for (int g = 0; g < kKT / 128; ++g)
            if (g < nsf) tc::copy_sf_chunk_desc(sfa_col + 4 * g, cp_s + 32 * g);
#pragma unroll
          for (int i = 0; i < kKT / 64; ++i) {
            if (i < nmma) {
              const uint32_t hi = static_cast<uint32_t>(i & 1) << 31;   // scale byte pair 2-3
              tc::mma_mxf4(d_tmem, a_s + static_cast<uint32_t>(i) * a_step,
                           b_s + static_cast<uint32_t>(i * 2 * kTcBlockBytes / 16), idesc[i & 1],
                           (sfa_col + 4 * (i >> 1)) | hi, (sfb_s + 4 * (i >> 1)) | hi,
                           kt > 1 || i > 0);
            }
          }
          tc::commit_to(&empty[s]);
        }
        __syncwarp();
      }
      if (ok && elect_one()) {
        tc::commit_to(&acc_full[buf]);
        // the chunk's last item: its B buffer is free once these MMAs complete
        if (!cur.next_same_b()) tc::commit_to(&b_empty[(bc - 1) & 1]);
      }
      __syncwarp();
    }
    if (lane == 0) {
      tc::commit_to(&iss_done[odd]);   // all of this issuer's MMAs completed
      if (!mbar_wait_bounded(&iss_done[odd], 0)) ok = false;
      // tensor memory goes back only after the epilogue read its last accumulator
      if (!odd && !mbar_wait_bounded(epi_done, 0)) ok = false;
      if (!ok) tc_record_timeout(p);
      if (!odd && p.ep_world) tc_ep_signal(p);   // all of this CTA's rows are stored
    }
    __syncwarp();
    if (!odd) {
      tc::fence_after_sync();
      tc::tmem_dealloc(tbase, 512);
    }
  } else if (warp < 6) {
    // ---------------- epilogue (TMEM lane quadrant = warp % 4) ----------------
    const int q = warp & 3;
    const int et = threadIdx.x - 64;   // 0..127
    bool ok = true;
    uint32_t item_no = 0;
    int chunk_items = 0;
    int4 ci = cinfo[cur.t.chunk];   // chunk of the current item
    for (; cur.valid(); cur.next(), ++item_no) {
      const TcItem t = cur.t;
      const TcProj& P = t.gu ? p.gu : p.dn;
      const int row = t.mt * 128 + 32 * q + lane;   // weight row of this lane
      const int e = ci.x, pos0 = ci.y, nt = ci.z;
      const float bias_v =
          (P.bias && row < P.L.R) ? __ldg(P.bias + static_cast<size_t>(e) * P.L.R + row) : 0.f;
      // the next item's chunk, fetched while this one is processed
      const bool same_next = cur.next_same_b();
      int4 ci_next = ci;
      if (!same_next) {
        TcRunCursor nx = cur;
        nx.next();
        if (nx.valid()) ci_next = cinfo[nx.t.chunk];
      }
      ++chunk_items;
      const uint32_t buf = item_no % kTcAcc, use = item_no / kTcAcc;
      if (ok && !mbar_wait_bounded(&acc_full[buf], use & 1)) {
        ok = false;
        tc_record_timeout(p);
      }
      tc::fence_after_sync();
      float val[kTcChunk];
      {
        uint32_t r[kTcChunk][8];
        uint32_t r2[kTcChunk][8];   // odd K-tile half (absent when the K extent is one tile)
        const bool two = P.L.NKT > 1;
        const uint32_t ta = tbase + buf * kTcAccCols + ((32u * q) << 16);
#pragma unroll
        for (int i = 0; i < kTcChunk; ++i) {
          if (i < nt) tc::tmem_ld8(ta + i * kTermSlots, r[i]);
          if (i < nt && two) tc::tmem_ld8(ta + kTcN + i * kTermSlots, r2[i]);
        }
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < kTcChunk; ++i) {
          float sum = 0.f;
          if (i < nt) {
#pragma unroll
            for (int tt = 0; tt < kTerms; ++tt) {
              sum += __uint_as_float(r[i][tt]);
              if (two) sum += __uint_as_float(r2[i][tt]);
            }
          }
          val[i] = ok ? sum : 0.f;
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (t.gu) {
        // tile row m: even = gate_j, odd = up_j, j = (mt*128 + m) / 2
        float* hb = hs + (item_no & 1) * kTcChunk * 64;   // two hand-off buffers
        const bool even = (lane & 1) == 0;
        const int jl = (32 * q + lane) >> 1;
        const float bias_up = __shfl_xor_sync(0xffffffffu, bias_v, 1);
#pragma unroll
        for (int i = 0; i < kTcChunk; ++i) {
          const float upv = __shfl_xor_sync(0xffffffffu, val[i], 1);
          if (even) {
            float h = 0.f;
            if (i < nt && row < P.L.R && p.situ) {
              h = tc_situ(bf16r(val[i]), bf16r(upv), p.alpha, p.limit);
            } else if (i < nt && row < P.L.R) {
              float gate = bf16r(val[i]);
              float up = bf16r(upv);
              if (P.bias) {
                gate = bf16r(__fadd_rn(gate, bias_v));
                up = bf16r(__fadd_rn(up, bias_up));
              }
              gate = gate > p.limit ? p.limit : gate;
              up = up > p.limit ? p.limit : (up < -p.limit ? -p.limit : up);
              const float ta = bf16r(__fmul_rn(gate, p.alpha));
              const float sg = bf16r(__frcp_rn(__fadd_rn(1.f, expf(-ta))));
              const float glu = bf16r(__fmul_rn(gate, sg));
              const float up1 = bf16r(__fadd_rn(up, 1.f));
              h = bf16r(__fmul_rn(up1, glu));
            }
            hb[i * 64 + jl] = h;
          }
        }
        named_barrier_sync(1, 128);
        // the tile's 64 SwiGLU outputs per token as e2m1 terms for the down
        // projection (2 blocks of 32, four lanes per (token, block)): the first
        // epilogue warp covers all kTcChunk tokens while the others move on
        if (et < 32) {
          const int unit = et >> 2, quarter = et & 3;
          const int tok = unit >> 1, b = unit & 1;
          const int blk = t.mt * 2 + b;
          const bool live = tok < nt && blk * 32 < p.inter;
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = live ? hb[tok * 64 + b * 32 + quarter * 8 + i] : 0.f;
          const int pos = pos0 + (live ? tok : 0);
          decompose_block(v, quarter,
                          p.h_terms + static_cast<size_t>(pos) * term_row_bytes(p.inter) +
                              static_cast<size_t>(blk) * kTcBlockBytes,
                          p.h_sf + static_cast<size_t>(pos) * term_sf_row_bytes(p.inter) +
                              term_sf_offset(blk, 0),
                          live);
          if (!same_next) {
            // this CTA's last tile of the chunk: release its rows to the down tiles
            __threadfence();
            __syncwarp();
            if (lane == 0) atomicAdd(&p.chunk_done[t.chunk], chunk_items);
          }
        }
      } else {
        tc_epilogue_down(p, val, ok ? nt : 0, pos0, t.mt, q, lane, bias_v, perm, wts);
        if (kFused && p.ep_world == 0) {
          // a token whose k pair rows of this 128-column slice are now all stored
          // is folded into y here (the item's tokens are distinct)
          __threadfence();
          named_barrier_sync(1, 128);
          if (et < kTcChunk) {
            bool last = false;
            if (et < nt) {
              const int m = perm[pos0 + et] / p.rt.k;
              last = atomicAdd(&p.rt.fold_cnt[m * mtd + t.mt], 1) == p.rt.k - 1;
            }
            const uint32_t mask = __ballot_sync(0xfu, last);
            if (et == 0) plan_words[1] = static_cast<int>(mask);
          }
          named_barrier_sync(1, 128);
          const uint32_t mask = static_cast<uint32_t>(plan_words[1]);
          if (mask) {
            __threadfence();
            const int o = t.mt * 128 + 32 * q + lane;
            for (int i = 0; i < kTcChunk; ++i)
              if (((mask >> i) & 1u) && o < p.hidden) tc_fold_token(p, perm[pos0 + i] / p.rt.k, o, plan_order);
          }
        }
      }
      if (!same_next) chunk_items = 0;
      ci = ci_next;
    }
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(epi_done);
  } else if (warp == 6) {
    // ---------------- B stager: activation terms of each chunk ----------------
    // Token i's whole term row lands at B + i*trb by one bulk copy; the MMA
    // reads it as core matrices of 8 term slots (slots past kTerms overlap the
    // next block and feed columns nobody reads).  Token i's scale row lands at
    // i * srb by one more bulk copy: the 8 term slots of one 128-K group are one
    // 8-row core matrix of tcgen05.cp's 32x128b chunk, and the copy's descriptor
    // strides srb from token to token (row n = token*8 + slot).  Two B buffers
    // let the next chunk's terms arrive while this one computes.
    bool ok = true;
    uint32_t bc = 0;
    TcItem prev{-1, -1, -1};
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      if (tc_same_b(t, prev)) continue;
      prev = t;
      const TcProj& P = t.gu ? p.gu : p.dn;
      const int4 ci = cinfo[t.chunk];
      const int nt = ci.z;
      const uint32_t j = bc & 1;
      if (lane == 0) {
        // buffer j held chunk bc-2; the gather buffer held chunk bc-1's scales
        if (bc >= 2 && !mbar_wait_bounded(&b_empty[j], ((bc >> 1) - 1) & 1)) ok = false;
        if (ok && bc >= 1 && !mbar_wait_bounded(sfb_done, (bc - 1) & 1)) ok = false;
        if (ok && !t.gu) {
          if (!wait_counter_geq(&p.chunk_done[t.chunk], mtg)) ok = false;
          fence_proxy_async_global();
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
      if (!ok) break;
      const size_t trb = term_row_bytes(P.L.K), srb = term_sf_row_bytes(P.L.K);
      uint8_t* bj = bsm + j * m.b_bytes;
      if (lane == 0) mbar_expect_tx_only(&b_full[j], static_cast<uint32_t>(nt * (trb + srb)));
      __syncwarp();
      if (lane < nt) {
        const int row = t.gu ? chunk_row(t.chunk, ci.y, lane) : ci.y + lane;
        bulk_g2s(bj + lane * trb, P.act_terms + static_cast<size_t>(row) * trb,
                 static_cast<uint32_t>(trb), &b_full[j]);
      }
      // scales: token i's whole scale row at i * srb; the tcgen05.cp descriptor
      // of group g strides srb between the tokens' 8-row core matrices
      if (lane >= 16 && lane - 16 < nt) {
        const int i = lane - 16;
        const int row = t.gu ? chunk_row(t.chunk, ci.y, i) : ci.y + i;
        bulk_g2s(sfbsm + static_cast<size_t>(i) * srb, P.act_sf + static_cast<size_t>(row) * srb,
                 static_cast<uint32_t>(srb), &b_full[j]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_full[j]);
      ++bc;
    }
    if (lane == 0) {
      // copies in flight land before the CTA exits
      for (uint32_t c = (bc >= 2 ? bc - 2 : 0); ok && c < bc; ++c)
        if (!mbar_wait_bounded(&b_full[c & 1], (c >> 1) & 1)) ok = false;
      if (!ok) tc_record_timeout(p);
    }
    __syncwarp();
  }
}

// Token rows -> e2m1 terms, for entry points whose call did not route (the
// route kernels split x themselves).  One CTA per token.
__global__ void __launch_bounds__(128) tc_split_rows_kernel(const uint16_t* __restrict__ x, int H,
                                                            uint8_t* __restrict__ terms,
                                                            uint8_t* __restrict__ sf) {
  pdl_wait();
  pdl_launch_dependents();
  const int m = blockIdx.x;
  decompose_rows(x, H, H, m, 1, terms + static_cast<size_t>(m) * term_row_bytes(H),
                 sf + static_cast<size_t>(m) * term_sf_row_bytes(H));
}

template <typename Kern, typename... Args>
static cudaError_t tc_launch_pdl(Kern kernel, int grid, int block, size_t smem, cudaStream_t s,
                                 Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// The persistent expert kernel: one CTA per SM whose items wait on other CTAs
// (a chunk's down tiles on its gate/up tiles; the fused layer's grid barrier),
// so the grid must be co-resident.  A cooperative launch guarantees that or
// fails with an error instead of leaving CTAs waiting for SMs held by others.
static cudaError_t tc_launch_persistent(const TcParams& prm, bool fused, int grid, size_t smem,
                                        cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return fused ? cudaLaunchKernelEx(&cfg, tc_moe_kernel<true>, prm)
               : cudaLaunchKernelEx(&cfg, tc_moe_kernel<false>, prm);
}

int launch_tc_experts(const flyai_moe_desc& d, int M, const void* x, bool x_split,
                      const flyai_moe_weights& w, uint16_t* pair_out, bool zero_pairs,
                      const Workspace& ws, cudaStream_t stream, void* y_fold, bool* folded,
                      const flyai_moe_ep_peers* ep) {
  if (folded) *folded = false;
  const int El = d.expert_end - d.expert_begin;
  const int P = M * d.top_k;
  if (zero_pairs && P > 0 &&
      cudaMemsetAsync(pair_out, 0, static_cast<size_t>(P) * d.hidden * 2, stream) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (P == 0 || El == 0) return FLYAI_OK;
  if (M >= kTcPrefillMinTokens) {   // the plan was built with prefill-size chunks
    if (!x_split &&
        cudaMemsetAsync(ws.chunk_done, 0, static_cast<size_t>(ws.max_chunks) * 4, stream) != cudaSuccess)
      return FLYAI_ERR_CUDA;
    return launch_tc_prefill(d, M, x, w, pair_out, ws, stream);
  }
  if (!x_split) {
    // a standalone experts call: split x here and restart the chunk counters
    if (cudaMemsetAsync(ws.chunk_done, 0, static_cast<size_t>(ws.max_chunks) * 4, stream) !=
        cudaSuccess)
      return FLYAI_ERR_CUDA;
    if (tc_launch_pdl(tc_split_rows_kernel, M, 128, 0, stream, static_cast<const uint16_t*>(x),
                      d.hidden, ws.x_terms, ws.x_sf) != cudaSuccess)
      return FLYAI_ERR_CUDA;
    note_launch();
  }
  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);

  TcParams prm{};
  prm.gu = TcProj{static_cast<const uint8_t*>(w.w13), tc_layout(d, FLYAI_PROJ_W13),
                  static_cast<const float*>(w.w13_bias), ws.x_terms, ws.x_sf};
  prm.dn = TcProj{static_cast<const uint8_t*>(w.w2), tc_layout(d, FLYAI_PROJ_W2),
                  static_cast<const float*>(w.w2_bias), ws.h_terms, ws.h_sf};
  prm.n_chunks = ws.n_chunks;
  prm.chunk_info = ws.chunk_info;
  prm.chunk_rows = ws.chunk_rows;
  prm.chunk_done = ws.chunk_done;
  prm.perm = ws.perm;
  prm.wts = ws.wts;
  prm.h_terms = ws.h_terms;
  prm.h_sf = ws.h_sf;
  prm.pair_out = pair_out;
  prm.hidden = d.hidden;
  prm.inter = d.inter;
  prm.kmax = d.hidden > d.inter ? d.hidden : d.inter;
  prm.limit = d.swiglu_limit;
  prm.alpha = d.swiglu_alpha;
  prm.situ = d.activation == FLYAI_ACT_SITU;
  prm.err = ws.err;
  if (ep) {
    const size_t rows_bytes = static_cast<size_t>(d.max_tokens) * d.top_k * d.hidden * 2;
    prm.ep_world = ep->world;
    prm.ep_rank = ep->rank;
    prm.ep_epoch = ep->epoch;
    for (int r = 0; r < ep->world; ++r) {
      uint8_t* mb = static_cast<uint8_t*>(ep->mailbox[r]);
      prm.ep_flags[r] = reinterpret_cast<uint32_t*>(mb);
      prm.ep_rows[r] = reinterpret_cast<uint16_t*>(mb + kEpFlagBytes + (ep->epoch & 1) * rows_bytes);
    }
    prm.ep_ticket = ws.route_ticket + kTicketEp;
  }

  const size_t smem = tc_smem_layout(prm.kmax, prm.gu.L.tile_full, false).total;
  if (smem > static_cast<size_t>(max_smem) || prm.kmax > kTcMaxK) return FLYAI_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(tc_moe_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (tc_launch_persistent(prm, false, sms, smem, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  note_launch();
  (void)y_fold;   // the caller folds pair rows into y with launch_combine
  return FLYAI_OK;
}

bool tc_fused_supported(const flyai_moe_desc& d, int M, bool ep) {
  return d.gating == FLYAI_GATE_SOFTMAX_TOPK && M >= 1 && M < kTcPrefillMinTokens && M * d.top_k <= kTcFusedMaxPairs &&
         (ep || (d.expert_begin == 0 && d.expert_end == d.num_experts));
}

int launch_tc_forward(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                      void* y, int32_t* ids_out, void* wts_out, const Workspace& ws,
                      cudaStream_t stream, const flyai_moe_ep_peers* ep) {
  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  TcParams prm{};
  prm.gu = TcProj{static_cast<const uint8_t*>(w.w13), tc_layout(d, FLYAI_PROJ_W13),
                  static_cast<const float*>(w.w13_bias), ws.x_terms, ws.x_sf};
  prm.dn = TcProj{static_cast<const uint8_t*>(w.w2), tc_layout(d, FLYAI_PROJ_W2),
                  static_cast<const float*>(w.w2_bias), ws.h_terms, ws.h_sf};
  prm.chunk_done = ws.chunk_done;
  prm.h_terms = ws.h_terms;
  prm.h_sf = ws.h_sf;
  prm.pair_out = ws.pair_out;
  prm.hidden = d.hidden;
  prm.inter = d.inter;
  prm.kmax = d.hidden > d.inter ? d.hidden : d.inter;
  prm.limit = d.swiglu_limit;
  prm.alpha = d.swiglu_alpha;
  prm.situ = d.activation == FLYAI_ACT_SITU;
  prm.err = ws.err;
  TcParams::Route& r = prm.rt;
  r.x = static_cast<const uint16_t*>(x);
  r.wr = static_cast<const uint16_t*>(w.router_w);
  r.br = static_cast<const uint16_t*>(w.router_b);
  r.M = M;
  r.E = d.num_experts;
  r.k = d.top_k;
  r.e_begin = d.expert_begin;
  r.e_end = d.expert_end;
  r.logits = ws.logits;
  r.ids_ws = ws.ids;
  r.wts_ws = ws.wts;
  r.ids_out = ids_out;
  r.wts_out = static_cast<uint16_t*>(wts_out);
  r.bar = ws.route_ticket + kTicketGridBarrier;
  r.fold_cnt = ws.fold_ticket;
  r.y = static_cast<uint16_t*>(y);
  r.clear_chunks = M * d.top_k < ws.max_chunks ? M * d.top_k : ws.max_chunks;
  if (ep) {   // pair rows into every rank's mailbox, then this rank's flag (tc_ep_signal)
    const size_t rows_bytes = static_cast<size_t>(d.max_tokens) * d.top_k * d.hidden * 2;
    prm.ep_world = ep->world;
    prm.ep_rank = ep->rank;
    prm.ep_epoch = ep->epoch;
    for (int i = 0; i < ep->world; ++i) {
      uint8_t* mb = static_cast<uint8_t*>(ep->mailbox[i]);
      prm.ep_flags[i] = reinterpret_cast<uint32_t*>(mb);
      prm.ep_rows[i] = reinterpret_cast<uint16_t*>(mb + kEpFlagBytes + (ep->epoch & 1) * rows_bytes);
    }
    prm.ep_ticket = ws.route_ticket + kTicketEp;
  }

  const size_t smem = tc_smem_layout(prm.kmax, prm.gu.L.tile_full, true).total;
  // prologue scratch in the weight ring: per warp E (value, index) pairs and E
  // logits, then the plan's counters
  const size_t scratch = static_cast<size_t>(kTcThreads / 32) * tc_topk_scratch(d.num_experts) +
                         (static_cast<size_t>(M) * d.top_k + 3 * d.num_experts + 2) * 4;
  if (smem > static_cast<size_t>(max_smem) || prm.kmax > kTcMaxK ||
      scratch > kTcStages * prm.gu.L.tile_full)
    return FLYAI_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(tc_moe_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (tc_launch_persistent(prm, true, sms, smem, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  note_launch();
  return FLYAI_OK;
}

}  // namespace flyai
