// Router kernels: exact bf16 logits, torch-identical top-k, gating weights,
// expert histogram and the stable token->expert permutation.
//
// Reference: transformers/models/gpt_oss/modeling_gpt_oss.py:117-131
// (GptOssTopKRouter.forward: F.linear in bf16, torch.topk, softmax over the k
// selected logits in bf16) and the gather order of the reference's GPU routing,
// transformers/integrations/mxfp4.py:473 (stable argsort of the flat expert ids).
#include "common.cuh"
#include "route.cuh"
#include "terms.cuh"
#include "route_dev.cuh"
#include "fp8_moe.cuh"

namespace flyai {

// 1) logits.  Verify sizes: logit_warp (route_dev.cuh) inside route_fused_kernel
// and the fused expert kernel.  Prefill sizes: nvp_logits_kernel's fp64 partial
// sums over K slices (a register-tiled DFMA product; bf16 products are exact in
// fp64), added here in slice order with the bias and rounded once to fp32 and
// once to bf16 -- the value logit_warp computes, to fp64 rounding of the sum.
__global__ void __launch_bounds__(256) route_logits_sum_kernel(const double* __restrict__ part,
                                                               const uint16_t* __restrict__ br, int M,
                                                               int E, float* __restrict__ logits,
                                                               uint16_t* __restrict__ logits_out) {
  const size_t n = static_cast<size_t>(M) * E;
  for (size_t u = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; u < n;
       u += static_cast<size_t>(gridDim.x) * blockDim.x) {
    double a = part[u];
#pragma unroll
    for (int s = 1; s < kNpLogitSlices; ++s) a += part[s * n + u];
    if (br) a += static_cast<double>(bf16_bits_to_float(br[u % E]));
    const float v = bf16r(__double2float_rn(a));
    logits[u] = v;
    if (logits_out) logits_out[u] = float_to_bf16_bits(v);
  }
}

// 2) top-k and gating weights: select_softmax_token (route_dev.cuh).
__global__ void __launch_bounds__(256) route_select_softmax_kernel(
    const float* __restrict__ logits, int M, int E, int k, int32_t* __restrict__ ids,
    float* __restrict__ wts, int32_t* __restrict__ ids_out, uint16_t* __restrict__ wts_out) {
  extern __shared__ KV route_smem[];
  const int warp = threadIdx.x >> 5;
  const int m = blockIdx.x * 8 + warp;
  if (m >= M) return;
  // per warp: E (value, index) pairs, then the tie path's scratch
  uint8_t* wsm = reinterpret_cast<uint8_t*>(route_smem) + warp * (E * sizeof(KV) + kTopkWarpScratch);
  select_softmax_token(logits + static_cast<size_t>(m) * E, reinterpret_cast<KV*>(wsm), m, E, k, ids,
                       wts, ids_out, wts_out, wsm + E * sizeof(KV));
}

// ---------------------------------------------------------------------------
// 3) histogram over this shard's experts, exclusive offsets, list of non-empty
// experts, and the stable permutation (flat pair index ascending within an
// expert).  One CTA; P = M*k pairs.
// ---------------------------------------------------------------------------
// Shared-memory plan: ids are staged once; per-warp histograms over contiguous
// pair ranges give each warp the base position of every expert, so the stable
// permutation (ascending flat index inside an expert) is written with one
// __match_any_sync rank per 32 pairs; a warp scan builds offsets, the active
// list and the chunk table.  No thread re-reads global memory it just wrote.
__host__ __device__ inline int plan_hist_warps(int nwarps, int e_count) {
  const int cap = e_count > 0 ? (32768 / e_count) : nwarps;
  const int w = nwarps < cap ? nwarps : cap;
  return w < 1 ? 1 : w;
}
__host__ __device__ inline size_t plan_smem_bytes(int P, int e_count, int nwarps) {
  const int wp = plan_hist_warps(nwarps, e_count);
  return (static_cast<size_t>(P) + 5ull * e_count + 8 + static_cast<size_t>(wp) * e_count) * 4;
}

__device__ void route_plan_block(const int32_t* __restrict__ ids, int P, int e_begin, int e_count,
                                 int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                 int32_t* __restrict__ active, int32_t* __restrict__ n_active,
                                 int32_t* __restrict__ perm, int32_t* __restrict__ n_chunks,
                                 int32_t* __restrict__ chunk_slot, int32_t* __restrict__ chunk_c0,
                                 int max_chunks, int32_t* plan_smem, int k, int4* chunk_info,
                                 int32_t* chunk_rows, int32_t* chunk_done) {
  // chunk size of the tcgen05 kernels (by batch size)
  const int ct = tc_chunk_tokens(P / k);
  const int tid = threadIdx.x, nth = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31, nwarps = nth >> 5;
  const int El = e_count;
  const int wp = plan_hist_warps(nwarps, El);
  int32_t* ids_s = plan_smem;            // [P] local expert or -1
  int32_t* cnt = ids_s + P;              // [El]
  int32_t* off = cnt + El;               // [El + 1]
  int32_t* act = off + El + 1;           // [El]
  int32_t* cbase = act + El;             // [El] first chunk of each active slot
  int32_t* tot = cbase + El;             // [4]  n_active, n_chunks
  int32_t* hist = tot + 7;               // [wp][El] per-warp counts, then bases
  for (int p = tid; p < P; p += nth) {
    const int v = ids[p] - e_begin;
    ids_s[p] = (v >= 0 && v < El) ? v : -1;
  }
  for (int i = tid; i < wp * El; i += nth) hist[i] = 0;
  __syncthreads();
  if (warp < wp) {
    const int p0 = static_cast<int>(static_cast<long long>(P) * warp / wp);
    const int p1 = static_cast<int>(static_cast<long long>(P) * (warp + 1) / wp);
    for (int p = p0 + lane; p < p1; p += 32) {
      const int v = ids_s[p];
      if (v >= 0) atomicAdd(&hist[warp * El + v], 1);
    }
  }
  __syncthreads();
  for (int e = tid; e < El; e += nth) {   // per-warp bases (exclusive over warps) and totals
    int run = 0;
    for (int w = 0; w < wp; ++w) {
      const int t = hist[w * El + e];
      hist[w * El + e] = run;
      run += t;
    }
    cnt[e] = run;
  }
  __syncthreads();
  if (warp == 0) {   // exclusive scans over experts: tokens, active slots, chunks
    const int per = (El + 31) / 32;
    const int e0 = min(El, lane * per), e1 = min(El, e0 + per);
    int s_tok = 0, s_act = 0, s_ch = 0;
    for (int e = e0; e < e1; ++e) {
      s_tok += cnt[e];
      s_act += cnt[e] > 0;
      s_ch += (cnt[e] + ct - 1) / ct;
    }
    int x_tok = s_tok, x_act = s_act, x_ch = s_ch;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, x_tok, o);
      const int b = __shfl_up_sync(0xffffffffu, x_act, o);
      const int c = __shfl_up_sync(0xffffffffu, x_ch, o);
      if (lane >= o) {
        x_tok += a;
        x_act += b;
        x_ch += c;
      }
    }
    int r_tok = x_tok - s_tok, r_act = x_act - s_act, r_ch = x_ch - s_ch;
    for (int e = e0; e < e1; ++e) {
      off[e] = r_tok;
      r_tok += cnt[e];
      if (cnt[e] > 0) {
        act[r_act] = e;
        cbase[r_act] = r_ch;
        ++r_act;
        r_ch += (cnt[e] + ct - 1) / ct;
      }
    }
    if (lane == 31) {
      off[El] = x_tok;
      tot[0] = x_act;
      tot[1] = min(x_ch, max_chunks);
    }
  }
  __syncthreads();
  const int na = tot[0];
  for (int e = tid; e < El; e += nth) {
    counts[e] = cnt[e];
    offsets[e] = off[e];
  }
  if (tid == 0) {
    offsets[El] = off[El];
    *n_active = na;
    *n_chunks = tot[1];
  }
  for (int j = tid; j < na; j += nth) {
    const int e = act[j];
    active[j] = e;
    const int nch = (cnt[e] + ct - 1) / ct;
    for (int c = 0; c < nch; ++c) {
      const int idx = cbase[j] + c;
      if (idx < max_chunks) {
        chunk_slot[idx] = j;
        chunk_c0[idx] = c * ct;
      }
    }
  }
  if (warp < wp) {   // stable permutation
    const int p0 = static_cast<int>(static_cast<long long>(P) * warp / wp);
    const int p1 = static_cast<int>(static_cast<long long>(P) * (warp + 1) / wp);
    for (int c = p0; c < p1; c += 32) {
      const int p = c + lane;
      const int v = p < p1 ? ids_s[p] : -2;
      const uint32_t same = __match_any_sync(0xffffffffu, v);
      const int rank = __popc(same & ((1u << lane) - 1u));
      const int base = v >= 0 ? hist[warp * El + v] : 0;
      if (v >= 0) perm[off[v] + base + rank] = p;
      __syncwarp();
      if (v >= 0 && rank == 0) hist[warp * El + v] = base + __popc(same);
      __syncwarp();
    }
  }
  if (!chunk_info) return;
  // Per-chunk descriptors for the tensor-core expert kernel: (local expert,
  // first permuted position, tokens) and each token's row; completion counters
  // start at zero.
  __syncthreads();
  const int nch = tot[1];
  for (int i = tid; i < nch; i += nth) chunk_done[i] = 0;   // the chunks this call uses
  for (int idx = tid; idx < nch * kChunkRowStride; idx += nth) {
    const int c = idx / kChunkRowStride, i = idx % kChunkRowStride;
    const int e = act[chunk_slot[c]], c0 = chunk_c0[c];
    const int pos0 = off[e] + c0;
    const int nt = min(ct, cnt[e] - c0);
    if (i == 0) chunk_info[c] = make_int4(e, pos0, nt, 0);
    chunk_rows[idx] = i < nt ? perm[pos0 + i] / k : 0;
  }
}

__global__ void __launch_bounds__(1024) route_plan_kernel(
    const int32_t* __restrict__ ids, int P, int e_begin, int e_count, int32_t* __restrict__ counts,
    int32_t* __restrict__ offsets, int32_t* __restrict__ active, int32_t* __restrict__ n_active,
    int32_t* __restrict__ perm, int32_t* __restrict__ n_chunks, int32_t* __restrict__ chunk_slot,
    int32_t* __restrict__ chunk_c0, int max_chunks, int32_t* __restrict__ fold_ticket, int fold_n,
    int k, int4* __restrict__ chunk_info, int32_t* __restrict__ chunk_rows,
    int32_t* __restrict__ chunk_done) {
  extern __shared__ int32_t plan_smem[];
  for (int i = threadIdx.x; i < fold_n; i += blockDim.x) fold_ticket[i] = 0;
  route_plan_block(ids, P, e_begin, e_count, counts, offsets, active, n_active, perm, n_chunks,
                   chunk_slot, chunk_c0, max_chunks, plan_smem, k, chunk_info, chunk_rows,
                   chunk_done);
}

// ---------------------------------------------------------------------------
// Plan for a verify-size batch (P <= kSmallPlanMaxPairs pairs, El <= 1024
// experts) built by ONE warp in shared memory: one match_any pass over the
// pairs in flat order gives each expert's count and each pair's rank inside
// its expert, a warp scan gives the offsets, active list and chunk bases, and
// the permutation and chunk descriptors follow.  No block barriers: the plan
// sits on the critical path of every layer call, where each barrier-separated
// phase costs about a microsecond.  Same outputs as route_plan_block.
// ---------------------------------------------------------------------------
constexpr int kSmallPlanMaxPairs = 512;
__host__ __device__ inline size_t small_plan_smem_bytes(int P, int El) {
  return (3ull * P + 3ull * El + 2) * 4;
}

__device__ void route_plan_small(const int32_t* __restrict__ ids, int P, int e_begin, int El, int k,
                                 int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                 int32_t* __restrict__ active, int32_t* __restrict__ n_active,
                                 int32_t* __restrict__ perm, int32_t* __restrict__ n_chunks,
                                 int32_t* __restrict__ chunk_slot, int32_t* __restrict__ chunk_c0,
                                 int max_chunks, int4* chunk_info, int32_t* chunk_rows,
                                 int32_t* chunk_done, int32_t* sm) {
  const int lane = threadIdx.x & 31;
  const int ct = tc_chunk_tokens(P / k);
  int32_t* ids_s = sm;              // [P] local expert or -1
  int32_t* rank_s = ids_s + P;      // [P] rank of the pair inside its expert (flat order)
  int32_t* perm_s = rank_s + P;     // [P]
  int32_t* cnt = perm_s + P;        // [El]
  int32_t* off = cnt + El;          // [El + 1]
  int32_t* cbase = off + El + 1;    // [El + 1]
  for (int e = lane; e < El; e += 32) cnt[e] = 0;
  __syncwarp();
  for (int g = 0; g < P; g += 32) {
    const int p = g + lane;
    int v = -2;
    if (p < P) {
      v = __ldcg(ids + p) - e_begin;   // written by other CTAs of this grid
      if (v < 0 || v >= El) v = -1;
      ids_s[p] = v;
    }
    const uint32_t same = __match_any_sync(0xffffffffu, v);
    const int r = __popc(same & ((1u << lane) - 1u));
    const int base = v >= 0 ? cnt[v] : 0;
    if (v >= 0) rank_s[p] = base + r;
    __syncwarp();
    if (v >= 0 && r == 0) cnt[v] = base + __popc(same);
    __syncwarp();
  }
  // exclusive scans of (tokens, active experts, chunks); lane owns a run of experts
  const int per = (El + 31) / 32;
  const int e0 = min(El, lane * per), e1 = min(El, e0 + per);
  int s_tok = 0, s_act = 0, s_ch = 0;
  for (int e = e0; e < e1; ++e) {
    const int c = cnt[e];
    s_tok += c;
    s_act += c > 0;
    s_ch += (c + ct - 1) / ct;
  }
  int x_tok = s_tok, x_act = s_act, x_ch = s_ch;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, x_tok, o);
    const int b = __shfl_up_sync(0xffffffffu, x_act, o);
    const int c = __shfl_up_sync(0xffffffffu, x_ch, o);
    if (lane >= o) {
      x_tok += a;
      x_act += b;
      x_ch += c;
    }
  }
  int r_tok = x_tok - s_tok, r_act = x_act - s_act, r_ch = x_ch - s_ch;
  for (int e = e0; e < e1; ++e) {
    const int c = cnt[e];
    off[e] = r_tok;
    cbase[e] = r_ch;
    counts[e] = c;
    offsets[e] = r_tok;
    if (c > 0) {
      active[r_act] = e;
      for (int j = 0; j < (c + ct - 1) / ct; ++j) {
        if (r_ch + j < max_chunks) {
          chunk_slot[r_ch + j] = r_act;
          chunk_c0[r_ch + j] = j * ct;
        }
      }
      ++r_act;
    }
    r_tok += c;
    r_ch += (c + ct - 1) / ct;
  }
  if (lane == 31) {
    off[El] = x_tok;
    offsets[El] = x_tok;
    *n_active = x_act;
    *n_chunks = min(x_ch, max_chunks);
  }
  // counters of the chunks this call uses (later kernels read no others)
  const int nch_used = min(__shfl_sync(0xffffffffu, x_ch, 31), max_chunks);
  for (int i = lane; chunk_done && i < nch_used; i += 32) chunk_done[i] = 0;
  __syncwarp();
  for (int p = lane; p < P; p += 32) {   // stable permutation
    const int v = ids_s[p];
    if (v >= 0) {
      perm_s[off[v] + rank_s[p]] = p;
      perm[off[v] + rank_s[p]] = p;
    }
  }
  if (!chunk_info) return;
  __syncwarp();
  for (int e = e0; e < e1; ++e) {
    const int c = cnt[e];
    for (int j = 0; j < (c + ct - 1) / ct; ++j) {
      const int idx = cbase[e] + j;
      if (idx >= max_chunks) break;
      const int pos0 = off[e] + j * ct, nt = min(ct, c - j * ct);
      chunk_info[idx] = make_int4(e, pos0, nt, 0);
      for (int i = 0; i < ct && i < kChunkRowStride; ++i)   // (prefill chunks read perm)
        chunk_rows[idx * kChunkRowStride + i] = i < nt ? perm_s[pos0 + i] / k : 0;
    }
  }
}

// ---------------------------------------------------------------------------
// Verify-size routing in ONE launch.  Grid (E/16 [+1], M): CTA (g, m) computes
// the logits of experts 16g..16g+15 for token m; the extra column splits token
// m into e2m1 terms for the tensor-core kernels.  The last logit CTA of a token
// (per-token ticket) selects its top-k and gating weights; the last token to
// finish (global ticket) builds the plan.  Tickets live at the start of the
// workspace and are reset by the CTA that completes them.
// ---------------------------------------------------------------------------
constexpr int kFusedRouteWarps = 16;
constexpr int kFusedRouteMaxTokens = 64;

__global__ void __launch_bounds__(kFusedRouteWarps * 32) route_fused_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr, const uint16_t* __restrict__ br,
    int M, int E, int H, int k, float* __restrict__ logits, uint16_t* __restrict__ logits_out,
    int32_t* __restrict__ ids, float* __restrict__ wts, int32_t* __restrict__ ids_out,
    uint16_t* __restrict__ wts_out, int32_t* __restrict__ ticket, int e_begin, int e_count,
    int32_t* __restrict__ counts, int32_t* __restrict__ offsets, int32_t* __restrict__ active,
    int32_t* __restrict__ n_active, int32_t* __restrict__ perm, int32_t* __restrict__ n_chunks,
    int32_t* __restrict__ chunk_slot, int32_t* __restrict__ chunk_c0, int max_chunks,
    int32_t* __restrict__ fold_ticket, int fold_n, uint8_t* __restrict__ x_terms,
    uint8_t* __restrict__ x_sf, int4* __restrict__ chunk_info, int32_t* __restrict__ chunk_rows,
    int32_t* __restrict__ chunk_done) {
  extern __shared__ __align__(16) uint8_t fused_smem[];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_logit = (E + kFusedRouteWarps - 1) / kFusedRouteWarps;
  pdl_wait();   // x is produced by whatever ran before us on the stream
  const int m = blockIdx.y;
  if (blockIdx.x == n_logit) {   // the token's e2m1 terms for the tensor-core expert kernel
    decompose_rows(x, H, H, m, 1, x_terms + static_cast<size_t>(m) * term_row_bytes(H),
                   x_sf + static_cast<size_t>(m) * term_sf_row_bytes(H));
    return;
  }
  const int e = blockIdx.x * kFusedRouteWarps + warp;
  if (e < E) {
    const float v = logit_warp(x, wr, br, m, e, H);
    if (lane == 0) {
      logits[static_cast<size_t>(m) * E + e] = v;
      if (logits_out) logits_out[static_cast<size_t>(m) * E + e] = float_to_bf16_bits(v);
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    is_last = (atomicAdd(&ticket[1 + m], 1) == n_logit - 1);
    if (is_last) ticket[1 + m] = 0;
  }
  __syncthreads();
  if (!is_last) return;
  // all logits of token m are written: its top-k and gating weights
  __threadfence();
  if (warp == 0)
    select_softmax_token(logits + static_cast<size_t>(m) * E, reinterpret_cast<KV*>(fused_smem), m,
                         E, k, ids, wts, ids_out, wts_out, fused_smem + E * sizeof(KV));
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    is_last = (atomicAdd(&ticket[0], 1) == M - 1);
    if (is_last) ticket[0] = 0;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < fold_n; i += blockDim.x) fold_ticket[i] = 0;
  if (warp != 0) return;
  route_plan_small(ids, M * k, e_begin, e_count, k, counts, offsets, active, n_active, perm,
                   n_chunks, chunk_slot, chunk_c0, max_chunks, chunk_info, chunk_rows, chunk_done,
                   reinterpret_cast<int32_t*>(fused_smem));
}

// ---------------------------------------------------------------------------
int launch_route(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                 void* logits_out, int32_t* ids_out, void* wts_out, const Workspace& ws,
                 cudaStream_t stream) {
  const int E = d.num_experts, H = d.hidden, k = d.top_k;
  const int El = d.expert_end - d.expert_begin;
  const bool tc = tc_supported(d);
  if (M > 0 && M <= kFusedRouteMaxTokens && M * k <= kSmallPlanMaxPairs && El <= 1024) {
    const size_t smem = max(static_cast<size_t>(E) * sizeof(KV) + kTopkWarpScratch,
                            small_plan_smem_bytes(M * k, El));
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(route_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return FLYAI_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((E + kFusedRouteWarps - 1) / kFusedRouteWarps + (tc ? 1 : 0), M);
    cfg.blockDim = dim3(kFusedRouteWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t st = cudaLaunchKernelEx(
        &cfg, route_fused_kernel, static_cast<const uint16_t*>(x),
        static_cast<const uint16_t*>(w.router_w), static_cast<const uint16_t*>(w.router_b), M, E, H,
        k, ws.logits, static_cast<uint16_t*>(logits_out), ws.ids, ws.wts, ids_out,
        static_cast<uint16_t*>(wts_out), ws.route_ticket, d.expert_begin, El, ws.counts,
        ws.offsets, ws.active, ws.n_active, ws.perm, ws.n_chunks, ws.chunk_slot, ws.chunk_c0,
        ws.max_chunks, ws.fold_ticket, M * (d.hidden / 16), tc ? ws.x_terms : nullptr,
        tc ? ws.x_sf : nullptr, tc ? ws.chunk_info : nullptr, ws.chunk_rows, ws.chunk_done);
    note_launch();
    return st == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
  }
  if (M > 0) {
    if (!ws.plog) return FLYAI_ERR_UNSUPPORTED;   // batches above 64 tokens carve the partials
    nvp_logits_kernel<<<dim3((E + kLgExp - 1) / kLgExp, (M + kLgTok - 1) / kLgTok, kNpLogitSlices), 256, 0,
                        stream>>>(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w.router_w), M,
                                  E, H, ws.plog, ws.pxm);
    note_launch();
    route_logits_sum_kernel<<<4 * 148, 256, 0, stream>>>(ws.plog, static_cast<const uint16_t*>(w.router_b), M, E,
                                                         ws.logits, static_cast<uint16_t*>(logits_out));
    note_launch();
    const size_t smem = 8 * (static_cast<size_t>(E) * sizeof(KV) + kTopkWarpScratch);
    route_select_softmax_kernel<<<(M + 7) / 8, 256, smem, stream>>>(
        ws.logits, M, E, k, ws.ids, ws.wts, ids_out, static_cast<uint16_t*>(wts_out));
    note_launch();
  }
  const size_t psmem = plan_smem_bytes(M * k, El, 32);
  if (psmem > 48 * 1024 &&
      cudaFuncSetAttribute(route_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(psmem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  route_plan_kernel<<<1, 1024, psmem, stream>>>(ws.ids, M * k, d.expert_begin, El, ws.counts,
                                                ws.offsets, ws.active, ws.n_active, ws.perm,
                                                ws.n_chunks, ws.chunk_slot, ws.chunk_c0,
                                                ws.max_chunks, ws.fold_ticket, M * (d.hidden / 16),
                                                k, tc ? ws.chunk_info : nullptr, ws.chunk_rows,
                                                ws.chunk_done);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Routing chosen by the caller (Kimi-K3's moe_infer seam): the ids are checked
// against [0, E) -- the expert kernels index the bank with them -- and copied
// with the weights; then the plan as for routed batches.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) route_ids_kernel(const int32_t* __restrict__ ids_in,
                                                        const float* __restrict__ wts_in, int P, int E,
                                                        int32_t* __restrict__ ids, float* __restrict__ wts,
                                                        int32_t* err) {
  pdl_wait();
  pdl_launch_dependents();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P; i += gridDim.x * blockDim.x) {
    int e = __ldg(&ids_in[i]);
    if (e < 0 || e >= E) {
      atomicOr(err, kErrBadIndex);
      e = 0;
    }
    ids[i] = e;
    wts[i] = __ldg(&wts_in[i]);
  }
}

int launch_route_ids(const flyai_moe_desc& d, int M, const int32_t* ids, const float* wts,
                     const Workspace& ws, cudaStream_t stream) {
  const int k = d.top_k, P = M * k, El = d.expert_end - d.expert_begin;
  if (P == 0) return FLYAI_OK;
  route_ids_kernel<<<(P + 255) / 256, 256, 0, stream>>>(ids, wts, P, d.num_experts, ws.ids, ws.wts,
                                                         ws.err);
  note_launch();
  const size_t psmem = plan_smem_bytes(P, El, 32);
  if (psmem > 48 * 1024 &&
      cudaFuncSetAttribute(route_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(psmem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  route_plan_kernel<<<1, 1024, psmem, stream>>>(ws.ids, P, d.expert_begin, El, ws.counts, ws.offsets,
                                                ws.active, ws.n_active, ws.perm, ws.n_chunks,
                                                ws.chunk_slot, ws.chunk_c0, ws.max_chunks, ws.fold_ticket,
                                                M * (d.hidden / 16), k, ws.chunk_info, ws.chunk_rows,
                                                ws.chunk_done);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

}  // namespace flyai
