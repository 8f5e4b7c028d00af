// DeepSeek-V3-style FP8 MoE layer on sm_100a (FLYAI_FMT_FP8_BLOCK with
// FLYAI_GATE_SIGMOID_GROUP and FLYAI_ACT_SILU).
//
// Reference arithmetic:
//   gate     KimiMoEGate.forward, vendor/kimi_k3_ref/modeling_kimi_linear.py:703-759
//            (fp32 logits, sigmoid, + e_score_correction_bias for the choice,
//            group score = sum of the group's top-2, top topk_group groups,
//            top-k inside them, unbiased scores renormalised / (sum + 1e-20),
//            x routed_scaling_factor);
//   experts  Expert.forward, vendor/deepseek_v4_ref/inference/model.py:599-611 with
//            fp8 Linear (model.py:114-124): act_quant per 1x128 (amax floored at
//            1e-4, scale = amax / 448, engines/deepseek_v4/v4_kernels_cpu.py:89-104),
//            fp8_gemm with 128x128 fp32 weight scales, output bf16 (:158-164);
//            silu(gate) * up in fp32, x routing weight, to bf16, then w2 likewise;
//   combine  MoE.forward, model.py:634-649: fp32 y, routed experts added in
//            ascending expert id, then the shared expert, y to bf16.
//
// Four launches, PDL-chained: f8_route_kernel (logits over all CTAs, the last
// CTA selects the experts of every token and builds the plan), f8_scatter_kernel
// (each chunk's token rows quantised to e4m3 in the MMA's K-major tile layout),
// f8_moe_kernel (gate/up and down on tcgen05 kind::f8f6f4, one persistent CTA
// per SM) and f8_combine_kernel.  Every wait is bounded (~2 s) and records
// kErrWaitTimeout.
#include <cuda_fp8.h>
#include <math.h>

#include <type_traits>

#include "act_quant.cuh"
#include "common.cuh"
#include "fp8_moe.cuh"
#include "tc_bank.cuh"
#include "tcgen05.cuh"
#include "torch_topk.cuh"
#include "v4.cuh"

namespace flyai {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename Kern, typename... Args>
static cudaError_t f8_launch(Kern kernel, dim3 grid, int block, size_t smem, cudaStream_t s,
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
size_t fp8_packed_bytes(const flyai_moe_desc& d, int proj) {
  return f8_bank(d.hidden, d.inter, proj).expert *
         static_cast<size_t>(d.expert_end - d.expert_begin + d.n_shared);
}

// One thread per 16-byte unit of the bank: unit 0 of a block is its header
// (the fp32 scale of each tile), the rest are tile chunks.
__global__ void f8_pack_kernel(const uint8_t* __restrict__ w, const float* __restrict__ sc,
                               uint8_t* __restrict__ packed, int nexp, int R, int K, F8Bank b) {
  const size_t upb = b.block / 16;
  const size_t total = upb * b.RB * b.KB * static_cast<size_t>(nexp);
  const int half_rows = b.tiles == 2 ? R / 2 : 0;
  for (size_t u = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; u < total;
       u += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t blk = u / upb;
    const int v = static_cast<int>(u % upb);
    const int e = static_cast<int>(blk / (static_cast<size_t>(b.RB) * b.KB));
    const int rem = static_cast<int>(blk % (static_cast<size_t>(b.RB) * b.KB));
    const int rb = rem / b.KB, kb = rem % b.KB;
    uint4 out;
    if (v == 0) {
      float h[4] = {0.f, 0.f, 0.f, 0.f};
      for (int tt = 0; tt < b.tiles; ++tt) {
        const int srb = (tt * half_rows) / kF8Blk + rb;
        h[tt] = sc[(static_cast<size_t>(e) * (R / kF8Blk) + srb) * (K / kF8Blk) + kb];
      }
      out = make_uint4(__float_as_uint(h[0]), __float_as_uint(h[1]), __float_as_uint(h[2]),
                       __float_as_uint(h[3]));
    } else {
      const int wi = v - 1, tt = wi / (kF8Tile / 16), ti = wi % (kF8Tile / 16);
      const int c = ti / kF8Blk, r = ti % kF8Blk;
      const size_t row = static_cast<size_t>(e) * R + tt * half_rows + rb * kF8Blk + r;
      out = *reinterpret_cast<const uint4*>(w + row * K + kb * kF8Blk + c * 16);
    }
    *reinterpret_cast<uint4*>(packed + blk * b.block + static_cast<size_t>(v) * 16) = out;
  }
}

int launch_fp8_pack(const flyai_moe_desc& d, int proj, const void* weight, const void* scale,
                    void* packed, cudaStream_t stream) {
  const int nexp = d.expert_end - d.expert_begin + d.n_shared;
  if (nexp == 0) return FLYAI_OK;
  const F8Bank b = f8_bank(d.hidden, d.inter, proj);
  const int R = proj == FLYAI_PROJ_W13 ? 2 * d.inter : d.hidden;
  const int K = proj == FLYAI_PROJ_W13 ? d.hidden : d.inter;
  f8_pack_kernel<<<2368, 256, 0, stream>>>(static_cast<const uint8_t*>(weight),
                                           static_cast<const float*>(scale),
                                           static_cast<uint8_t*>(packed), nexp, R, K, b);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Gate + routing plan
// ---------------------------------------------------------------------------
// f8_route_kernel, grid (E/2, ceil(M/8)), 8 warps: CTA (b, g) computes the fp32
// logits of experts 2b, 2b+1 for the 8 tokens of group g (warp w: K slice w of
// 1024 elements, the lane's 32 weights of both experts held in registers, two
// tokens' activations in flight at a time) and act_quant's a share of the token
// rows (token-major e4m3 + scales, gathered into chunk tiles by the scatter).
// The last CTA of a token group selects its tokens' experts (one warp per
// token); the last group to finish builds the plan.
constexpr int kF8RouteThreads = 256;
constexpr int kF8RouteExperts = 2;    // experts per CTA
constexpr int kF8RouteTokens = 8;     // tokens per CTA
constexpr int kF8Slice = 1024;        // K elements per warp (32 per lane)
// The NVFP4 gate sums exact products in fp64 (order-free): rows up to 4096 use
// 512-element slices (16 per lane) so more of the 8 warps share a row.
__host__ __device__ inline int f8_route_slice(bool nv, int H) { return nv && H <= 4096 ? 512 : kF8Slice; }

struct F8RouteParams {
  const uint16_t* x;
  uint8_t* xsf;          // NVFP4: [M, H/128, kNvRowSf] term scale words
  const uint16_t* w;     // bf16 [E, H]
  const float* bias;     // fp32 [E] correction bias (choice only)
  int M, E, H, k, n_group, topk_group, e0, El, nsh;
  float scale;
  float* logits;
  int32_t* ids;
  float* wts;
  float* out_logits;
  int32_t* out_ids;
  float* out_wts;
  uint8_t* xq;           // [M, H] e4m3 token rows
  float* xs;             // [M, H/128] their scales
  int32_t* counts;
  int32_t* offsets;
  int32_t* perm;
  int32_t* inv;
  int32_t* n_chunks;
  int4* chunk_info;
  int32_t* chunk_done;
  int32_t* ticket;       // [0] token groups finished, [1 + g] CTAs of group g finished
  // DeepSeek-V4 gate (FLYAI_GATE_SQRTSOFTPLUS): scores sqrt(softplus(logit)),
  // torch.topk sorted (descending, torch's order among ties), and on a
  // hash-routed layer ids = tid2eid[input_ids[t]] instead of the top-k
  int score_fn;          // 0: sigmoid, 1: sqrt(softplus)
  int sorted;            // top-k order: torch.topk(sorted=True) instead of sorted=False
  const int32_t* tid2eid;    // [vocab, k] or null
  const int32_t* input_ids;  // [M] (with tid2eid)
  int vocab;
  int ue8m0;             // act_quant scales 2^ceil(log2(amax/448)) (scale_fmt "ue8m0")
  // bf16 [M, E] router logits the caller computed (MiniMax-M2.5's stage passes
  // F.linear(h, gate) to its FusedMoE): the selection reads these instead of the
  // kernel's own (which still runs for the token-row factors)
  const uint16_t* logits_in;
  int32_t* err;          // error word (bit 2: an input id or table entry out of range)
};


// The gate's score of a logit: sigmoid (DeepSeek-V3, MiniMax-M2) or
// sqrt(softplus) with torch's threshold 20 (DeepSeek-V4, model.py:575-576).
__device__ __forceinline__ float f8_score(int fn, float l) {
  if (fn == 1) return sqrtf(l > 20.f ? l : log1pf(expf(l)));
  return __frcp_rn(__fadd_rn(1.f, expf(-l)));
}

// The ids of token t when the layer is hash-routed: tid2eid[input_ids[t]], an id
// or table entry out of range recorded in the error word (and replaced by 0).
__device__ __forceinline__ int f8_hash_id(const F8RouteParams& p, int t, int r) {
  int tok = __ldg(&p.input_ids[t]);
  if (tok < 0 || tok >= p.vocab) {
    atomicOr(p.err, kErrBadIndex);
    tok = 0;
  }
  int id = __ldg(&p.tid2eid[static_cast<size_t>(tok) * p.k + r]);
  if (id < 0 || id >= p.E) {
    atomicOr(p.err, kErrBadIndex);
    id = 0;
  }
  return id;
}

// The top-k of the choice row (already in row[0..E)): torch.topk's order, sorted
// or not, or the hash table's ids.  Leaves the ids in row[0..k).i.
__device__ __forceinline__ void f8_topk_row(const F8RouteParams& p, int t, KV* row, void* tks) {
  const int lane = threadIdx.x & 31;
  if (p.tid2eid) {
    __syncwarp();
    if (lane < p.k) row[lane].i = f8_hash_id(p, t, lane);
    __syncwarp();
    return;
  }
  torch_topk_warp(row, p.E, p.k, tks);
  if (p.sorted && p.k * 64 > p.E) {   // std::sort(q, q+k-1) after nth_element
    if (lane == 0) kv_insertion_sort(row, 0, p.k - 1);
    __syncwarp();
  }
}

// Exclusive prefix of one int per thread over the block; *total = block sum.
__device__ int f8_block_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) tmp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int t = lane < nw ? tmp[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += n;
    }
    if (lane < nw) tmp[lane] = ti - t;
    if (lane == nw - 1) tmp[32] = ti;
  }
  __syncthreads();
  const int r = tmp[warp] + inc - v;
  *total = tmp[32];
  __syncthreads();
  return r;
}

// act_quant of one 128-element block of a bf16 row by one warp (4 elements per lane).
// ue8m0: the scale is 2^ceil(log2(amax/448)) (scale_fmt "ue8m0"), else amax/448.
__device__ __forceinline__ void f8_quant_block(const uint16_t* src, uint8_t* q, float* sc, int lane,
                                               int ue8m0) {
  float s;
  const uint32_t packed = act_quant4(src, lane, ue8m0, s);
  *reinterpret_cast<uint32_t*>(q + lane * 4) = packed;
  if (lane == 0) *sc = s;
}

// Per-warp selection scratch: torch_topk_warp's, then 32 (value, index) pairs
// for the group scores.
constexpr int kF8SelScratch = kTopkWarpScratch + 32 * static_cast<int>(sizeof(KV));

// The groups torch.topk(group_scores, topk_group, sorted=False) keeps -- a set,
// but with tied scores at the boundary which group wins is decided by torch's
// selection order, so it is computed by the restatement (one lane, n_group <= 32
// pairs).  Lanes with holder set pass group g's score; all lanes get the mask.
__device__ uint32_t f8_keep_groups(float gs, int g, bool holder, int n_group, int topk_group,
                                   void* tks) {
  KV* gk = reinterpret_cast<KV*>(static_cast<char*>(tks) + kTopkWarpScratch);
  __syncwarp();
  if (holder) gk[g] = KV{gs, g};
  __syncwarp();
  if ((threadIdx.x & 31) == 0) torch_topk_serial(gk, n_group, topk_group, false);
  __syncwarp();
  uint32_t keep = 0;
  for (int r = 0; r < topk_group; ++r) keep |= 1u << gk[r].i;
  __syncwarp();
  return keep;
}

// Experts of token t, one warp.  Lane l holds experts l*nj .. l*nj+nj-1; row is
// a warp-private shared buffer of E (value, index) pairs (group scores, then the
// top-k), tks the warp's torch_topk_warp scratch.  The ids come out in the order
// torch.topk(sorted=False) returns them on CPU (torch_topk.cuh); the weights are
// renormalised in that slot order, as the reference sums them.
__device__ void f8_select_token(const F8RouteParams& p, int t, KV* row, void* tks) {
  const int lane = threadIdx.x & 31, E = p.E, nj = E >> 5, k = p.k;
  float sc[16], ch[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    sc[j] = 0.f;
    ch[j] = -INFINITY;
    if (j < nj) {
      const int e = lane * nj + j;
      const float l = p.logits_in ? __uint_as_float(static_cast<uint32_t>(__ldg(p.logits_in + static_cast<size_t>(t) * E + e)) << 16)
                                  : __ldcg(p.logits + static_cast<size_t>(t) * E + e);
      const float s = f8_score(p.score_fn, l);
      sc[j] = s;
      ch[j] = __fadd_rn(s, __ldg(p.bias + e));
      row[e].v = ch[j];
    }
  }
  __syncwarp();
  if (p.n_group > 1 && p.n_group > p.topk_group) {
    // group score = sum of the group's two largest choice scores (as values)
    const int gsize = E / p.n_group;
    float gs = -INFINITY;
    if (lane < p.n_group) {
      float m1 = -INFINITY, m2 = -INFINITY;
      for (int i = 0; i < gsize; ++i) {
        const float v = row[lane * gsize + i].v;
        if (v > m1) {
          m2 = m1;
          m1 = v;
        } else if (v > m2) {
          m2 = v;
        }
      }
      gs = __fadd_rn(m1, m2);
    }
    const uint32_t keep = f8_keep_groups(gs, lane, lane < p.n_group, p.n_group, p.topk_group, tks);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nj && !((keep >> ((lane * nj + j) / gsize)) & 1u)) ch[j] = -INFINITY;
  }
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j < nj) row[lane * nj + j] = KV{ch[j], lane * nj + j};
  f8_topk_row(p, t, row, tks);
  int my_id = 0;
  float my_w = 0.f;
  for (int r = 0; r < k; ++r) {
    const int id = row[r].i;
    const int owner = id / nj, jj = id - owner * nj;
    float s_sel = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j == jj) s_sel = sc[j];
    s_sel = __shfl_sync(0xffffffffu, s_sel, owner);
    if (lane == r) {
      my_id = id;
      my_w = s_sel;
    }
  }
  float sum = 0.f;
  for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, my_w, r));
  const float denom = __fadd_rn(sum, 1e-20f);
  if (lane < k) {
    const float wv = __fmul_rn(__fdiv_rn(my_w, denom), p.scale);
    const int f = t * k + lane;
    p.ids[f] = my_id;
    p.wts[f] = wv;
    if (p.out_ids) p.out_ids[f] = my_id;
    if (p.out_wts) p.out_wts[f] = wv;
  }
}

// kNv: the NVFP4 layer -- bf16 logits (exact fp64 sum rounded like a bf16
// F.linear), token rows split into e2m1 terms, chunks of kNvChunk tokens.
// Experts of token t for E = 256 (both configured layer shapes), one warp, as
// f8_select_token with shorter latency chains: lane l's eight experts 8l..8l+7
// load as two float4 each of logits and bias; groups whose size is a multiple
// of 8 (a power-of-two number of lanes) get their top-2 sums by shuffles within
// the lane group; the top-k pops the heads of per-lane lists sorted once by an
// odd-even merge network.  The top-k then comes from torch_topk_warp, in torch's
// sorted=False order, as in f8_select_token.
__device__ void f8_select_token_256(const F8RouteParams& p, int t, KV* row, void* tks) {
  const int lane = threadIdx.x & 31, k = p.k;
  const float4* bs = reinterpret_cast<const float4*>(p.bias + lane * 8);
  const float4 b0 = __ldg(bs), b1 = __ldg(bs + 1);
  float lv[8];
  if (p.logits_in) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(p.logits_in + static_cast<size_t>(t) * 256 + lane * 8));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lv[2 * j] = __uint_as_float(w[j] << 16);
      lv[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  } else {
    const float4* lg = reinterpret_cast<const float4*>(p.logits + static_cast<size_t>(t) * 256 + lane * 8);
    const float4 l0 = __ldcg(lg), l1 = __ldcg(lg + 1);
    lv[0] = l0.x, lv[1] = l0.y, lv[2] = l0.z, lv[3] = l0.w;
    lv[4] = l1.x, lv[5] = l1.y, lv[6] = l1.z, lv[7] = l1.w;
  }
  const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  float sc[8], ch[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sc[j] = f8_score(p.score_fn, lv[j]);
    ch[j] = __fadd_rn(sc[j], bv[j]);
  }
  if (p.n_group > 1 && p.n_group > p.topk_group) {
    const int gsize = 256 / p.n_group, lpg = gsize / 8;
    if (gsize % 8 == 0 && (lpg & (lpg - 1)) == 0) {
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (ch[j] > m1) {
          m2 = m1;
          m1 = ch[j];
        } else if (ch[j] > m2) {
          m2 = ch[j];
        }
      }
      for (int o = 1; o < lpg; o <<= 1) {
        const float c1 = __shfl_xor_sync(0xffffffffu, m1, o);
        const float c2 = __shfl_xor_sync(0xffffffffu, m2, o);
        const float n2 = m1 >= c1 ? fmaxf(m2, c1) : fmaxf(m1, c2);
        m1 = fmaxf(m1, c1);
        m2 = n2;
      }
      const float gs = __fadd_rn(m1, m2);
      const int my_g = lane / lpg;
      const bool leader = (lane % lpg) == 0;
      const uint32_t keep = f8_keep_groups(gs, my_g, leader, p.n_group, p.topk_group, tks);
      if (!((keep >> my_g) & 1u)) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ch[j] = -INFINITY;
      }
    } else {   // other group sizes: group scores from a shared-memory row
#pragma unroll
      for (int j = 0; j < 8; ++j) row[lane * 8 + j].v = ch[j];
      __syncwarp();
      float gsc = -INFINITY;
      if (lane < p.n_group) {
        float m1 = -INFINITY, m2 = -INFINITY;
        for (int i = 0; i < gsize; ++i) {
          const float v = row[lane * gsize + i].v;
          if (v > m1) {
            m2 = m1;
            m1 = v;
          } else if (v > m2) {
            m2 = v;
          }
        }
        gsc = __fadd_rn(m1, m2);
      }
      const uint32_t keep = f8_keep_groups(gsc, lane, lane < p.n_group, p.n_group, p.topk_group, tks);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (!((keep >> ((lane * 8 + j) / gsize)) & 1u)) ch[j] = -INFINITY;
    }
  }
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) row[lane * 8 + j] = KV{ch[j], lane * 8 + j};
  f8_topk_row(p, t, row, tks);
  int my_id = 0;
  float my_w = 0.f;
  for (int r = 0; r < k; ++r) {
    const int id = row[r].i;
    const int owner = id >> 3, jj = id & 7;
    float s_sel = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j == jj) s_sel = sc[j];
    s_sel = __shfl_sync(0xffffffffu, s_sel, owner);
    if (lane == r) {
      my_id = id;
      my_w = s_sel;
    }
  }
  float sum = 0.f;
  for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, my_w, r));
  const float denom = __fadd_rn(sum, 1e-20f);
  if (lane < k) {
    const float wv = __fmul_rn(__fdiv_rn(my_w, denom), p.scale);
    const int f = t * k + lane;
    p.ids[f] = my_id;
    p.wts[f] = wv;
    if (p.out_ids) p.out_ids[f] = my_id;
    if (p.out_wts) p.out_wts[f] = wv;
  }
}

template <bool kNv>
__global__ void __launch_bounds__(kF8RouteThreads, kNv ? 1 : 2) f8_route_kernel(const __grid_constant__ F8RouteParams p) {
  constexpr int C = kNv ? kNvChunk : kF8Chunk;
  using Acc = typename std::conditional<kNv, double, float>::type;
  __shared__ Acc part[kF8RouteTokens][8][kF8RouteExperts];
  __shared__ float rowmax[kF8RouteTokens][8];   // NVFP4: |x| maximum per token and K slice
  __shared__ int32_t ids_s[kF8MaxTokens * kMaxTopK];
  __shared__ int32_t off_s[kF8MaxExperts];
  __shared__ __align__(16) int32_t scratch[16 * kF8MaxExperts];   // choice rows (KV), then warp histograms
  __shared__ __align__(16) uint8_t tk_s[8][kF8SelScratch];
  __shared__ int scan_tmp[33];
  __shared__ int last_s;
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = p.M, E = p.E, H = p.H;
  const int eb = blockIdx.x * kF8RouteExperts, t0 = blockIdx.y * kF8RouteTokens;
  const int nt = min(kF8RouteTokens, M - t0);

  // ---- logits of experts eb, eb+1 for tokens t0 .. t0+nt-1 ----
  const int slice = f8_route_slice(kNv, H), nc = slice / 256;   // 16-byte loads per lane
  for (int s = warp; s * slice < H; s += 8) {
    const int k0 = s * slice + lane * (slice / 32);
    const bool live = k0 < H;
    uint4 wv[kF8RouteExperts][4];
#pragma unroll
    for (int e = 0; e < kF8RouteExperts; ++e)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        wv[e][c] = (live && c < nc && eb + e < E)
                       ? ldg_nc_v4(p.w + static_cast<size_t>(eb + e) * H + k0 + c * 8)
                       : make_uint4(0u, 0u, 0u, 0u);
    for (int i0 = 0; i0 < nt; i0 += 2) {
      uint4 xv[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          xv[i][c] = (live && c < nc && i0 + i < nt)
                         ? __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t0 + i0 + i) * H + k0 + c * 8))
                         : make_uint4(0u, 0u, 0u, 0u);
      if constexpr (kNv) {   // the row maxima the term split is normalised by
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          float m = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t xr[4] = {xv[i][c].x, xv[i][c].y, xv[i][c].z, xv[i][c].w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
              m = fmaxf(m, fmaxf(fabsf(__uint_as_float(xr[q] << 16)),
                                 fabsf(__uint_as_float(xr[q] & 0xFFFF0000u))));
          }
          m = warp_max(m);
          if (lane == 0 && i0 + i < nt)
            rowmax[i0 + i][warp] = s == warp ? m : fmaxf(rowmax[i0 + i][warp], m);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        Acc acc[kF8RouteExperts];
#pragma unroll
        for (int e = 0; e < kF8RouteExperts; ++e) {
          acc[e] = 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t xr[4] = {xv[i][c].x, xv[i][c].y, xv[i][c].z, xv[i][c].w};
            const uint32_t wr[4] = {wv[e][c].x, wv[e][c].y, wv[e][c].z, wv[e][c].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float x0 = __uint_as_float(xr[q] << 16), w0 = __uint_as_float(wr[q] << 16);
              const float x1 = __uint_as_float(xr[q] & 0xFFFF0000u), w1 = __uint_as_float(wr[q] & 0xFFFF0000u);
              if constexpr (kNv) {   // bf16 x bf16 products are exact in fp32
                acc[e] += static_cast<double>(__fmul_rn(x0, w0));
                acc[e] += static_cast<double>(__fmul_rn(x1, w1));
              } else {
                acc[e] = fmaf(x0, w0, acc[e]);
                acc[e] = fmaf(x1, w1, acc[e]);
              }
            }
          }
          if constexpr (kNv) acc[e] = warp_sum_f64(acc[e]);
          else acc[e] = warp_sum(acc[e]);
        }
        if (lane == 0 && i0 + i < nt) {
#pragma unroll
          for (int e = 0; e < kF8RouteExperts; ++e)
            part[i0 + i][warp][e] = s == warp ? acc[e] : part[i0 + i][warp][e] + acc[e];
        }
      }
    }
  }
  // ---- token rows quantised (FP8: over every warp of the grid) or split into
  // terms (NVFP4: this token group's rows over the warps of its CTAs) ----
  if constexpr (kNv) {
    __syncthreads();
    const int KB = H / kF8Blk, nsl0 = min(8, (H + slice - 1) / slice);
    const int nw = gridDim.x * 8, gw = blockIdx.x * 8 + warp;
    for (int u = gw; u < nt * KB; u += nw) {
      const int i = u / KB, kb = u - i * KB, t = t0 + i;
      float m = rowmax[i][0];
      for (int s = 1; s < nsl0; ++s) m = fmaxf(m, rowmax[i][s]);
      const int r = nv_block_exp(m);
      const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p.x + static_cast<size_t>(t) * H +
                                                            kb * kF8Blk + lane * 4));
      float v[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u),
                    __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xFFFF0000u)};
      const size_t tu = static_cast<size_t>(t) * KB + kb;
      nv_split_block(v, lane, r, p.xq + tu * kNvRowBytes, p.xsf + tu * kNvRowSf);
      if (lane == 0) p.xs[tu] = exp2i(r);
    }
  } else {
    const int KB = H / kF8Blk;
    const int nw = gridDim.x * gridDim.y * 8;
    const int gw = (blockIdx.y * gridDim.x + blockIdx.x) * 8 + warp;
    for (int u = gw; u < M * KB; u += nw) {
      const int t = u / KB, kb = u - t * KB;
      f8_quant_block(p.x + static_cast<size_t>(t) * H + kb * kF8Blk,
                     p.xq + static_cast<size_t>(t) * H + kb * kF8Blk,
                     p.xs + static_cast<size_t>(t) * KB + kb, lane, p.ue8m0);
    }
  }
  __syncthreads();
  const int nsl = min(8, (H + slice - 1) / slice);
  for (int u = threadIdx.x; u < nt * kF8RouteExperts; u += blockDim.x) {
    const int i = u / kF8RouteExperts, e = u % kF8RouteExperts;
    if (eb + e >= E) continue;
    float v;
    if constexpr (kNv) {   // exact sum, rounded once to fp32 and once to bf16
      Acc a = part[i][0][e];
      for (int s = 1; s < nsl; ++s) a += part[i][s][e];
      v = bf16r(__double2float_rn(a));
    } else {
      v = part[i][0][e];
      for (int s = 1; s < nsl; ++s) v = __fadd_rn(v, part[i][s][e]);
    }
    p.logits[static_cast<size_t>(t0 + i) * E + eb + e] = v;
    if (p.out_logits) p.out_logits[static_cast<size_t>(t0 + i) * E + eb + e] = v;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    last_s = atomicAdd(&p.ticket[1 + blockIdx.y], 1) == static_cast<int>(gridDim.x) - 1;
    if (last_s) p.ticket[1 + blockIdx.y] = 0;
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();

  // ---- this token group's experts ----
  KV* rows = reinterpret_cast<KV*>(scratch);
  if (warp < nt) {
    if (E == 256) f8_select_token_256(p, t0 + warp, rows + warp * E, tk_s[warp]);
    else f8_select_token(p, t0 + warp, rows + warp * E, tk_s[warp]);
  }
  if (gridDim.y > 1) {   // (one token group: this CTA is the last one already)
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      last_s = atomicAdd(&p.ticket[0], 1) == static_cast<int>(gridDim.y) - 1;
      if (last_s) p.ticket[0] = 0;
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
  } else {
    __syncthreads();
  }

  // ---- plan: pairs by ascending local expert, ascending flat index inside one ----
  // Ranks come from per-32-pair histograms (match_any), so no pass is O(P) per thread.
  const int k = p.k, P = M * k, El = p.El, e0 = p.e0;
  int32_t* hist = scratch;   // [16][El]: pairs of local expert el in 32-pair group vw
  for (int q = threadIdx.x; q < P; q += blockDim.x) ids_s[q] = __ldcg(p.ids + q);
  for (int i = threadIdx.x; i < 16 * El; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  int el_r[2], rank_r[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = r * blockDim.x + threadIdx.x, vw = q >> 5;
    int el = q < P ? ids_s[q] - e0 : -1;
    if (el >= El) el = -1;
    const int key = el >= 0 ? el : -1 - lane;
    const uint32_t mask = __match_any_sync(0xffffffffu, key);
    const int below = __popc(mask & ((1u << lane) - 1u));
    if (el >= 0 && below == 0) hist[vw * El + el] = __popc(mask);
    el_r[r] = el;
    rank_r[r] = below;
  }
  __syncthreads();
  // experts 2*tid, 2*tid+1 of this thread: counts, histograms to exclusive prefixes
  int cnt2[2] = {0, 0};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int el = 2 * threadIdx.x + h;
    if (el < El) {
      int pre = 0;
      for (int vw = 0; vw < 16; ++vw) {
        const int c = hist[vw * El + el];
        hist[vw * El + el] = pre;
        pre += c;
      }
      cnt2[h] = pre;
    }
  }
  int pairs_local = 0, routed_chunks = 0;
  const int off = f8_block_scan(cnt2[0] + cnt2[1], scan_tmp, &pairs_local);
  const int nch0 = (cnt2[0] + C - 1) / C, nch1 = (cnt2[1] + C - 1) / C;
  const int cbase = f8_block_scan(nch0 + nch1, scan_tmp, &routed_chunks);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int el = 2 * threadIdx.x + h;
    if (el >= El) continue;
    const int o = off + (h ? cnt2[0] : 0), cb = cbase + (h ? nch0 : 0), cnt = cnt2[h];
    off_s[el] = o;
    p.counts[el] = cnt;
    p.offsets[el] = o;
    for (int c = 0; c * C < cnt; ++c)
      p.chunk_info[cb + c] = make_int4(el, o + c * C, min(C, cnt - c * C), 0);
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = r * blockDim.x + threadIdx.x;
    if (q >= P) continue;
    const int el = el_r[r];
    if (el < 0) {
      p.inv[q] = -1;
      continue;
    }
    const int pos = off_s[el] + hist[(q >> 5) * El + el] + rank_r[r];
    p.perm[pos] = q;
    p.inv[q] = pos;
  }
  // the shared expert is computed by the shard that holds expert 0
  const int nsc = (p.nsh && p.e0 == 0) ? (M + C - 1) / C : 0;
  for (int c = threadIdx.x; c < nsc; c += blockDim.x)
    p.chunk_info[routed_chunks + c] = make_int4(El, P + c * C, min(C, M - c * C), 0);
  const int nchunks = routed_chunks + nsc;
  for (int c = threadIdx.x; c < nchunks; c += blockDim.x) p.chunk_done[c] = 0;
  if (threadIdx.x == 0) {
    p.offsets[El] = pairs_local;
    *p.n_chunks = nchunks;
  }
}

int launch_fp8_route(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                     float* logits, int32_t* topk_ids, float* topk_weights,
                     const Fp8Workspace& ws, cudaStream_t stream, const int32_t* tid2eid,
                     const int32_t* input_ids, int vocab, const void* logits_in) {
  if (M == 0) return FLYAI_OK;
  F8RouteParams prm{};
  prm.logits_in = static_cast<const uint16_t*>(logits_in);
  prm.score_fn = d.gating == FLYAI_GATE_SQRTSOFTPLUS ? 1 : 0;
  prm.sorted = d.gating == FLYAI_GATE_SQRTSOFTPLUS ? 1 : 0;
  prm.ue8m0 = is_v4(d) ? 1 : 0;
  prm.tid2eid = tid2eid;
  prm.input_ids = input_ids;
  prm.vocab = vocab;
  prm.err = ws.err;
  prm.x = static_cast<const uint16_t*>(x);
  prm.w = static_cast<const uint16_t*>(w.router_w);
  prm.bias = static_cast<const float*>(w.router_b);
  prm.M = M;
  prm.E = d.num_experts;
  prm.H = d.hidden;
  prm.k = d.top_k;
  prm.n_group = d.n_group;
  prm.topk_group = d.topk_group;
  prm.e0 = d.expert_begin;
  prm.El = d.expert_end - d.expert_begin;
  prm.nsh = d.n_shared;
  prm.scale = d.route_scale;
  prm.logits = ws.logits;
  prm.ids = ws.ids;
  prm.wts = ws.wts;
  prm.out_logits = logits;
  prm.out_ids = topk_ids;
  prm.out_wts = topk_weights;
  prm.xq = ws.xq;
  prm.xs = ws.xs;
  prm.xsf = ws.xsf;
  prm.counts = ws.counts;
  prm.offsets = ws.offsets;
  prm.perm = ws.perm;
  prm.inv = ws.inv;
  prm.n_chunks = ws.n_chunks;
  prm.chunk_info = ws.chunk_info;
  prm.chunk_done = ws.chunk_done;
  prm.ticket = ws.route_ticket;
  const dim3 grid((d.num_experts + kF8RouteExperts - 1) / kF8RouteExperts,
                  (M + kF8RouteTokens - 1) / kF8RouteTokens);
  const cudaError_t st = is_nv4(d) ? f8_launch(f8_route_kernel<true>, grid, kF8RouteThreads, 0, stream, false, prm)
                                   : f8_launch(f8_route_kernel<false>, grid, kF8RouteThreads, 0, stream, false, prm);
  if (st != cudaSuccess) return FLYAI_ERR_CUDA;
  note_launch();
  return FLYAI_OK;
}

// Prefill-size batches: the selection as a launch of its own (one warp per
// token) on the logits ws.logits already holds (nv4_prefill.cu computes them).
__global__ void __launch_bounds__(256) f8_select_kernel(const __grid_constant__ F8RouteParams p) {
  __shared__ __align__(16) KV rows[8 * kF8MaxExperts];
  __shared__ __align__(16) uint8_t tk_s[8][kF8SelScratch];
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, t = blockIdx.x * 8 + warp;
  if (t >= p.M) return;   // whole warps
  if (p.E == 256) f8_select_token_256(p, t, rows + warp * p.E, tk_s[warp]);
  else f8_select_token(p, t, rows + warp * p.E, tk_s[warp]);
}

int launch_fp8_select(const flyai_moe_desc& d, int M, const flyai_moe_weights& w,
                      int32_t* topk_ids, float* topk_weights, const Fp8Workspace& ws,
                      cudaStream_t stream, const void* logits_in) {
  if (M == 0) return FLYAI_OK;
  F8RouteParams prm{};
  prm.logits_in = static_cast<const uint16_t*>(logits_in);
  prm.err = ws.err;
  prm.bias = static_cast<const float*>(w.router_b);
  prm.M = M;
  prm.E = d.num_experts;
  prm.k = d.top_k;
  prm.n_group = d.n_group;
  prm.topk_group = d.topk_group;
  prm.scale = d.route_scale;
  prm.logits = ws.logits;
  prm.ids = ws.ids;
  prm.wts = ws.wts;
  prm.out_ids = topk_ids;
  prm.out_wts = topk_weights;
  if (f8_launch(f8_select_kernel, dim3((M + 7) / 8), 256, 0, stream, true, prm) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  return FLYAI_OK;
}

// ---------------------------------------------------------------------------
// Quantised token rows -> each chunk's B tiles
// ---------------------------------------------------------------------------
struct F8ScatterParams {
  const uint8_t* xq;
  const float* xs;
  const int32_t* perm;
  const int32_t* n_chunks;
  const int4* chunk_info;
  uint8_t* xb;
  int H, k, P;
};

// Byte offset of K element kk (0..127) of token row i inside a B tile.
__host__ __device__ __forceinline__ int f8_btile_offset(int i, int kk) {
  return (kk >> 4) * 256 + (i >> 3) * 128 + (i & 7) * 16 + (kk & 15);
}

// CTA (group of 8 K blocks, chunk): copies the chunk's token rows, 16 bytes per
// thread and step.  Rows past the chunk's token count are left as they are:
// they only feed MMA columns nobody reads.
__global__ void __launch_bounds__(256) f8_scatter_kernel(const __grid_constant__ F8ScatterParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.y;
  if (c >= *p.n_chunks) return;
  const int4 ci = p.chunk_info[c];
  const int KB = p.H / kF8Blk, kb0 = blockIdx.x * 8;
  for (int u = threadIdx.x; u < ci.z * 64; u += blockDim.x) {
    const int i = u >> 6, kb = kb0 + ((u >> 3) & 7), cc = u & 7;
    if (kb >= KB) continue;
    const int pos = ci.y + i;
    const int t = pos < p.P ? __ldg(&p.perm[pos]) / p.k : pos - p.P;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.xq + static_cast<size_t>(t) * p.H +
                                                         kb * kF8Blk + cc * 16));
    uint8_t* tile = p.xb + (static_cast<size_t>(c) * KB + kb) * kF8BBytes;
    *reinterpret_cast<uint4*>(tile + f8_btile_offset(i, cc * 16)) = v;
    if (cc == 0) reinterpret_cast<float*>(tile + kF8BTile)[i] = __ldg(&p.xs[static_cast<size_t>(t) * KB + kb]);
  }
}

// ---------------------------------------------------------------------------
// The expert kernel
// ---------------------------------------------------------------------------
// Work items: (chunk, 128-row block) of gate/up -- a w1 tile and the w3 tile of
// the same rows, K = H -- and of down (w2, K = I).  Each CTA takes one
// contiguous share of the gate/up items and the matching share of the down
// items, gate/up first; a chunk's down items wait until all I/128 of its
// gate/up items stored their quantised SwiGLU tiles (chunk_done).
// One K-step = one 128-wide K block: a bulk copy of the weight block (header +
// tiles) and one of the chunk's B tile (+ 16 activation scales).  The MMA
// writes each K-step into its own TMEM buffer (no accumulation across blocks);
// the epilogue folds buffer kb into fp32 registers with the block's scales,
// acc += D_kb * (s_act[token, kb] * s_w[kb]), so the per-block scaling of
// fp8_gemm is exact in fp32 and the tensor core never sees a scale.
constexpr int kF8Stages = 6;
constexpr int kF8Acc = 8;                 // TMEM buffers (K-steps in flight)
constexpr int kF8AccCols = 2 * kF8Chunk;  // gate 16 + up 16 columns
constexpr int kF8ABytes = kF8Hdr + 2 * kF8Tile;
constexpr int kF8Stage = kF8ABytes + kF8BBytes;
constexpr int kF8Threads = 192;           // warp 0 producer, 1 MMA issuer, 2..5 epilogue
static_assert(kF8Stage % 16 == 0, "stage alignment");
static_assert(kF8Acc * kF8AccCols <= 256, "tensor memory budget");

struct F8Params {
  const uint8_t* w13;
  const uint8_t* w2;
  F8Bank b13, b2;
  const int32_t* n_chunks;
  const int4* chunk_info;
  int32_t* chunk_done;
  const int32_t* perm;
  const float* wts;
  const uint8_t* xb;
  uint8_t* hb;
  uint16_t* rows;
  int H, P;
  float limit;
  int32_t* err;
};

__host__ __device__ inline size_t f8_smem_bytes() {
  return static_cast<size_t>(kF8Stages) * kF8Stage + kF8BTile + 4 * kF8Chunk * 4 +
         (2 * kF8Stages + 2 * kF8Acc + 1) * 8 + 16;
}

__global__ void __launch_bounds__(kF8Threads, 1) f8_moe_kernel(const __grid_constant__ F8Params p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  constexpr int S = kF8Stages;
  uint8_t* ring = sm;
  uint8_t* hst = sm + S * kF8Stage;                          // h tile staging (2 KB)
  float* red = reinterpret_cast<float*>(hst + kF8BTile);     // [4][16] amax partials
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 4 * kF8Chunk);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + kF8Acc;
  uint64_t* epi_done = acc_empty + kF8Acc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 4);   // MMA completion + the four epilogue warps read the scales
    }
    for (int b = 0; b < kF8Acc; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(epi_done, 4);
    mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tmem_slot;
  pdl_wait();   // plan, B tiles and cleared counters are visible
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
    if (warp == 1) tc::tmem_dealloc(tbase, 256);
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
        const F8Bank& B = t.gu ? p.b13 : p.b2;
        const uint8_t* a = (t.gu ? p.w13 : p.w2) + static_cast<size_t>(e) * B.expert +
                           static_cast<size_t>(t.mt) * B.KB * B.block;
        const uint8_t* b = (t.gu ? p.xb : p.hb) + static_cast<size_t>(t.chunk) * B.KB * kF8BBytes;
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
            mbar_expect_tx(&full[s], abytes + kF8BBytes);
            bulk_g2s_hint(ring + s * kF8Stage, a + static_cast<size_t>(kb) * abytes, abytes, &full[s], wpol);
          }
          if (!wait_counter_geq(&p.chunk_done[t.chunk], NI)) ok = false;
          fence_proxy_async_global();
          for (int j = 0; j < kb; ++j) {   // (issued also after a failed wait: the phases complete)
            const uint32_t s = (ks + j) % S;
            bulk_g2s(ring + s * kF8Stage + kF8ABytes, b + static_cast<size_t>(j) * kF8BBytes, kF8BBytes, &full[s]);
          }
          ks += kb;
        }
        for (; ok && kb < B.KB; ++kb, ++ks) {
          const uint32_t s = ks % S, use = ks / S;
          if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], abytes + kF8BBytes);
          bulk_g2s_hint(ring + s * kF8Stage, a + static_cast<size_t>(kb) * abytes, abytes, &full[s], wpol);
          bulk_g2s(ring + s * kF8Stage + kF8ABytes, b + static_cast<size_t>(kb) * kF8BBytes,
                   kF8BBytes, &full[s]);
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
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    bool ok = true;
    uint32_t ks = 0;
    const uint32_t idesc = tc::idesc_f8_e4m3(kF8Chunk);
    const uint64_t a0 = tc::smem_desc_kmajor(ring + kF8Hdr, 2048, 128);
    const uint64_t b0 = tc::smem_desc_kmajor(ring + kF8ABytes, 256, 128);
    // the whole warp walks the items and waits (operands stay warp-uniform); one
    // elected lane issues the tcgen05 ops
    for (; ok && cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const int nk = t.gu ? KB1 : KB2;
      for (int kb = 0; kb < nk; ++kb, ++ks) {
        const uint32_t s = ks % S, buf = ks % kF8Acc;
        ok = mbar_wait_bounded(&full[s], (ks / S) & 1) &&
             (ks < kF8Acc || mbar_wait_bounded(&acc_empty[buf], ((ks / kF8Acc) - 1) & 1));
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc::fence_after_sync();
        const uint32_t st16 = static_cast<uint32_t>((s * kF8Stage) >> 4);
        const uint64_t a = a0 + st16, b = b0 + st16;
        const uint32_t d = tbase + buf * kF8AccCols;
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < 4; ++j)   // K = 32 bytes per MMA: chunks 2j, 2j+1
            tc::mma_f8(d, a + j * (4096 >> 4), b + j * (512 >> 4), idesc, j > 0);
          if (t.gu) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tc::mma_f8(d + kF8Chunk, a + (kF8Tile >> 4) + j * (4096 >> 4), b + j * (512 >> 4),
                         idesc, j > 0);
          }
          tc::commit_to(&empty[s]);
          tc::commit_to(&acc_full[buf]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      // tensor memory goes back only after the epilogue read its last buffer
      if (!mbar_wait_bounded(epi_done, 0)) ok = false;
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 256);
  } else {
    // ---------------- epilogue (TMEM lane quadrant = warp % 4) ----------------
    const int q = warp & 3;
    const int r = 32 * q + lane;   // row of the 128-row block
    bool ok = true;
    uint32_t ks = 0;
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const int4 ci = __ldg(&p.chunk_info[t.chunk]);
      const int pos0 = ci.y, nt = ci.z;
      const int nk = t.gu ? KB1 : KB2;
      float accg[kF8Chunk], accu[kF8Chunk];
#pragma unroll
      for (int i = 0; i < kF8Chunk; ++i) accg[i] = accu[i] = 0.f;
      for (int kb = 0; kb < nk; ++kb, ++ks) {
        const uint32_t s = ks % S, buf = ks % kF8Acc;
        if (ok && !mbar_wait_bounded(&full[s], (ks / S) & 1)) ok = false;
        const uint8_t* st = ring + s * kF8Stage;
        const float4 hdr = *reinterpret_cast<const float4*>(st);
        float sa[kF8Chunk];
#pragma unroll
        for (int i = 0; i < kF8Chunk; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(st + kF8ABytes + kF8BTile + i * 4);
          sa[i] = v.x;
          sa[i + 1] = v.y;
          sa[i + 2] = v.z;
          sa[i + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (ok && !mbar_wait_bounded(&acc_full[buf], (ks / kF8Acc) & 1)) ok = false;
        tc::fence_after_sync();
        uint32_t vg[kF8Chunk], vu[kF8Chunk];
        const uint32_t ta = tbase + buf * kF8AccCols + ((32u * q) << 16);
        tc::tmem_ld16(ta, vg);
        if (t.gu) tc::tmem_ld16(ta + kF8Chunk, vu);
        tc::tmem_wait_ld();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
#pragma unroll
        for (int i = 0; i < kF8Chunk; ++i)
          accg[i] = fmaf(__uint_as_float(vg[i]), __fmul_rn(sa[i], hdr.x), accg[i]);
        if (t.gu) {
#pragma unroll
          for (int i = 0; i < kF8Chunk; ++i)
            accu[i] = fmaf(__uint_as_float(vu[i]), __fmul_rn(sa[i], hdr.y), accu[i]);
        }
      }
      // (after a failed wait the item still runs through the named barriers,
      // which every epilogue warp must reach equally often; its data is void)
      if (t.gu) {
        // SwiGLU row r of the chunk's tokens, then act_quant of the 128-block
        float h[kF8Chunk];
#pragma unroll
        for (int i = 0; i < kF8Chunk; ++i) {
          float g = bf16r(accg[i]), u = bf16r(accu[i]);
          if (p.limit > 0.f) {
            u = fminf(fmaxf(u, -p.limit), p.limit);
            g = fminf(g, p.limit);
          }
          float v = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
          if (i < nt && pos0 + i < p.P) v = __fmul_rn(__ldg(&p.wts[__ldg(&p.perm[pos0 + i])]), v);
          h[i] = i < nt ? bf16r(v) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kF8Chunk; ++i) {
          const float a = warp_max(fabsf(h[i]));
          if (lane == 0) red[q * kF8Chunk + i] = a;
        }
        named_barrier_sync(1, 128);
        float s_mine = 0.f;
#pragma unroll
        for (int i = 0; i < kF8Chunk; ++i) {
          const float a = fmaxf(fmaxf(fmaxf(red[i], red[kF8Chunk + i]),
                                      fmaxf(red[2 * kF8Chunk + i], red[3 * kF8Chunk + i])),
                                1e-4f);
          const float s = __fmul_rn(a, kF8Inv448);
          if (i == (r & (kF8Chunk - 1))) s_mine = s;
          hst[f8_btile_offset(i, r)] = static_cast<uint8_t>(f32_to_e4m3(__fdiv_rn(h[i], s)));
        }
        named_barrier_sync(1, 128);
        uint8_t* tile = p.hb + (static_cast<size_t>(t.chunk) * KB2 + t.mt) * kF8BBytes;
        *reinterpret_cast<uint4*>(tile + r * 16) = *reinterpret_cast<const uint4*>(hst + r * 16);
        if (r < kF8Chunk) reinterpret_cast<float*>(tile + kF8BTile)[r] = s_mine;
        fence_proxy_async_global();
        __threadfence();
        named_barrier_sync(1, 128);
        if (r == 0) atomicAdd(&p.chunk_done[t.chunk], 1);
      } else {
        const int col = t.mt * kF8Blk + r;
#pragma unroll
        for (int i = 0; i < kF8Chunk; ++i) {
          if (i < nt) {   // rows by flat pair index (the shared expert's after the pairs)
            const int pos = pos0 + i, row = pos < p.P ? __ldg(&p.perm[pos]) : pos;
            p.rows[static_cast<size_t>(row) * p.H + col] = float_to_bf16_bits(accg[i]);
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

// ---------------------------------------------------------------------------
// Combine: fp32 sum in ascending expert id, then the shared expert
// ---------------------------------------------------------------------------
struct F8CombineParams {
  const uint16_t* rows;   // [M*k + M*nsh, H] by flat pair index, the shared rows after
  const int32_t* ids;
  uint16_t* y;
  int H, k, P, nsh;
  int fold_bf16;   // round to bf16 after every add (a bf16 index_add), else fp32 sum
};

__global__ void __launch_bounds__(128) f8_combine_kernel(const __grid_constant__ F8CombineParams p) {
  pdl_wait();
  const int t = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (col >= p.H) return;
  int id[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) id[j] = j < p.k ? __ldg(&p.ids[t * p.k + j]) : 0x7fffffff;
  // an expert named by several slots (a hash-routed layer) counts once, with its
  // last slot: the reference's y[idx] += v writes every duplicate back and the
  // last write wins (vendor/deepseek_v4_ref/inference/model.py:641-644)
  uint32_t used = 0;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j)
#pragma unroll
    for (int j2 = j + 1; j2 < kMaxTopK; ++j2)
      if (j2 < p.k && id[j2] == id[j]) used |= 1u << j;
  const int live = p.k - __popc(used);
  // flat pair rows in ascending expert id, then every row's load in flight at once
  int order[kMaxTopK];
#pragma unroll
  for (int r = 0; r < kMaxTopK; ++r) {
    int best = 0, bid = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j)
      if (j < p.k && !((used >> j) & 1u) && id[j] < bid) {
        bid = id[j];
        best = j;
      }
    used |= 1u << best;
    order[r] = r < live ? t * p.k + best : -1;
  }
  uint4 v[kMaxTopK + 1];
#pragma unroll
  for (int r = 0; r < kMaxTopK; ++r)
    v[r] = order[r] >= 0
               ? __ldg(reinterpret_cast<const uint4*>(p.rows + static_cast<size_t>(order[r]) * p.H + col))
               : make_uint4(0u, 0u, 0u, 0u);
  v[kMaxTopK] = p.nsh ? __ldg(reinterpret_cast<const uint4*>(p.rows + static_cast<size_t>(p.P + t) * p.H + col))
                      : make_uint4(0u, 0u, 0u, 0u);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
  for (int r = 0; r <= kMaxTopK; ++r) {
    if (r < kMaxTopK ? order[r] < 0 : !p.nsh) continue;
    const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] = __fadd_rn(acc[2 * i], __uint_as_float(w[i] << 16));
      acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __uint_as_float(w[i] & 0xFFFF0000u));
      if (p.fold_bf16) {
        acc[2 * i] = bf16r(acc[2 * i]);
        acc[2 * i + 1] = bf16r(acc[2 * i + 1]);
      }
    }
  }
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    o[i] = static_cast<uint32_t>(float_to_bf16_bits(acc[2 * i])) |
           (static_cast<uint32_t>(float_to_bf16_bits(acc[2 * i + 1])) << 16);
  *reinterpret_cast<uint4*>(p.y + static_cast<size_t>(t) * p.H + col) = make_uint4(o[0], o[1], o[2], o[3]);
}

int launch_fp8_experts(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                       void* y, uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream,
                       cudaEvent_t ev0, cudaEvent_t ev1) {
  if (M == 0) return FLYAI_OK;
  const int P = M * d.top_k;
  F8ScatterParams sp{ws.xq, ws.xs, ws.perm, ws.n_chunks, ws.chunk_info, ws.xb, d.hidden, d.top_k, P};
  if (f8_launch(f8_scatter_kernel, dim3((d.hidden / kF8Blk + 7) / 8, f8_max_chunks(d, M)), 256, 0,
                stream, true, sp) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();

  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem = f8_smem_bytes();
  if (smem > static_cast<size_t>(max_smem)) return FLYAI_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(f8_moe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  F8Params prm{};
  prm.w13 = static_cast<const uint8_t*>(w.w13);
  prm.w2 = static_cast<const uint8_t*>(w.w2);
  prm.b13 = f8_bank(d.hidden, d.inter, FLYAI_PROJ_W13);
  prm.b2 = f8_bank(d.hidden, d.inter, FLYAI_PROJ_W2);
  prm.n_chunks = ws.n_chunks;
  prm.chunk_info = ws.chunk_info;
  prm.chunk_done = ws.chunk_done;
  prm.perm = ws.perm;
  prm.wts = ws.wts;
  prm.xb = ws.xb;
  prm.hb = ws.hb;
  prm.rows = rows;
  prm.H = d.hidden;
  prm.P = P;
  prm.limit = d.swiglu_limit;
  prm.err = ws.err;
  if (ev0 && ev1 && cudaEventRecord(ev0, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  if (f8_launch(f8_moe_kernel, dim3(sms), kF8Threads, smem, stream, true, prm) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  if (ev0 && ev1 && cudaEventRecord(ev1, stream) != cudaSuccess) return FLYAI_ERR_CUDA;

  return y ? launch_fp8_combine(d, M, rows, y, ws, stream, false) : FLYAI_OK;
}

int launch_fp8_combine(const flyai_moe_desc& d, int M, const uint16_t* rows, void* y,
                       const Fp8Workspace& ws, cudaStream_t stream, bool fold_bf16) {
  if (M == 0) return FLYAI_OK;
  F8CombineParams cp{rows, ws.ids, static_cast<uint16_t*>(y), d.hidden, d.top_k, M * d.top_k,
                     d.n_shared, fold_bf16 ? 1 : 0};
  const dim3 cg(M, (d.hidden / 8 + 127) / 128);
  if (f8_launch(f8_combine_kernel, cg, 128, 0, stream, true, cp) != cudaSuccess) return FLYAI_ERR_CUDA;
  note_launch();
  return FLYAI_OK;
}

}  // namespace flyai
