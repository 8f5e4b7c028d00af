// Verify-size layers whose projections are streamed one 128-wide K block per
// pipeline stage: the DeepSeek-V3-style FP8 layer (FLYAI_FMT_FP8_BLOCK,
// fp8_moe.cu) and the MiniMax-M2.5-style NVFP4 layer (FLYAI_FMT_NVFP4,
// nv4_moe.cu).  Bank and workspace layouts shared by the launchers and kernels.
#pragma once
#include "common.cuh"
#include "nv4.cuh"

namespace flyai {

constexpr int kF8Blk = 128;                      // scale block edge (rows and K)
constexpr int kF8Chunk = 16;                     // tokens of one expert per chunk = MMA N
constexpr int kF8Tile = kF8Blk * kF8Blk;         // 16 KB: one 128x128 e4m3 weight tile
constexpr int kF8Hdr = 16;                       // block header: fp32 weight scale(s)
constexpr int kF8BTile = kF8Chunk * kF8Blk;      // 2 KB: 16 token rows x 128 K, e4m3
constexpr int kF8BBytes = kF8BTile + kF8Chunk * 4;   // + 16 fp32 activation scales
constexpr int kF8MaxTokens = 64;                 // verify-size batches
constexpr int kF8MaxExperts = 512;

// Prefill-size NVFP4 batches (nv4_prefill.cu): more than kF8MaxTokens tokens, up
// to kNvPfMaxTokens.  A chunk holds up to kNpChunk pairs of one expert (the MMA
// N, rounded up to 16); its bf16 rows are stored per 64-wide K slice as the
// canonical K-major operand of that N (16-byte K-chunk c of row i at c*N*16 + i*16):
// token rows as f16 (x / 2^r per row), SwiGLU rows as bf16.
constexpr int kNvPfMaxTokens = 8192;
constexpr int kNpChunk = 128;
constexpr int kNpK = 64;                          // K elements per slice / pipeline stage
constexpr int kNpBlk = kNpChunk * kNpK * 2;       // 16 KB: one slice of a full chunk
__host__ __device__ inline int nvp_max_chunks(int El, int P) {
  return (El < P ? El : P) + P / kNpChunk + 1;
}

// Bank of one projection: per expert, per 128-row output block, per 128-wide K
// block one contiguous "block" = header (fp32 scale of each tile, padded to 16
// bytes) + the tiles (W13: gate tile of w1 then up tile of w3, same rows; W2:
// one tile of w2).  A tile is the canonical no-swizzle K-major operand of
// tcgen05: 16-byte chunk c of row r at c*2048 + (r/8)*128 + (r%8)*16.
struct F8Bank {
  int tiles;        // tiles per block: 2 (W13) or 1 (W2)
  int RB, KB;       // 128-row output blocks, 128-wide K blocks
  size_t block;     // bytes per block
  size_t expert;    // bytes per expert
};
__host__ __device__ inline F8Bank f8_bank(int hidden, int inter, int proj) {
  F8Bank b;
  b.tiles = proj == FLYAI_PROJ_W13 ? 2 : 1;
  b.RB = (proj == FLYAI_PROJ_W13 ? inter : hidden) / kF8Blk;
  b.KB = (proj == FLYAI_PROJ_W13 ? hidden : inter) / kF8Blk;
  b.block = kF8Hdr + static_cast<size_t>(b.tiles) * kF8Tile;
  b.expert = b.block * b.RB * b.KB;
  return b;
}

struct Fp8Workspace {
  int32_t* route_ticket;  // [1 + 64 + 1] at offset 0 (same place as the MXFP4 workspace):
                          // token groups routed, then CTAs finished per token group
  float* logits;          // [M, E] fp32
  int32_t* ids;           // [M*k] expert of each flat pair (descending choice score)
  float* wts;             // [M*k] routing weight of each flat pair
  int32_t* counts;        // [E_local]
  int32_t* offsets;       // [E_local + 1]
  int32_t* perm;          // [M*k] flat pair at each routed position
  int32_t* inv;           // [M*k] routed position of each flat pair (-1: other shard)
  uint8_t* xq;            // FP8: [M, H] e4m3 token rows (act_quant per 1x128)
                          // NVFP4: [M, H/128, kNvRowBytes] e2m1 term rows
  float* xs;              // FP8: [M, H/128] their scales; NVFP4: [M, H/128] factors R
  uint8_t* xsf;           // NVFP4: [M, H/128, kNvRowSf] term scale words
  int32_t* n_chunks;      // [1]
  int4* chunk_info;       // [max_chunks] (bank expert, first position, tokens, 0)
  int32_t* chunk_done;    // [max_chunks] gate/up blocks of the chunk finished
  uint8_t* xb;            // [max_chunks][H/128][B block] quantised token rows
  uint8_t* hb;            // [max_chunks][I/128][B block] quantised SwiGLU rows
  uint8_t* pxb;           // prefill: [chunks][H/64][kNpBlk] bf16 token rows by chunk
  uint8_t* phb;           // prefill: [chunks][I/64][kNpBlk] bf16 SwiGLU rows by chunk
  float* pxr;             // prefill: [M] token row factors R = 2^r (x / R is the f16 operand)
  float* pcr;             // prefill: [chunks][kNpChunk] the factors of each chunk's tokens
  int32_t* pcf;           // prefill: [chunks][kNpChunk] flat pair index of each chunk slot (-1: none)
  float* pcw;             // prefill: [chunks][kNpChunk] its routing weight
  double* plog;           // prefill: [kNpLogitSlices][M, E] fp64 partial router logits
  float* pxm;             // prefill: [kNpLogitSlices][M] partial row maxima of |x|
  uint16_t* rows;         // [M*k + M*n_shared, H] bf16 expert outputs by flat pair index
  int32_t* err;
  int32_t* dbg;
  int max_chunks;
  size_t total;
};

__host__ __device__ inline bool is_nv4(const flyai_moe_desc& d) { return d.format == FLYAI_FMT_NVFP4; }
__host__ __device__ inline int layer_chunk(const flyai_moe_desc& d) { return is_nv4(d) ? kNvChunk : kF8Chunk; }
// bytes of the B block of one chunk and one 128-wide K block (FLYAI_FMT_FP4_W4A8:
// 16 token rows of e4m3 and their 512-byte scale chunk)
__host__ __device__ inline int layer_bblock(const flyai_moe_desc& d) {
  return is_nv4(d) ? kNvBBytes : d.format == FLYAI_FMT_FP4_W4A8 ? kF8BTile + 512 : kF8BBytes;
}

// Chunks a batch of M tokens can need: every non-empty expert rounds its
// count up to a chunk once, plus the shared expert's chunks.
__host__ __device__ inline int f8_max_chunks(const flyai_moe_desc& d, int M) {
  const int El = d.expert_end - d.expert_begin, P = M * d.top_k, C = layer_chunk(d);
  return (El < P ? El : P) + P / C + 1 + d.n_shared * ((M + C - 1) / C);
}

inline Fp8Workspace carve_fp8_workspace(const flyai_moe_desc& d, int M, void* base) {
  Fp8Workspace w{};
  const size_t E = d.num_experts, El = d.expert_end - d.expert_begin, k = d.top_k;
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = base ? static_cast<char*>(base) + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  const size_t P = static_cast<size_t>(M) * k;
  w.route_ticket = reinterpret_cast<int32_t*>(take(4 * (1 + 64 + 1)));
  w.err = reinterpret_cast<int32_t*>(take(4));
  w.dbg = reinterpret_cast<int32_t*>(take(32));
  w.logits = reinterpret_cast<float*>(take(static_cast<size_t>(M) * E * 4));
  w.ids = reinterpret_cast<int32_t*>(take(P * 4));
  w.wts = reinterpret_cast<float*>(take(P * 4));
  w.counts = reinterpret_cast<int32_t*>(take(El * 4));
  w.offsets = reinterpret_cast<int32_t*>(take((El + 1) * 4));
  w.perm = reinterpret_cast<int32_t*>(take(P * 4));
  w.inv = reinterpret_cast<int32_t*>(take(P * 4));
  // verify-size buffers for up to Mv tokens; an NVFP4 layer configured for more
  // tokens also gets the prefill path's chunk buffers
  const int Mv = (is_nv4(d) && M > kF8MaxTokens) ? kF8MaxTokens : M;
  const size_t KB = d.hidden / kF8Blk;
  if (is_nv4(d)) {
    w.xq = reinterpret_cast<uint8_t*>(take(static_cast<size_t>(Mv) * KB * kNvRowBytes));
    w.xsf = reinterpret_cast<uint8_t*>(take(static_cast<size_t>(Mv) * KB * kNvRowSf));
  } else {
    w.xq = reinterpret_cast<uint8_t*>(take(static_cast<size_t>(Mv) * d.hidden));
  }
  w.xs = reinterpret_cast<float*>(take(static_cast<size_t>(Mv) * KB * 4));
  w.n_chunks = reinterpret_cast<int32_t*>(take(4));
  const int vmc = f8_max_chunks(d, Mv);
  const int pmc = Mv < M ? nvp_max_chunks(static_cast<int>(El), M * d.top_k) : 0;
  w.max_chunks = vmc > pmc ? vmc : pmc;
  const size_t mc = static_cast<size_t>(w.max_chunks);
  w.chunk_info = reinterpret_cast<int4*>(take(mc * 16));
  w.chunk_done = reinterpret_cast<int32_t*>(take(mc * 4));
  const size_t bb = layer_bblock(d);
  w.xb = reinterpret_cast<uint8_t*>(take(static_cast<size_t>(vmc) * (d.hidden / kF8Blk) * bb));
  w.hb = reinterpret_cast<uint8_t*>(take(static_cast<size_t>(vmc) * (d.inter / kF8Blk) * bb));
  if (pmc > 0) {
    w.pxb = reinterpret_cast<uint8_t*>(take(static_cast<size_t>(pmc) * (d.hidden / kNpK) * kNpBlk));
    w.phb = reinterpret_cast<uint8_t*>(take(static_cast<size_t>(pmc) * (d.inter / kNpK) * kNpBlk));
    w.pxr = reinterpret_cast<float*>(take(static_cast<size_t>(M) * 4));
    w.pcr = reinterpret_cast<float*>(take(static_cast<size_t>(pmc) * kNpChunk * 4));
    w.pcf = reinterpret_cast<int32_t*>(take(static_cast<size_t>(pmc) * kNpChunk * 4));
    w.pcw = reinterpret_cast<float*>(take(static_cast<size_t>(pmc) * kNpChunk * 4));
    w.plog = reinterpret_cast<double*>(take(static_cast<size_t>(kNpLogitSlices) * M * E * 8));
    w.pxm = reinterpret_cast<float*>(take(static_cast<size_t>(kNpLogitSlices) * M * 4));
  }
  w.rows = reinterpret_cast<uint16_t*>(
      take((P + static_cast<size_t>(M) * d.n_shared) * static_cast<size_t>(d.hidden) * 2));
  w.total = off;
  return w;
}

size_t fp8_packed_bytes(const flyai_moe_desc& d, int proj);
int launch_fp8_pack(const flyai_moe_desc& d, int proj, const void* weight, const void* scale,
                    void* packed, cudaStream_t stream);
// Gate (grouped sigmoid, or the bf16-logit sigmoid gate of FLYAI_GATE_SIGMOID_BF16)
// + token rows quantised (FP8) or split into terms (NVFP4) + routing plan;
// logits/ids/weights outputs may be null.
// tid2eid / input_ids / vocab: a hash-routed layer (FLYAI_GATE_SQRTSOFTPLUS);
// logits_in: bf16 [M, E] logits the caller computed, selected from instead of the
// kernel's own (FLYAI_GATE_SIGMOID_BF16).
int launch_fp8_route(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                     float* logits, int32_t* topk_ids, float* topk_weights,
                     const Fp8Workspace& ws, cudaStream_t stream, const int32_t* tid2eid = nullptr,
                     const int32_t* input_ids = nullptr, int vocab = 0,
                     const void* logits_in = nullptr);
size_t nv4_packed_bytes(const flyai_moe_desc& d, int proj);
int launch_nv4_pack(const flyai_moe_desc& d, int proj, const void* blocks, const void* scales,
                    const void* global_scale, void* packed, cudaStream_t stream, bool swizzled = false);
// Expert projections on the plan flyai_moe_route left in ws: this shard's rows
// (by flat pair index, the shared expert's after the M*k pairs) into `rows`,
// then, when y is not null, the fold of all rows into y.
int launch_nv4_experts(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                       void* y, uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream,
                       cudaEvent_t ev0, cudaEvent_t ev1);
int launch_fp8_experts(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                       void* y, uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream,
                       cudaEvent_t ev0, cudaEvent_t ev1);
// Fold of the pair rows (every shard's) into y: fp32 in ascending expert id then
// the shared expert (FP8), or bf16 after every add (NVFP4, fold_bf16).
int launch_fp8_combine(const flyai_moe_desc& d, int M, const uint16_t* rows, void* y,
                       const Fp8Workspace& ws, cudaStream_t stream, bool fold_bf16);
// Selection alone (f8_route_kernel's per-token step) on the logits in ws.logits.
int launch_fp8_select(const flyai_moe_desc& d, int M, const flyai_moe_weights& w,
                      int32_t* topk_ids, float* topk_weights, const Fp8Workspace& ws,
                      cudaStream_t stream, const void* logits_in = nullptr);
// NVFP4 prefill (M > kF8MaxTokens): router logits, selection, plan of kNpChunk-pair
// chunks and the chunks' bf16 token rows; then the expert kernel (and the fold
// into y when y is not null).
// Prefill router logits (nv4_prefill.cu): fp64 partial dot products of
// kLgTok-token x kLgExp-expert tiles over kNpLogitSlices K slices -- part
// [slice][M][E] -- and the slices' |x| row maxima.  Grid (ceil(E/kLgExp),
// ceil(M/kLgTok), kNpLogitSlices) x 256 threads; H a multiple of 32.
constexpr int kLgTok = 64, kLgExp = 128;
__global__ void nvp_logits_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, int M,
                                  int E, int H, double* __restrict__ part, float* __restrict__ xmax_part);

int launch_nvp_route(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                     float* logits, int32_t* topk_ids, float* topk_weights,
                     const Fp8Workspace& ws, cudaStream_t stream, const void* logits_in = nullptr);
int launch_nvp_experts(const flyai_moe_desc& d, int M, const flyai_moe_weights& w, void* y,
                       uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream,
                       cudaEvent_t ev0, cudaEvent_t ev1);
// DeepSeek-V4 W4A8 layer (v4_moe.cu): bank sizes and packing (routed experts
// e2m1 + e8m0/32; the shared expert e4m3 + e8m0 per 128x128), and the expert
// kernels on the plan the route left in ws (then the fold into y when y is set).
size_t v4_packed_bytes(const flyai_moe_desc& d, int proj);
int launch_v4_pack_fp4(const flyai_moe_desc& d, int proj, const void* blocks, const void* scales,
                       void* packed, cudaStream_t stream);
int launch_v4_pack_shared(const flyai_moe_desc& d, int proj, const void* weight, const void* scale,
                          void* packed, cudaStream_t stream);
// slot_of != null: the bank is an expert cache of `slots` routed experts then the
// shared expert; routed expert e (local index) sits in slot slot_of[e].
int launch_v4_experts(const flyai_moe_desc& d, int M, const flyai_moe_weights& w, void* y,
                      uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream, cudaEvent_t ev0,
                      cudaEvent_t ev1, const int32_t* slot_of = nullptr, int slots = 0);
// Rows of the pair-row buffer of a batch of M tokens.
inline size_t layer_pair_rows(const flyai_moe_desc& d, int M) {
  return static_cast<size_t>(M) * (d.top_k + d.n_shared);
}

}  // namespace flyai
