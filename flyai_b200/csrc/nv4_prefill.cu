// MiniMax-M2.5-style NVFP4 layer for prefill-size batches (more than 64
// tokens) on sm_100a.
//
// Same arithmetic as nv4_moe.cu (HF transformers' MiniMaxM2 modules on NVFP4
// weights, which the M2.5 stage's vLLM FusedMoE configuration mirrors:
// engines/minimax_m25/m25_stage.py:288-311, 412-416), arranged for many tokens
// per expert.  At verify sizes the layer is weight-bandwidth bound and the
// activations go through the e2m1 MMA as six terms; with hundreds of tokens per
// expert the MMA work dominates and a 16-bit form is cheaper: an NVFP4 weight
// without its global scale (e2m1 x e4m3: at most 6 significant bits, magnitudes
// 2^-10 .. 2688) is exact in f16 and in bf16, so the weights are expanded in
// shared memory and multiplied on tcgen05 kind::f16 (fp32 accumulate); the
// global scales are applied in the epilogue.
//   gate/up: f16 weights (one cvt + one multiply per pair) against the token
//            rows as f16 after dividing each row by R = 2^r, r chosen so the
//            row maximum lands in [2^14, 2^15): every element down to 2^-32 of
//            the row maximum keeps all its bits (smaller ones are rounded to
//            f16 subnormals, a change below 2^-40 of the maximum); the epilogue
//            multiplies by R;
//   down:    bf16 weights against the SwiGLU rows in bf16 (their range is not
//            known per row in advance), exact products.
//
// Launches (PDL-chained): nvp_logits_kernel + nvp_logits_sum_kernel (router
// logits as fp64 sums over K slices added in a fixed order, rounded once to fp32
// and to bf16 as the verify route does; token row maxima), f8_select_kernel (the
// verify path's per-token selection), nvp_plan_kernel (pairs by expert, chunks of
// up to kNpChunk pairs), nvp_scatter_kernel (each chunk's f16 token rows in
// operand layout, per-slot row factor, flat pair index and routing weight),
// nvp_moe_kernel (gate/up + SwiGLU + down; items dealt to CTAs strided),
// f8_combine_kernel (bf16 fold in ascending expert id).
//
// nvp_moe_kernel, one persistent CTA per SM, 704 threads:
//   warp 0      producer: bulk copies of one NVFP4 bank block (128 rows x 128 K,
//               both tiles of gate/up) into a raw ring of 4 and, per 64-wide K
//               slice, the chunk's rows into a row ring of 5 (each ring deep
//               enough to cover a copy's latency on its own);
//   warp 1      MMA issuer: 4 (down) or 8 (gate/up) kind::f16 MMAs per stage
//               into one of two 256-column TMEM slots (gate at +0, up at +128);
//   warps 2..5  epilogue: gate/up -> SwiGLU rows straight into the chunk's
//               operand layout for the down items (chunk_done counts them);
//               down -> weighted bf16 rows by flat pair index;
//   warps 6..21 expansion: raw block -> two 16-bit stages of the weight operand
//               (a ring of 2; one group of 8 warps per K half).
// Items (chunk, 128-row block) and their order are the verify kernels'.  Every
// wait is bounded (~2 s) and records kErrWaitTimeout.
#include <cuda_fp8.h>
#include <math.h>

#include "common.cuh"
#include "fp8_moe.cuh"
#include "nv4.cuh"
#include "tc_bank.cuh"
#include "tcgen05.cuh"

namespace flyai {

template <typename Kern, typename... Args>
static cudaError_t np_launch(Kern kernel, dim3 grid, int block, size_t smem, cudaStream_t s,
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
// Router logits in fp64: CTA (64-token tile, 128-expert tile, K slice); each
// thread keeps 8 tokens x 4 experts of fp64 sums (bf16 -> fp64 is exact, and so
// is every product), K staged in steps of 32 as fp64 in shared memory ([k][token]
// read as broadcasts, [k][expert] one value per lane).  The kLgSlices partial
// sums of a logit are added in a fixed order by nvp_logits_sum_kernel, so the
// result is the exact dot product to fp64 rounding -- the value the verify route
// kernel computes -- rounded once to fp32 and once to bf16.  The same pass takes
// each token row's |x| maximum for the f16 row factor.
// ---------------------------------------------------------------------------
constexpr int kLgK = 32, kLgSlices = kNpLogitSlices;

__global__ void __launch_bounds__(256) nvp_logits_kernel(const uint16_t* __restrict__ x,
                                                         const uint16_t* __restrict__ w, int M,
                                                         int E, int H,
                                                         double* __restrict__ part,
                                                         float* __restrict__ xmax_part) {
  __shared__ double xs[kLgK][kLgTok];   // [k][token]
  __shared__ double ws[kLgK][kLgExp];   // [k][expert]
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * kLgExp, t0 = blockIdx.y * kLgTok, sl = blockIdx.z;
  // slices of whole 32-wide steps (H is a multiple of 128); trailing ones may be empty
  const int kspan = (H + kLgSlices * kLgK - 1) / (kLgSlices * kLgK) * kLgK;
  const int kbeg = sl * kspan, kend = min(H, kbeg + kspan);
  double acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
  float xm = 0.f;   // |x| maximum of this thread's share of its token row and slice
  for (int k0 = kbeg; k0 < kend; k0 += kLgK) {
    __syncthreads();   // the previous step's tiles are consumed
    {   // x: 64 tokens x 32 K, 8 per thread (token tid/4, K quarter tid%4)
      const int i = threadIdx.x >> 2, kk = (threadIdx.x & 3) * 8, t = t0 + i;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (t < M) v = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H + k0 + kk));
      const uint32_t r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a0 = __uint_as_float(r[q] << 16), a1 = __uint_as_float(r[q] & 0xFFFF0000u);
        xs[kk + 2 * q][i] = a0;
        xs[kk + 2 * q + 1][i] = a1;
        xm = fmaxf(xm, fmaxf(fabsf(a0), fabsf(a1)));
      }
    }
    {   // w: 128 experts x 32 K, 16 per thread (expert tid/2, K half tid%2)
      const int j = threadIdx.x >> 1, kk = (threadIdx.x & 1) * 16, e = e0 + j;
      uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
      if (e < E) {
        const uint4* src = reinterpret_cast<const uint4*>(w + static_cast<size_t>(e) * H + k0 + kk);
        a = ldg_nc_v4(src);
        b = ldg_nc_v4(src + 1);
      }
      const uint32_t r[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        ws[kk + 2 * q][j] = __uint_as_float(r[q] << 16);
        ws[kk + 2 * q + 1][j] = __uint_as_float(r[q] & 0xFFFF0000u);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < kLgK; ++kk) {
      double xv[8], wv[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] = xs[kk][warp * 8 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[j] = ws[kk][lane + 32 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(xv[i], wv[j], acc[i][j]);
    }
  }
  if (blockIdx.x == 0) {   // the slice's |x| maximum per token
    xm = fmaxf(xm, __shfl_xor_sync(0xffffffffu, xm, 1));
    xm = fmaxf(xm, __shfl_xor_sync(0xffffffffu, xm, 2));
    const int t = t0 + (threadIdx.x >> 2);
    if ((threadIdx.x & 3) == 0 && t < M) xmax_part[static_cast<size_t>(sl) * M + t] = xm;
  }
  double* dst = part + static_cast<size_t>(sl) * M * E;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = t0 + warp * 8 + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + lane + 32 * j;
      if (t < M && e < E) dst[static_cast<size_t>(t) * E + e] = acc[i][j];
    }
  }
}

// Logit = the slices' partial sums in slice order, rounded to fp32 then bf16;
// token row factor R = 2^r with max|x| / R in [2^14, 2^15).
__global__ void __launch_bounds__(256) nvp_logits_sum_kernel(const double* __restrict__ part,
                                                             const float* __restrict__ xmax_part,
                                                             int M, int E, float* __restrict__ logits,
                                                             float* __restrict__ out_logits,
                                                             float* __restrict__ xr) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t n = static_cast<size_t>(M) * E;
  for (size_t u = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; u < n;
       u += static_cast<size_t>(gridDim.x) * blockDim.x) {
    double a = part[u];
#pragma unroll
    for (int s = 1; s < kLgSlices; ++s) a += part[s * n + u];
    const float v = bf16r(__double2float_rn(a));
    logits[u] = v;
    if (out_logits) out_logits[u] = v;
    if (u < static_cast<size_t>(M)) {
      float m = 0.f;
#pragma unroll
      for (int s = 0; s < kLgSlices; ++s) m = fmaxf(m, xmax_part[s * static_cast<size_t>(M) + u]);
      int r = 0;
      if (m > 0.f && isfinite(m)) {
        int ex;
        frexpf(m, &ex);   // m = f * 2^ex, f in [0.5, 1)
        r = max(-110, min(110, ex - 15));
      }
      xr[u] = exp2i(r);
    }
  }
}

// ---------------------------------------------------------------------------
// Plan, one CTA of 1024 threads: per-warp expert histograms over 32 contiguous
// segments of the flat pairs, exclusive bases, block scans over experts, then
// each warp ranks its segment in flat order (match_any per 32 pairs): pairs by
// ascending local expert, ascending flat index inside one -- the verify plan's
// order -- cut into chunks of up to kNpChunk pairs.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

__device__ int np_block_scan(int v, int* tmp, int* total) {
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

struct NpPlanParams {
  const int32_t* ids;
  int P, e0, El, max_chunks;
  int32_t* counts;
  int32_t* offsets;
  int32_t* perm;
  int32_t* inv;
  int32_t* n_chunks;
  int4* chunk_info;
  int32_t* chunk_done;
};

__host__ __device__ inline size_t np_plan_smem(int El) {
  return (32ull * El + 2ull * El + 1 + 33) * 4;
}

__global__ void __launch_bounds__(kPlanThreads) nvp_plan_kernel(const __grid_constant__ NpPlanParams p) {
  extern __shared__ int32_t psm[];
  const int El = p.El, P = p.P;
  int32_t* hist = psm;            // [32][El]: pairs of expert el in warp w's segment, then bases
  int32_t* off = hist + 32 * El;  // [El] first position of each expert
  int32_t* cnt = off + El;        // [El + 1]
  int* tmp = cnt + El + 1;        // [33]
  pdl_wait();
  pdl_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < 32 * El; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int p0 = static_cast<int>(static_cast<long long>(P) * warp / 32);
  const int p1 = static_cast<int>(static_cast<long long>(P) * (warp + 1) / 32);
  for (int q = p0 + lane; q < p1; q += 32) {
    const int el = __ldg(&p.ids[q]) - p.e0;
    if (el >= 0 && el < El) atomicAdd(&hist[warp * El + el], 1);
  }
  __syncthreads();
  for (int e = tid; e < El; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = hist[w * El + e];
      hist[w * El + e] = run;
      run += c;
    }
    cnt[e] = run;
  }
  __syncthreads();
  // El <= 1024: thread e owns expert e in the scans
  const int c_e = tid < El ? cnt[tid] : 0;
  const int nch_e = (c_e + kNpChunk - 1) / kNpChunk;
  int pairs = 0, chunks = 0;
  const int o_e = np_block_scan(c_e, tmp, &pairs);
  const int cb_e = np_block_scan(nch_e, tmp, &chunks);
  const int nch = chunks < p.max_chunks ? chunks : p.max_chunks;
  if (tid < El) {
    off[tid] = o_e;
    p.counts[tid] = c_e;
    p.offsets[tid] = o_e;
    for (int j = 0; j < nch_e; ++j)
      if (cb_e + j < nch)
        p.chunk_info[cb_e + j] = make_int4(tid, o_e + j * kNpChunk, min(kNpChunk, c_e - j * kNpChunk), 0);
  }
  for (int c = tid; c < nch; c += blockDim.x) p.chunk_done[c] = 0;
  if (tid == 0) {
    p.offsets[El] = pairs;
    *p.n_chunks = nch;
  }
  __syncthreads();
  for (int b = p0; b < p1; b += 32) {   // stable permutation
    const int q = b + lane;
    int el = -2;
    if (q < p1) {
      el = __ldg(&p.ids[q]) - p.e0;
      if (el < 0 || el >= El) el = -1;
    }
    const uint32_t same = __match_any_sync(0xffffffffu, el);
    const int rank = __popc(same & ((1u << lane) - 1u));
    const int base = el >= 0 ? hist[warp * El + el] : 0;
    if (el >= 0) {
      const int pos = off[el] + base + rank;
      p.perm[pos] = q;
      p.inv[q] = pos;
    } else if (el == -1) {
      p.inv[q] = -1;
    }
    __syncwarp();
    if (el >= 0 && rank == 0) hist[warp * El + el] = base + __popc(same);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Token rows -> each chunk's K slices in operand layout, as f16 after dividing by
// the row factor R; per chunk slot the factor (cr), flat pair index (cf) and
// routing weight (cw) for the epilogues.  CTA (group of 8 slices,
// chunk); token slots from the chunk's count up to N (a multiple of 16) are zero.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) nvp_scatter_kernel(const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ perm,
                                                          const int32_t* __restrict__ n_chunks,
                                                          const int4* __restrict__ chunk_info,
                                                          const float* __restrict__ xr,
                                                          const float* __restrict__ wts,
                                                          uint8_t* __restrict__ xb,
                                                          float* __restrict__ cr,
                                                          int32_t* __restrict__ cf,
                                                          float* __restrict__ cw, int H, int k) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.y;
  if (c >= *n_chunks) return;
  const int4 ci = chunk_info[c];
  const int nt = ci.z, np = (nt + 15) & ~15, KS = H / kNpK, ks0 = blockIdx.x * 8;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < np; i += blockDim.x) {
      const int flat = i < nt ? __ldg(&perm[ci.y + i]) : -1;
      const size_t o = static_cast<size_t>(c) * kNpChunk + i;
      cr[o] = flat >= 0 ? __ldg(&xr[flat / k]) : 1.f;
      cf[o] = flat;
      cw[o] = flat >= 0 ? __ldg(&wts[flat]) : 0.f;
    }
  const int units = 8 * np * 8;   // (slice, token slot, 16-byte piece)
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int q = u & 7, i = (u >> 3) % np, ks = ks0 + (u >> 3) / np;
    if (ks >= KS) continue;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (i < nt) {
      const int tok = __ldg(&perm[ci.y + i]) / k;
      const float rinv = __frcp_rn(__ldg(&xr[tok]));   // a power of two: exact
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(tok) * H + ks * kNpK + q * 8));
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
      uint32_t hw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 h = __floats2half2_rn(__fmul_rn(__uint_as_float(bw[j] << 16), rinv),
                                            __fmul_rn(__uint_as_float(bw[j] & 0xFFFF0000u), rinv));
        hw[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      v = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
    *reinterpret_cast<uint4*>(xb + (static_cast<size_t>(c) * KS + ks) * kNpBlk + q * (np * 16) + i * 16) = v;
  }
}

// ---------------------------------------------------------------------------
// The expert kernel
// ---------------------------------------------------------------------------
constexpr int kNpAStages = 2;    // expanded weight stages
constexpr int kNpBStages = 5;    // token / SwiGLU row stages
constexpr int kNpRaw = 4;        // raw NVFP4 blocks (two stages each)
constexpr int kNpRawBytes = 2 * kNvTileBytes;    // 18432: one bank block (K = 128), gate/up
constexpr int kNpATile = 128 * kNpK * 2;         // 16 KB: 128 weight rows x 64 K, 16-bit
constexpr int kNpAStage = 2 * kNpATile;          // gate and up tiles
constexpr int kNpDqWarps = 16;
constexpr int kNpDqThreads = kNpDqWarps * 32;
constexpr int kNpThreads = (6 + kNpDqWarps) * 32;
constexpr int kNpSlotCols = 256;
constexpr int kNpOffA = kNpRaw * kNpRawBytes;
constexpr int kNpOffB = kNpOffA + kNpAStages * kNpAStage;
constexpr int kNpOffBar = kNpOffB + kNpBStages * kNpBlk;
static_assert(kNpOffA % 1024 == 0 && kNpOffB % 1024 == 0, "stage alignment");
static_assert(kNpDqThreads == 2 * 2 * 128, "two groups x (row, 32-weight chunk) per thread");
static_assert(2 * kNpSlotCols <= 512, "tensor memory budget");

__host__ __device__ inline size_t np_smem_bytes() {
  return kNpOffBar + (2 * kNpRaw + 2 * kNpAStages + 2 * kNpBStages + 2 * 2 + 1) * 8 + 16;
}

struct NpParams {
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
  const float* cr;    // [chunks][kNpChunk] token row factors
  const int32_t* cf;  // [chunks][kNpChunk] flat pair index of each slot
  const float* cw;    // [chunks][kNpChunk] routing weight of each slot
  uint16_t* rows;
  int H, I;
  int32_t* err;
};

// e4m3 scale byte -> bf16x2 {s * 2^112, s * 2^112} (exact: 4 significant bits,
// every e4m3 value times 2^112 is a normal bf16).
__device__ __forceinline__ uint32_t np_scale_pair(uint32_t s) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(s & 0xFFu), __NV_E4M3);
  const float v = __fmul_rn(__half2float(__half(h)), exp2i(112));
  const uint32_t b = float_to_bf16_bits(v);
  return b | (b << 16);
}

// Eight e2m1 weights (a 32-bit word, element 0 in the low nibble) times their
// block scale -> four bf16x2 words.  An f16 e2m1 value shifted right by 3 is the
// bf16 of that value times 2^-112 (zeros stay zero); the bf16 product with
// s * 2^112 is then exact and normal.
__device__ __forceinline__ void np_expand8(uint32_t w, uint32_t sc, uint32_t (&o)[4]) {
  uint32_t f[4];
  e2m1x8_to_f16x8(w, f[0], f[1], f[2], f[3]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t b = ((f[i] >> 3) & 0x0FFF0FFFu) | (f[i] & 0x80008000u);
    __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&b),
                               *reinterpret_cast<const __nv_bfloat162*>(&sc));
    o[i] = *reinterpret_cast<uint32_t*>(&r);
  }
}

// The scale word of row r for one 64-wide K half of a raw tile: four e4m3 block
// scales (blocks of 16 along K), from the tcgen05 scale-factor layout.
__device__ __forceinline__ uint32_t np_scale_word(const uint8_t* tile, int half, int r) {
  const uint4 line = lds128(tile + kNvTile + half * kNvSfChunk + (r & 31) * 16);
  const int qd = r >> 5;
  return qd == 0 ? line.x : qd == 1 ? line.y : qd == 2 ? line.z : line.w;
}

// Gate/up (f16): row r, 16-byte raw chunk cc of the half (32 weights, scale
// blocks 2cc and 2cc+1) -> four 16-byte units of the f16 tile (K-chunk c of row r
// at c*2048 + r*16).  e2m1 -> f16 and e4m3 -> f16 are hardware conversions; the
// f16 product is exact.
__device__ __forceinline__ void np_expand_f16(const uint8_t* tile, uint8_t* dst, int half, int r,
                                              int cc) {
  const uint4 q = lds128(tile + (2 * half + cc) * 2048 + r * 16);
  const uint32_t sw = np_scale_word(tile, half, r) >> (16 * cc);
  const __half2_raw s01 = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(sw & 0xFFFFu), __NV_E4M3);
  const uint32_t sp = static_cast<uint32_t>(s01.x) | (static_cast<uint32_t>(s01.y) << 16);
  const uint32_t s0 = __byte_perm(sp, 0u, 0x1010), s1 = __byte_perm(sp, 0u, 0x3232);
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t f[4];
    e2m1x8_to_f16x8(words[j], f[0], f[1], f[2], f[3]);
    const uint32_t sc = j < 2 ? s0 : s1;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 r2 = __hmul2(*reinterpret_cast<const __half2*>(&f[i]),
                                 *reinterpret_cast<const __half2*>(&sc));
      f[i] = *reinterpret_cast<const uint32_t*>(&r2);
    }
    *reinterpret_cast<uint4*>(dst + (cc * 4 + j) * 2048 + r * 16) = make_uint4(f[0], f[1], f[2], f[3]);
  }
}

// Down (bf16): row r, 8-byte half sub of raw chunk cc (16 weights, scale block
// 2cc + sub) -> two 16-byte units of the bf16 tile.
__device__ __forceinline__ void np_expand_bf16(const uint8_t* tile, uint8_t* dst, int half, int r,
                                               int cc, int sub) {
  const uint2 q = *reinterpret_cast<const uint2*>(tile + (2 * half + cc) * 2048 + r * 16 + sub * 8);
  const uint32_t sc = np_scale_pair(np_scale_word(tile, half, r) >> (8 * (2 * cc + sub)));
  const uint32_t words[2] = {q.x, q.y};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint32_t o[4];
    np_expand8(words[j], sc, o);
    *reinterpret_cast<uint4*>(dst + (cc * 4 + sub * 2 + j) * 2048 + r * 16) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(kNpThreads, 1) nvp_moe_kernel(const __grid_constant__ NpParams p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  constexpr int SA = kNpAStages, SB = kNpBStages, R = kNpRaw;
  uint8_t* raw = sm;
  uint8_t* sa = sm + kNpOffA;
  uint8_t* sb = sm + kNpOffB;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(sm + kNpOffBar);
  uint64_t* raw_empty = raw_full + R;   // the expansion warps are done with the block
  uint64_t* a_full = raw_empty + R;     // the expansion warps wrote the stage
  uint64_t* a_empty = a_full + SA;      // the stage's MMAs completed
  uint64_t* b_full = a_empty + SA;      // the producer's bytes landed
  uint64_t* b_empty = b_full + SB;      // the stage's MMAs completed
  uint64_t* acc_full = b_empty + SB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* epi_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int r = 0; r < R; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], kNpDqWarps);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], kNpDqWarps / 2);   // the slot's expansion group
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
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

  const int NI = p.b13.RB, NT = p.b2.RB, KB1 = p.b13.KB, KB2 = p.b2.KB;
  const int KS1 = p.H / kNpK, KS2 = p.I / kNpK;
  TcStridedCursor cur;   // concurrent CTAs share a chunk's rows and an expert's weights in L2
  cur.start(blockIdx.x, gridDim.x, *p.n_chunks, NI, NT);
  if (!cur.valid()) {
    if (warp == 1) tc::tmem_dealloc(tbase, 512);
    return;
  }

  if (warp == 0) {
    // ---------------- producer ----------------
    bool ok = true;
    uint32_t rr = 0, ks = 0;
    for (; cur.valid(); cur.next()) {
      if (lane == 0 && ok) {
        const TcItem t = cur.t;
        const int4 ci = __ldg(&p.chunk_info[t.chunk]);
        const int np = (ci.z + 15) & ~15;
        const NvBank& B = t.gu ? p.b13 : p.b2;
        const uint8_t* a = (t.gu ? p.w13 : p.w2) + static_cast<size_t>(ci.x) * B.expert +
                           static_cast<size_t>(t.mt) * B.KB * B.block;
        const uint8_t* b = (t.gu ? p.xb : p.hb) + static_cast<size_t>(t.chunk) * (t.gu ? KS1 : KS2) * kNpBlk;
        const uint32_t abytes = static_cast<uint32_t>(B.block), bbytes = static_cast<uint32_t>(np) * 128u;
        bool dep = !t.gu;   // down: the chunk's SwiGLU rows come from its gate/up items
        for (int kb = 0; ok && kb < B.KB; ++kb, ++rr) {
          const uint32_t r = rr % R;
          if (rr >= R && !mbar_wait_bounded(&raw_empty[r], ((rr / R) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&raw_full[r], abytes);
          bulk_g2s(raw + r * kNpRawBytes, a + static_cast<size_t>(kb) * abytes, abytes, &raw_full[r]);
          if (dep) {   // (the first weight block is already on its way)
            if (!wait_counter_geq(&p.chunk_done[t.chunk], NI)) ok = false;
            fence_proxy_async_global();
            dep = false;
          }
          for (int h = 0; ok && h < 2; ++h, ++ks) {
            const uint32_t s = ks % SB;
            if (ks >= SB && !mbar_wait_bounded(&b_empty[s], ((ks / SB) - 1) & 1)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&b_full[s], bbytes);
            bulk_g2s(sb + s * kNpBlk, b + static_cast<size_t>(2 * kb + h) * kNpBlk, bbytes, &b_full[s]);
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
      for (uint32_t s = 0; s < SB && s < ks; ++s) {
        const uint32_t last = ((ks - 1 - s) / SB) * SB + s;
        if (!mbar_wait_bounded(&b_full[s], (last / SB) & 1)) ok = false;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp walks the items and waits (operands stay warp-uniform); one
    // elected lane issues the tcgen05 instructions.
    bool ok = true;
    uint32_t ks = 0, item = 0;
    for (; ok && cur.valid(); cur.next(), ++item) {
      const TcItem t = cur.t;
      const int np = (__ldg(&p.chunk_info[t.chunk].z) + 15) & ~15;
      const uint32_t idesc = t.gu ? tc::idesc_f16(np) : tc::idesc_bf16(np);
      const int nsteps = 2 * (t.gu ? KB1 : KB2);
      const uint32_t slot = item & 1u;
      if (item >= 2) ok = mbar_wait_bounded(&acc_empty[slot], ((item >> 1) - 1) & 1);
      ok = __all_sync(0xffffffffu, ok);
      tc::fence_after_sync();
      const uint32_t d = tbase + slot * kNpSlotCols;
      const uint64_t a0 = tc::smem_desc_kmajor(sa, 2048, 128);
      const uint64_t b0 = tc::smem_desc_kmajor(sb, static_cast<uint32_t>(np) * 16, 128);
      const uint32_t bstep = static_cast<uint32_t>(np) * 2;   // 2 K-chunks of N rows, in 16 B
      for (int st = 0; ok && st < nsteps; ++st, ++ks) {
        const uint32_t s = ks % SA, u = ks % SB;
        ok = mbar_wait_bounded(&a_full[s], (ks / SA) & 1) && mbar_wait_bounded(&b_full[u], (ks / SB) & 1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc::fence_after_sync();
        const uint64_t as = a0 + ((s * kNpAStage) >> 4), bs = b0 + ((u * kNpBlk) >> 4);
        if (elect_one()) {
#pragma unroll
          for (int i = 0; i < 4; ++i)   // K = 16 per MMA: K-chunks 2i, 2i+1
            tc::mma_kf16(d, as + ((i * 2 * 2048) >> 4), bs + i * bstep, idesc, st > 0 || i > 0);
          if (t.gu) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              tc::mma_kf16(d + 128, as + ((kNpATile + i * 2 * 2048) >> 4), bs + i * bstep, idesc,
                           st > 0 || i > 0);
          }
          tc::commit_to(&a_empty[s]);
          tc::commit_to(&b_empty[u]);
        }
        __syncwarp();
      }
      if (ok && elect_one()) tc::commit_to(&acc_full[slot]);
      __syncwarp();
    }
    if (lane == 0) {
      if (!mbar_wait_bounded(epi_done, 0)) ok = false;   // last accumulator read
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  } else if (warp < 6) {
    // ---------------- epilogue (TMEM lane quadrant = warp % 4) ----------------
    const int q = warp & 3, r = 32 * q + lane;
    bool ok = true;
    uint32_t item = 0;
    for (; cur.valid(); cur.next(), ++item) {
      const TcItem t = cur.t;
      const int4 ci = __ldg(&p.chunk_info[t.chunk]);
      const int e = ci.x, nt = ci.z, np = (nt + 15) & ~15;
      const uint32_t slot = item & 1u;
      if (ok && !mbar_wait_bounded(&acc_full[slot], (item >> 1) & 1)) ok = false;
      tc::fence_after_sync();
      const uint32_t ta = tbase + slot * kNpSlotCols + ((32u * q) << 16);
      if (t.gu) {
        // SwiGLU element (token i, feature mt*128 + r) -> down operand, slice mt*2 + r/64
        const float g1 = __ldg(&p.g13[2 * e]), g3 = __ldg(&p.g13[2 * e + 1]);
        const float* crow = p.cr + static_cast<size_t>(t.chunk) * kNpChunk;
        uint8_t* hrow = p.hb + (static_cast<size_t>(t.chunk) * KS2 + t.mt * 2 + (r >> 6)) * kNpBlk +
                        ((r & 63) >> 3) * (np * 16) + (r & 7) * 2;
        for (int c0 = 0; c0 < np; c0 += 16) {
          uint32_t gv[16], uv[16];
          tc::tmem_ld16(ta + c0, gv);
          tc::tmem_ld16(ta + 128 + c0, uv);
          float R[16];
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(crow + c0 + j));
            R[j] = f.x, R[j + 1] = f.y, R[j + 2] = f.z, R[j + 3] = f.w;
          }
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int i = c0 + j;   // R is a power of two: acc * R is exact
            const float gate = bf16r(__fmul_rn(__fmul_rn(__uint_as_float(gv[j]), R[j]), g1));
            const float up = bf16r(__fmul_rn(__fmul_rn(__uint_as_float(uv[j]), R[j]), g3));
            const float sg = bf16r(__fdiv_rn(gate, __fadd_rn(1.f, expf(-gate))));
            const float h = i < nt ? bf16r(__fmul_rn(sg, up)) : 0.f;
            *reinterpret_cast<uint16_t*>(hrow + i * 16) = float_to_bf16_bits(h);
          }
        }
      } else {
        const float g2 = __ldg(&p.g2[e]);
        const int col = t.mt * 128 + r;
        const int32_t* cfl = p.cf + static_cast<size_t>(t.chunk) * kNpChunk;
        const float* cwt = p.cw + static_cast<size_t>(t.chunk) * kNpChunk;
        for (int c0 = 0; c0 < np; c0 += 16) {
          uint32_t v[16];
          tc::tmem_ld16(ta + c0, v);
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
            if (c0 + j < nt) {   // rows by flat pair index
              const float o = bf16r(__fmul_rn(__uint_as_float(v[j]), g2));
              p.rows[static_cast<size_t>(fl[j]) * p.H + col] = float_to_bf16_bits(__fmul_rn(o, wt[j]));
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
        if (r == 0) atomicAdd(&p.chunk_done[t.chunk], 1);
      }
    }
    if (!ok) atomicOr(p.err, kErrWaitTimeout);
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(epi_done);
  } else {
    // ---------------- weight expansion ----------------
    // Two groups of 8 warps, one per 64-wide K half of every raw block: group g
    // writes stage 2*rr + g, always into A slot g, so each group has two stage
    // times per stage.  A thread expands two 32-weight units per stage: both
    // tiles of (row, chunk) for gate/up, both 16-weight halves for down.
    static_assert(kNpAStages == 2, "one A slot per expansion group");
    const int et = threadIdx.x - 6 * 32;   // 0..kNpDqThreads-1
    const int grp = et >> 8, row = et & 127, cc = (et >> 7) & 1;
    bool ok = true;
    uint32_t rr = 0;
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const int nk = t.gu ? KB1 : KB2;
      for (int kb = 0; kb < nk; ++kb, ++rr) {
        const uint32_t r = rr % R;
        if (ok && !mbar_wait_bounded(&raw_full[r], (rr / R) & 1)) ok = false;
        // slot grp's previous use was this group's stage of raw block rr-1
        if (ok && rr >= 1 && !mbar_wait_bounded(&a_empty[grp], (rr - 1) & 1)) ok = false;
        const uint8_t* src = raw + r * kNpRawBytes;
        uint8_t* dst = sa + grp * kNpAStage;
        if (ok) {
          if (t.gu) {
            np_expand_f16(src, dst, grp, row, cc);
            np_expand_f16(src + kNvTileBytes, dst + kNpATile, grp, row, cc);
          } else {
            np_expand_bf16(src, dst, grp, row, cc, 0);
            np_expand_bf16(src, dst, grp, row, cc, 1);
          }
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        }
        __syncwarp();
        if (ok && lane == 0) {
          mbar_arrive(&a_full[grp]);
          mbar_arrive(&raw_empty[r]);
        }
      }
    }
    if (!ok && lane == 0) atomicOr(p.err, kErrWaitTimeout);
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
int launch_nvp_route(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                     float* logits, int32_t* topk_ids, float* topk_weights,
                     const Fp8Workspace& ws, cudaStream_t stream, const void* logits_in) {
  if (M == 0) return FLYAI_OK;
  const int E = d.num_experts, H = d.hidden, k = d.top_k;
  const int El = d.expert_end - d.expert_begin;
  if (!ws.pxb) return FLYAI_ERR_UNSUPPORTED;
  if (np_launch(nvp_logits_kernel,
                dim3((E + kLgExp - 1) / kLgExp, (M + kLgTok - 1) / kLgTok, kLgSlices), 256, 0, stream,
                false, static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w.router_w), M, E,
                H, ws.plog, ws.pxm) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  if (np_launch(nvp_logits_sum_kernel, dim3(4 * 148), 256, 0, stream, true,
                static_cast<const double*>(ws.plog), static_cast<const float*>(ws.pxm), M, E,
                ws.logits, logits, ws.pxr) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  const int st = launch_fp8_select(d, M, w, topk_ids, topk_weights, ws, stream, logits_in);
  if (st != FLYAI_OK) return st;
  NpPlanParams pp{ws.ids, M * k, d.expert_begin, El, ws.max_chunks, ws.counts, ws.offsets, ws.perm,
                  ws.inv, ws.n_chunks, ws.chunk_info, ws.chunk_done};
  const size_t psmem = np_plan_smem(El);
  if (cudaFuncSetAttribute(nvp_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(psmem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (np_launch(nvp_plan_kernel, dim3(1), kPlanThreads, psmem, stream, true, pp) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  const int KS = H / kNpK;
  if (np_launch(nvp_scatter_kernel, dim3((KS + 7) / 8, nvp_max_chunks(El, M * k)), 256, 0, stream,
                true, static_cast<const uint16_t*>(x), static_cast<const int32_t*>(ws.perm),
                static_cast<const int32_t*>(ws.n_chunks), static_cast<const int4*>(ws.chunk_info),
                static_cast<const float*>(ws.pxr), static_cast<const float*>(ws.wts), ws.pxb, ws.pcr,
                ws.pcf, ws.pcw, H, k) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  return FLYAI_OK;
}

static size_t np_global_offset(const flyai_moe_desc& d, int proj) {
  const size_t nexp = d.expert_end - d.expert_begin + d.n_shared;
  return nv_bank(d.hidden, d.inter, proj).expert * nexp;
}

int launch_nvp_experts(const flyai_moe_desc& d, int M, const flyai_moe_weights& w, void* y,
                       uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream,
                       cudaEvent_t ev0, cudaEvent_t ev1) {
  if (M == 0) return FLYAI_OK;
  if (!ws.pxb) return FLYAI_ERR_UNSUPPORTED;
  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem = np_smem_bytes();
  if (smem > static_cast<size_t>(max_smem)) return FLYAI_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(nvp_moe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  NpParams prm{};
  prm.w13 = static_cast<const uint8_t*>(w.w13);
  prm.w2 = static_cast<const uint8_t*>(w.w2);
  prm.b13 = nv_bank(d.hidden, d.inter, FLYAI_PROJ_W13);
  prm.b2 = nv_bank(d.hidden, d.inter, FLYAI_PROJ_W2);
  prm.g13 = reinterpret_cast<const float*>(prm.w13 + np_global_offset(d, FLYAI_PROJ_W13));
  prm.g2 = reinterpret_cast<const float*>(prm.w2 + np_global_offset(d, FLYAI_PROJ_W2));
  prm.n_chunks = ws.n_chunks;
  prm.chunk_info = ws.chunk_info;
  prm.chunk_done = ws.chunk_done;
  prm.perm = ws.perm;
  prm.wts = ws.wts;
  prm.xb = ws.pxb;
  prm.hb = ws.phb;
  prm.cr = ws.pcr;
  prm.cf = ws.pcf;
  prm.cw = ws.pcw;
  prm.rows = rows;
  prm.H = d.hidden;
  prm.I = d.inter;
  prm.err = ws.err;
  if (ev0 && ev1 && cudaEventRecord(ev0, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  if (np_launch(nvp_moe_kernel, dim3(sms), kNpThreads, smem, stream, true, prm) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  if (ev0 && ev1 && cudaEventRecord(ev1, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  return y ? launch_fp8_combine(d, M, rows, y, ws, stream, true) : FLYAI_OK;
}

}  // namespace flyai
