// Dense FP8 linear at decode / verify sizes on sm_100a: y = linear(x, W) for an
// e4m3 weight W [N, K] with one scale per 128x128 block, x bf16 [M, K], y bf16
// [M, N] -- the attention projections (wq_a, wq_b, wkv, wo_b, the indexer's wq_b)
// and the shared expert's w1 / w3 / w2 of a DeepSeek-V4 layer, each one single-row
// GEMM per decode token.
//
// Reference arithmetic:
//   linear     vendor/deepseek_v4_ref/inference/model.py:114-124: act_quant of x,
//              then fp8_gemm on the weight and its scale, bf16 out;
//   act_quant  kernel.py:40-125 (act_quant.cuh);
//   fp8_gemm   kernel.py:203-274: per 128-wide K block kb a tensor-core partial
//              D_kb of the e4m3 values, acc = D_kb * (s_x[m, kb] * s_w[n/128, kb])
//              + acc in fp32 in ascending kb, rounded once to bf16;
//   lever      engines/deepseek_v4/v4_fp8_gemv.py:1-97, 178-262 (the same GEMM
//              re-tiled for occupancy at M <= 32; w1 and w3 of the shared expert
//              as one bank, v4_fp8_gemv.py:280-441).
//
// Two or three launches, PDL-chained:
//   ln_quant_kernel   act_quant of x straight into the MMA's B tiles (one warp per
//                     token and 128-block);
//   ln_gemm_kernel    persistent, at most one CTA per SM.  Work units are pieces of
//                     kLnUnit consecutive 128-wide K blocks of one 128-row block,
//                     row-block-major; each CTA takes a contiguous run of the same
//                     number of units, so a 512-row wkv (cut along K into 8 pieces
//                     per row block) and a 32768-row wq_b both spread over the SMs.
//                     Per K block: a bulk copy of the 16 KB weight block
//                     (evict-first) and of the B tile, four tcgen05 kind::f8f6f4
//                     MMAs (M = 128 weight rows, N = 16/32/64 token columns) into a
//                     TMEM buffer of their own, and the epilogue's fp32 fold
//                     acc = fma(D_kb, s_x * s_w, acc) over the piece.  A row block
//                     whose pieces all belong to one CTA is summed and written as
//                     bf16 there; pieces of a row block that CTAs share go to the
//                     workspace.  The weight copies of a CTA's first stages are
//                     issued before griddepcontrol.wait, so the stream starts while
//                     the quantisation kernel runs;
//   ln_reduce_kernel  (only when a row block is shared) adds the pieces of each
//                     shared row block in ascending K and writes bf16.
// Per element the result is the reference's fp32 chain over each kLnUnit-block
// piece, the pieces' sums added in ascending K: a function of K only, the same
// whichever CTA computed which piece (so a stacked [w1; w3] bank gives the two
// separate calls' bits).  Every wait is bounded (~2 s) and records
// kErrWaitTimeout in workspace word 0.
#include "act_quant.cuh"
#include "common.cuh"
#include "fp8_moe.cuh"
#include "tcgen05.cuh"

namespace flyai {
namespace {

constexpr int kLnBlock = kF8Hdr + kF8Tile;   // bank block: fp32 scale (16-byte header) + one tile
constexpr int kLnThreads = 192;              // warp 0 producer, 1 MMA issuer, 2..5 epilogue
constexpr int kLnAcc = 8;                    // TMEM buffers (K-steps in flight)
constexpr int kLnMaxTokens = 64;             // tokens per launch (larger calls run in slices)
constexpr int kLnUnit = 4;                   // weight blocks per work unit (64 KB)
constexpr int kLnSmemBudget = 227 * 1024;
constexpr int kLnWsHead = 256;               // error word, then the B tiles

// Byte offset of K element kk (0..127) of token row i inside a B tile of Np rows:
// the canonical no-swizzle K-major operand (16-byte K chunks Np*16 bytes apart).
__host__ __device__ __forceinline__ int ln_btile_offset(int Np, int i, int kk) {
  return (kk >> 4) * (Np * 16) + (i >> 3) * 128 + (i & 7) * 16 + (kk & 15);
}
__host__ __device__ constexpr int ln_bbytes(int Np) { return Np * kF8Blk + Np * 4; }
__host__ __device__ inline int ln_np(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : 64; }

template <int Np>
struct LnGeo {
  static constexpr int kBTile = Np * kF8Blk;
  static constexpr int kBBytes = ln_bbytes(Np);
  static constexpr int kStage = kLnBlock + kBBytes;
  static constexpr int kBarBytes = 1024;
  static constexpr int kStages = (kLnSmemBudget - kBarBytes) / kStage;
  static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStage + kBarBytes;
  static constexpr uint32_t kCols = kLnAcc * Np;   // 128, 256 or 512 TMEM columns
  static_assert(kStage % 16 == 0, "stage alignment");
  static_assert((2 * kStages + 2 * kLnAcc + 1) * 8 + 16 <= kBarBytes, "barrier area");
};

// Work units: each row block's K range in pieces of kLnUnit weight blocks (the
// last piece may be shorter), row-block-major.  The arithmetic of an output is a
// function of K alone: an fp32 fma chain over each piece, the pieces' sums added
// in ascending K.  Which CTA computes which piece does not change a bit.
struct LnPlan {
  int RB, KB, SU;   // row blocks, K blocks, units per row block
  long long UT;     // units
  int G;            // CTAs: CTA c takes units [UT*c/G, UT*(c+1)/G)
};
__host__ __device__ inline long long ln_unit_step(const LnPlan& q, long long u) {
  return (u / q.SU) * q.KB + (u % q.SU) * kLnUnit;
}
// The CTA whose units hold unit u: c = ceil((u+1) G / UT) - 1.
__host__ __device__ inline int ln_cta_of(const LnPlan& q, long long u) {
  return static_cast<int>(((u + 1) * q.G + q.UT - 1) / q.UT) - 1;
}
__host__ __device__ inline bool ln_row_cut(const LnPlan& q, int rb) {
  const long long f = static_cast<long long>(rb) * q.SU;
  return ln_cta_of(q, f) != ln_cta_of(q, f + q.SU - 1);
}
inline LnPlan ln_plan(int N, int K, int sms) {
  LnPlan q;
  q.RB = N / kF8Blk;
  q.KB = K / kF8Blk;
  q.SU = (q.KB + kLnUnit - 1) / kLnUnit;
  q.UT = static_cast<long long>(q.RB) * q.SU;
  // as few CTAs as give every SM the same whole number of units
  const long long per = (q.UT + sms - 1) / sms;
  q.G = static_cast<int>((q.UT + per - 1) / per);
  return q;
}

// Workspace: [0, 4) error word, [4, 256) unused, the B tiles [K/128][ln_bbytes(Np)]
// and the piece sums of cut row blocks [N/128][units per row block][Mw][128] fp32,
// Mw = the tokens of one launch.
struct LnWs {
  size_t xb, part, total;
};
inline LnWs ln_ws_layout(int Mw, int N, int K) {
  const int m = Mw > 0 ? Mw : 1;
  const size_t KB = K / kF8Blk, SU = (KB + kLnUnit - 1) / kLnUnit;
  LnWs w;
  w.xb = kLnWsHead;
  w.part = align_up(w.xb + KB * ln_bbytes(ln_np(m)), 256);
  w.total = w.part + static_cast<size_t>(N / kF8Blk) * SU * m * kF8Blk * 4;
  return w;
}

// ---------------------------------------------------------------------------
// Bank packing: block (rb, kb) = fp32 scale of the weight block (e8m0 bytes
// become their exact powers of two) + the 128x128 tile, 16-byte chunk c of row r
// at c*2048 + r*16.
// ---------------------------------------------------------------------------
__global__ void ln_pack_kernel(const uint8_t* __restrict__ w, const void* __restrict__ scale,
                               int e8m0, uint8_t* __restrict__ bank, int N, int K) {
  constexpr int kUnits = kLnBlock / 16;   // header + 1024 tile chunks
  const int RB = N / kF8Blk, KB = K / kF8Blk;
  const size_t total = static_cast<size_t>(RB) * KB * kUnits;
  for (size_t u = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; u < total;
       u += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t blk = u / kUnits;
    const int v = static_cast<int>(u % kUnits);
    const int rb = static_cast<int>(blk / KB), kb = static_cast<int>(blk % KB);
    uint4 out;
    if (v == 0) {
      const size_t si = static_cast<size_t>(rb) * KB + kb;
      const float s = e8m0 ? e8m0_to_float(static_cast<const uint8_t*>(scale)[si])
                           : static_cast<const float*>(scale)[si];
      out = make_uint4(__float_as_uint(s), 0u, 0u, 0u);
    } else {
      const int c = (v - 1) / kF8Blk, r = (v - 1) % kF8Blk;
      out = *reinterpret_cast<const uint4*>(w + (static_cast<size_t>(rb) * kF8Blk + r) * K +
                                            kb * kF8Blk + c * 16);
    }
    *reinterpret_cast<uint4*>(bank + blk * kLnBlock + static_cast<size_t>(v) * 16) = out;
  }
}

// ---------------------------------------------------------------------------
// act_quant of the call's token rows into the B tiles (rows M..Np-1 are left as
// they are: they only feed MMA columns nobody reads)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) ln_quant_kernel(const uint16_t* __restrict__ x,
                                                       uint8_t* __restrict__ xb, int M, int K,
                                                       int Np, int ue8m0) {
  pdl_wait();
  pdl_launch_dependents();
  const int KB = K / kF8Blk;
  const int wid = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (wid >= M * KB) return;
  const int i = wid / KB, kb = wid % KB;
  float s;
  const uint32_t q = act_quant4(x + static_cast<size_t>(i) * K + kb * kF8Blk, lane, ue8m0, s);
  uint8_t* tile = xb + static_cast<size_t>(kb) * ln_bbytes(Np);
  *reinterpret_cast<uint32_t*>(tile + ln_btile_offset(Np, i, lane * 4)) = q;
  if (lane == 0) reinterpret_cast<float*>(tile + Np * kF8Blk)[i] = s;
}

// ---------------------------------------------------------------------------
// The GEMM
// ---------------------------------------------------------------------------
struct LnParams {
  const uint8_t* bank;   // [N/128][K/128] blocks of kLnBlock bytes
  const uint8_t* xb;     // [K/128] B tiles
  uint16_t* y;           // bf16 [M, N]
  float* part;           // [N/128][units per row block][M][128]: pieces of cut row blocks
  int32_t* err;
  LnPlan q;
  int M, N;
};

template <int Np>
__global__ void __launch_bounds__(kLnThreads, 1) ln_gemm_kernel(const __grid_constant__ LnParams p) {
  using G = LnGeo<Np>;
  constexpr int S = G::kStages;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* ring = sm;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + S * G::kStage);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + kLnAcc;
  uint64_t* epi_done = acc_empty + kLnAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 4);   // MMA completion + the four epilogue warps read the scales
    }
    for (int b = 0; b < kLnAcc; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(epi_done, 4);
    mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, G::kCols);
    tc::tmem_relinquish();
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tmem_slot;
  pdl_launch_dependents();

  const LnPlan& q = p.q;
  const long long u0 = q.UT * blockIdx.x / q.G, u1 = q.UT * (blockIdx.x + 1) / q.G;
  const long long s0 = ln_unit_step(q, u0);
  const int n = static_cast<int>(ln_unit_step(q, u1) - s0);   // weight blocks of this CTA

  if (warp == 0) {
    // ---------------- producer ----------------
    // The weight blocks do not depend on the preceding launch: the first stages
    // are requested before the wait (one lane per stage), their B tiles after it.
    const uint64_t wpol = l2_policy_evict_first();
    const int npre = n < S ? n : S;
    for (int j = lane; j < npre; j += 32) {
      mbar_expect_tx(&full[j], kLnBlock + G::kBBytes);
      bulk_g2s_hint(ring + j * G::kStage, p.bank + (s0 + j) * kLnBlock, kLnBlock, &full[j], wpol);
    }
    pdl_wait();
    for (int j = lane; j < npre; j += 32) {
      const int kb = static_cast<int>((s0 + j) % q.KB);
      bulk_g2s(ring + j * G::kStage + kLnBlock, p.xb + static_cast<size_t>(kb) * G::kBBytes,
               G::kBBytes, &full[j]);
    }
    if (lane == 0) {
      bool ok = true;
      int issued = npre;
      for (; issued < n; ++issued) {
        const int s = issued % S;
        const uint32_t use = issued / S;
        if (!mbar_wait_bounded(&empty[s], (use - 1) & 1)) {
          ok = false;
          break;
        }
        const long long st = s0 + issued;
        const int kb = static_cast<int>(st % q.KB);
        mbar_expect_tx(&full[s], kLnBlock + G::kBBytes);
        bulk_g2s_hint(ring + s * G::kStage, p.bank + st * kLnBlock, kLnBlock, &full[s], wpol);
        bulk_g2s(ring + s * G::kStage + kLnBlock, p.xb + static_cast<size_t>(kb) * G::kBBytes,
                 G::kBBytes, &full[s]);
      }
      for (int s = 0; s < S && s < issued; ++s) {   // copies in flight land before exit
        const int last = ((issued - 1 - s) / S) * S + s;
        if (!mbar_wait_bounded(&full[s], (last / S) & 1)) ok = false;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    bool ok = true;
    const uint32_t idesc = tc::idesc_f8_e4m3(Np);
    const uint64_t a0 = tc::smem_desc_kmajor(ring + kF8Hdr, 2048, 128);
    const uint64_t b0 = tc::smem_desc_kmajor(ring + kLnBlock, Np * 16, 128);
    for (int j = 0; j < n; ++j) {
      const int s = j % S, buf = j % kLnAcc;
      ok = mbar_wait_bounded(&full[s], (j / S) & 1) &&
           (j < kLnAcc || mbar_wait_bounded(&acc_empty[buf], ((j / kLnAcc) - 1) & 1));
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc::fence_after_sync();
      const uint32_t st16 = static_cast<uint32_t>((s * G::kStage) >> 4);
      const uint32_t d = tbase + buf * Np;
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < 4; ++k)   // K = 32 bytes per MMA: 16-byte chunks 2k, 2k+1
          tc::mma_f8(d, a0 + st16 + k * (4096 >> 4), b0 + st16 + k * ((Np * 32) >> 4), idesc, k > 0);
        tc::commit_to(&empty[s]);
        tc::commit_to(&acc_full[buf]);
      }
      __syncwarp();
    }
    if (lane == 0) {
      // tensor memory goes back only after the epilogue read its last buffer
      if (!mbar_wait_bounded(epi_done, 0)) ok = false;
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, G::kCols);
  } else {
    // ---------------- epilogue (TMEM lane quadrant = warp % 4) ----------------
    pdl_wait();
    const int qd = warp & 3;
    const int r = 32 * qd + lane;   // row of the 128-row block
    bool ok = true;
    int j = 0;
    float tot[Np];
    for (long long u = u0; u < u1; ++u) {
      const int rb = static_cast<int>(u / q.SU), su = static_cast<int>(u % q.SU);
      const int kb0 = su * kLnUnit, kb1 = kb0 + kLnUnit < q.KB ? kb0 + kLnUnit : q.KB;
      float acc[Np];
#pragma unroll
      for (int i = 0; i < Np; ++i) acc[i] = 0.f;
      for (int kb = kb0; kb < kb1; ++kb, ++j) {
        const int s = j % S, buf = j % kLnAcc;
        if (ok && !mbar_wait_bounded(&full[s], (j / S) & 1)) ok = false;
        const uint8_t* stg = ring + s * G::kStage;
        const float sw = *reinterpret_cast<const float*>(stg);
        float sc[Np];
#pragma unroll
        for (int i = 0; i < Np; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(stg + kLnBlock + G::kBTile + i * 4);
          sc[i] = __fmul_rn(v.x, sw);
          sc[i + 1] = __fmul_rn(v.y, sw);
          sc[i + 2] = __fmul_rn(v.z, sw);
          sc[i + 3] = __fmul_rn(v.w, sw);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (ok && !mbar_wait_bounded(&acc_full[buf], (j / kLnAcc) & 1)) ok = false;
        tc::fence_after_sync();
        const uint32_t ta = tbase + buf * Np + ((32u * qd) << 16);
#pragma unroll
        for (int c = 0; c < Np; c += 16) {
          uint32_t v[16];
          tc::tmem_ld16(ta + c, v);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[c + i] = fmaf(__uint_as_float(v[i]), sc[c + i], acc[c + i]);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      const long long first = static_cast<long long>(rb) * q.SU;
      if (first >= u0 && first + q.SU <= u1) {
        // the whole row block is this CTA's: its pieces add up here, in ascending K
#pragma unroll
        for (int i = 0; i < Np; ++i) tot[i] = su == 0 ? acc[i] : __fadd_rn(tot[i], acc[i]);
        if (su == q.SU - 1) {
#pragma unroll
          for (int i = 0; i < Np; ++i)
            if (i < p.M) p.y[static_cast<size_t>(i) * p.N + rb * kF8Blk + r] = float_to_bf16_bits(tot[i]);
        }
      } else {
        // a piece of a row block other CTAs share: ln_reduce_kernel adds it
        float* dst = p.part + static_cast<size_t>(u) * p.M * kF8Blk + r;
#pragma unroll
        for (int i = 0; i < Np; ++i)
          if (i < p.M) dst[i * kF8Blk] = acc[i];
      }
    }
    if (!ok) atomicOr(p.err, kErrWaitTimeout);
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(epi_done);
  }
}

// Row blocks cut between CTAs: block (rb, 8-token group), thread = row.  The
// pieces' sums are added in ascending K (8 pieces x 8 tokens of loads in flight).
__global__ void __launch_bounds__(kF8Blk) ln_reduce_kernel(const float* __restrict__ part,
                                                           uint16_t* __restrict__ y, LnPlan q, int M,
                                                           int N) {
  pdl_launch_dependents();
  const int rb = blockIdx.x, r = threadIdx.x, i0 = blockIdx.y * 8;
  if (!ln_row_cut(q, rb)) return;
  pdl_wait();
  const float* src = part + static_cast<size_t>(rb) * q.SU * M * kF8Blk + r;
  float v[8];
#pragma unroll
  for (int ii = 0; ii < 8; ++ii) v[ii] = 0.f;
  for (int s0 = 0; s0 < q.SU; s0 += 8) {
    float pc[8][8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int ii = 0; ii < 8; ++ii)
        pc[u][ii] = s0 + u < q.SU && i0 + ii < M
                        ? __ldcg(src + (static_cast<size_t>(s0 + u) * M + i0 + ii) * kF8Blk)
                        : 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int ii = 0; ii < 8; ++ii)
        if (s0 + u < q.SU) v[ii] = s0 + u == 0 ? pc[u][ii] : __fadd_rn(v[ii], pc[u][ii]);
  }
#pragma unroll
  for (int ii = 0; ii < 8; ++ii)
    if (i0 + ii < M) y[static_cast<size_t>(i0 + ii) * N + rb * kF8Blk + r] = float_to_bf16_bits(v[ii]);
}

template <typename Kern, typename... Args>
cudaError_t ln_launch(Kern kernel, dim3 grid, int block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
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

int ln_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev < 64) cached[dev] = n;
  return n;
}

template <int Np>
int ln_gemm_launch(const LnParams& p, int grid, cudaStream_t stream) {
  using G = LnGeo<Np>;
  if (cudaFuncSetAttribute(ln_gemm_kernel<Np>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(G::kSmem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (ln_launch(ln_gemm_kernel<Np>, dim3(grid), kLnThreads, G::kSmem, stream, p) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  return FLYAI_OK;
}

bool ln_shape_ok(int N, int K) {
  return N >= kF8Blk && K >= kF8Blk && N % kF8Blk == 0 && K % kF8Blk == 0 && N <= (1 << 20) &&
         K <= (1 << 20);
}

}  // namespace
}  // namespace flyai

using namespace flyai;

extern "C" int flyai_fp8_linear_bank_bytes(int32_t N, int32_t K, size_t* bytes) {
  if (!bytes) return FLYAI_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0) return FLYAI_ERR_INVALID_ARG;
  if (!ln_shape_ok(N, K)) return FLYAI_ERR_ALIGNMENT;
  *bytes = static_cast<size_t>(N / kF8Blk) * (K / kF8Blk) * kLnBlock;
  return FLYAI_OK;
}

extern "C" int flyai_fp8_linear_pack(int32_t N, int32_t K, const void* weight, const void* scale,
                                     int32_t scale_dtype, void* bank, void* stream) {
  if (N <= 0 || K <= 0) return FLYAI_ERR_INVALID_ARG;
  if (!ln_shape_ok(N, K)) return FLYAI_ERR_ALIGNMENT;
  if (scale_dtype != FLYAI_LIN_SCALE_F32 && scale_dtype != FLYAI_LIN_SCALE_E8M0)
    return FLYAI_ERR_INVALID_ARG;
  if (!weight || !scale || !bank) return FLYAI_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(weight) % 16 || reinterpret_cast<uintptr_t>(bank) % 16 ||
      (scale_dtype == FLYAI_LIN_SCALE_F32 && reinterpret_cast<uintptr_t>(scale) % 4))
    return FLYAI_ERR_ALIGNMENT;
  ln_pack_kernel<<<1184, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(weight), scale, scale_dtype == FLYAI_LIN_SCALE_E8M0 ? 1 : 0,
      static_cast<uint8_t*>(bank), N, K);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

extern "C" int flyai_fp8_linear_workspace_bytes(int32_t max_tokens, int32_t N, int32_t K,
                                                size_t* bytes) {
  if (!bytes || max_tokens < 0 || N <= 0 || K <= 0) return FLYAI_ERR_INVALID_ARG;
  if (!ln_shape_ok(N, K)) return FLYAI_ERR_ALIGNMENT;
  *bytes = ln_ws_layout(max_tokens < kLnMaxTokens ? max_tokens : kLnMaxTokens, N, K).total;
  return FLYAI_OK;
}

extern "C" int flyai_fp8_linear(int32_t M, int32_t N, int32_t K, const void* x, const void* bank,
                                int32_t scale_fmt, void* y, void* workspace, size_t workspace_bytes,
                                void* stream) {
  if (M < 0 || N <= 0 || K <= 0) return FLYAI_ERR_INVALID_ARG;
  if (!ln_shape_ok(N, K)) return FLYAI_ERR_ALIGNMENT;
  if (scale_fmt != FLYAI_LIN_FMT_AMAX && scale_fmt != FLYAI_LIN_FMT_UE8M0) return FLYAI_ERR_INVALID_ARG;
  if (M == 0) return FLYAI_OK;
  if (!x || !bank || !y) return FLYAI_ERR_INVALID_ARG;
  if (!workspace) return FLYAI_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(bank) % 16 ||
      reinterpret_cast<uintptr_t>(y) % 4 || reinterpret_cast<uintptr_t>(workspace) % 256)
    return FLYAI_ERR_ALIGNMENT;
  // tokens per launch: up to kLnMaxTokens, as many as the workspace holds
  int Mw = M < kLnMaxTokens ? M : kLnMaxTokens;
  while (Mw > 0 && ln_ws_layout(Mw, N, K).total > workspace_bytes) --Mw;
  if (Mw == 0) return FLYAI_ERR_WORKSPACE;
  const int sms = ln_sm_count();
  if (sms <= 0) return FLYAI_ERR_CUDA;
  const LnPlan q = ln_plan(N, K, sms);
  bool any_cut = false;
  for (int c = 1; c < q.G && !any_cut; ++c) any_cut = (q.UT * c / q.G) % q.SU != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  for (int t0 = 0; t0 < M; t0 += Mw) {
    const int m = M - t0 < Mw ? M - t0 : Mw;
    const LnWs w = ln_ws_layout(m, N, K);
    const int Np = ln_np(m);
    const uint16_t* xs = static_cast<const uint16_t*>(x) + static_cast<size_t>(t0) * K;
    const int warps = m * (K / kF8Blk);
    if (ln_launch(ln_quant_kernel, dim3((warps + 7) / 8), 256, 0, s, xs, ws + w.xb, m, K, Np,
                  scale_fmt == FLYAI_LIN_FMT_UE8M0 ? 1 : 0) != cudaSuccess)
      return FLYAI_ERR_CUDA;
    note_launch();
    LnParams p;
    p.bank = static_cast<const uint8_t*>(bank);
    p.xb = ws + w.xb;
    p.y = static_cast<uint16_t*>(y) + static_cast<size_t>(t0) * N;
    p.part = reinterpret_cast<float*>(ws + w.part);
    p.err = reinterpret_cast<int32_t*>(ws);
    p.q = q;
    p.M = m;
    p.N = N;
    const int st = Np == 16 ? ln_gemm_launch<16>(p, q.G, s)
                 : Np == 32 ? ln_gemm_launch<32>(p, q.G, s)
                            : ln_gemm_launch<64>(p, q.G, s);
    if (st != FLYAI_OK) return st;
    if (any_cut) {
      if (ln_launch(ln_reduce_kernel, dim3(q.RB, (m + 7) / 8), kF8Blk, 0, s,
                    static_cast<const float*>(p.part), p.y, q, m, N) != cudaSuccess)
        return FLYAI_ERR_CUDA;
      note_launch();
    }
  }
  return FLYAI_OK;
}
