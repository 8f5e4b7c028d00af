// DeepSeek-V4-style W4A8 MoE layer on sm_100a (FLYAI_FMT_FP4_W4A8 with
// FLYAI_GATE_SQRTSOFTPLUS and FLYAI_ACT_SILU).
//
// Reference arithmetic (vendor/deepseek_v4_ref/inference/model.py, run with the
// V4-Flash configuration -- expert_dtype "fp4", dtype "fp8", scale_fmt "ue8m0"):
// Expert.forward (:599-611) with fp4 Linears (:114-121): act_quant per 1x128 with
// power-of-two scales, fp4_gemm = e4m3 activations x e2m1 weights with one e8m0
// scale per 32, fp32 accumulation, bf16 out; gate/up to fp32, up clamped to
// +-swiglu_limit and gate to <= swiglu_limit, silu(gate) * up, times the routing
// weight, to bf16; then w2 the same way.  The shared expert is the same Expert
// with fp8 Linears (e4m3 weights, e8m0 per 128x128 block).  MoE.forward
// (:634-649) folds the routed outputs in fp32 in ascending expert id -- an
// expert repeated within a token (hash routing) counts once, with its last slot
// -- then adds the shared expert and rounds to bf16.
//
// Launch chain: f8_route_kernel (gate, ue8m0 act_quant of the token rows, plan),
// v4_scatter_kernel (each chunk's token rows into B blocks with their scale
// chunk), v4_moe_kernel (every expert projection, one persistent CTA per SM),
// f8_combine_kernel (the fold).
//
// v4_moe_kernel: items are the FP8 kernel's -- (chunk, 128-row block) of gate/up
// (w1 and w3 tiles of the same rows, K = H) then of down (K = I); a chunk's down
// items wait for its gate/up items (chunk_done).  Per 128-wide K block:
//   producer warp   bulk-copies the bank block (routed: e2m1 tiles; shared:
//                   e4m3 tiles) and the chunk's B block into a raw ring slot;
//   expander warps  turn e2m1 into e4m3 (exact) in the canonical K-major
//                   operand layout of an X slot, or copy e4m3 as it is;
//   two MMA warps   (X slot = issuer = K-block parity) copy the weight and
//                   activation scale chunks to tensor memory and issue
//                   tcgen05.mma kind::mxf8f6f4 block32 (M=128, N=16, K=32) --
//                   the weights' e8m0 scales and the tokens' ue8m0 scales are
//                   applied by the tensor core, so an item accumulates its
//                   whole K in fp32 in one tensor-memory slot (one half per
//                   issuer);
//   epilogue warps  add the halves, round to bf16 and run the reference's
//                   elementwise chain (gate/up: SwiGLU, weight, bf16, ue8m0
//                   act_quant straight into the chunk's down B block; down:
//                   bf16 rows by flat pair index).
// Every wait is bounded (~2 s) and records kErrWaitTimeout.
#include <cuda_fp8.h>
#include <math.h>

#include "common.cuh"
#include "fp8_moe.cuh"
#include "tc_bank.cuh"
#include "tcgen05.cuh"
#include "v4.cuh"

namespace flyai {

namespace {
template <typename Kern, typename... Args>
cudaError_t v4_launch(Kern kernel, dim3 grid, int block, size_t smem, cudaStream_t s, bool pdl,
                      Args... args) {
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

__device__ __constant__ float kV4Inv448 = static_cast<float>(1.0 / 448.0);

__device__ __forceinline__ uint32_t to_e4m3(float v) {
  v = fminf(fmaxf(v, -448.f), 448.f);
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float v4_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
}  // namespace

// ---------------------------------------------------------------------------
// Bank packing
// ---------------------------------------------------------------------------
size_t v4_packed_bytes(const flyai_moe_desc& d, int proj) {
  const V4Bank b = v4_bank(d, proj);
  return b.shared_off + b.f8_expert * static_cast<size_t>(d.n_shared);
}

// Routed experts: one thread per 16-byte unit of a raw tile (544 units: 512 of
// e2m1 -- K-chunk c, rows 2h and 2h+1 of 8-row group g at unit c*64 + g*4 + h --
// then 32 lines of the scale chunk).
__global__ void v4_pack_fp4_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                                   uint8_t* __restrict__ packed, int nexp, int R, int K, V4Bank b) {
  constexpr int kUnits = kV4RawTile / 16;   // 544
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
    if (v < kV4Fp4Tile / 16) {
      const int c = v / 64, g = (v % 64) / 4, h = v % 4;
      const int r = g * 8 + 2 * h;
      const uint2 a = *reinterpret_cast<const uint2*>(blocks + (row0 + r) * (K / 2) + kb * 64 + c * 8);
      const uint2 bb = *reinterpret_cast<const uint2*>(blocks + (row0 + r + 1) * (K / 2) + kb * 64 + c * 8);
      out = make_uint4(a.x, a.y, bb.x, bb.y);
    } else {
      const int l = v - kV4Fp4Tile / 16;   // line: rows l, l+32, l+64, l+96, four 32-blocks each
      uint32_t word[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        word[q] = *reinterpret_cast<const uint32_t*>(scales + (row0 + 32 * q + l) * (K / 32) + kb * 4);
      out = make_uint4(word[0], word[1], word[2], word[3]);
    }
    *reinterpret_cast<uint4*>(packed + blk * b.fp4_block + static_cast<size_t>(tt) * kV4RawTile +
                              static_cast<size_t>(v) * 16) = out;
  }
}

// Shared expert(s): one thread per 16-byte unit of an e4m3 tile (1056 units:
// 1024 of data in the canonical K-major layout, then the scale chunk, whose 512
// bytes all hold the tile's e8m0 block scale).
__global__ void v4_pack_f8_kernel(const uint8_t* __restrict__ weight, const uint8_t* __restrict__ scale,
                                  uint8_t* __restrict__ packed, int nexp, int R, int K, V4Bank b) {
  constexpr int kUnits = kV4XTile / 16;   // 1056
  const size_t total = static_cast<size_t>(nexp) * b.RB * b.KB * b.tiles * kUnits;
  const int half_rows = b.tiles == 2 ? R / 2 : 0;
  for (size_t u = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; u < total;
       u += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t tile_id = u / kUnits;
    const int v = static_cast<int>(u % kUnits);
    const int tt = static_cast<int>(tile_id % b.tiles);
    const size_t blk = tile_id / b.tiles;
    const int kb = static_cast<int>(blk % b.KB);
    const int rb = static_cast<int>((blk / b.KB) % b.RB);
    const int e = static_cast<int>(blk / (static_cast<size_t>(b.KB) * b.RB));
    const size_t row0 = static_cast<size_t>(e) * R + tt * half_rows + rb * 128;
    uint4 out;
    if (v < kV4F8Tile / 16) {
      const int c = v / 128, r = v % 128;
      out = *reinterpret_cast<const uint4*>(weight + (row0 + r) * K + kb * 128 + c * 16);
    } else {
      const uint32_t s = scale[(static_cast<size_t>(e) * (R / 128) + row0 % R / 128) * (K / 128) + kb];
      const uint32_t w = s * 0x01010101u;
      out = make_uint4(w, w, w, w);
    }
    *reinterpret_cast<uint4*>(packed + blk * b.f8_block + static_cast<size_t>(tt) * kV4XTile +
                              static_cast<size_t>(v) * 16) = out;
  }
}

int launch_v4_pack_fp4(const flyai_moe_desc& d, int proj, const void* blocks, const void* scales,
                       void* packed, cudaStream_t stream) {
  const int nexp = d.expert_end - d.expert_begin;
  if (nexp == 0) return FLYAI_OK;
  const V4Bank b = v4_bank(d, proj);
  const int R = proj == FLYAI_PROJ_W13 ? 2 * d.inter : d.hidden;
  const int K = proj == FLYAI_PROJ_W13 ? d.hidden : d.inter;
  v4_pack_fp4_kernel<<<2368, 256, 0, stream>>>(static_cast<const uint8_t*>(blocks),
                                               static_cast<const uint8_t*>(scales),
                                               static_cast<uint8_t*>(packed), nexp, R, K, b);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

int launch_v4_pack_shared(const flyai_moe_desc& d, int proj, const void* weight, const void* scale,
                          void* packed, cudaStream_t stream) {
  if (d.n_shared == 0) return FLYAI_OK;
  const V4Bank b = v4_bank(d, proj);
  const int R = proj == FLYAI_PROJ_W13 ? 2 * d.inter : d.hidden;
  const int K = proj == FLYAI_PROJ_W13 ? d.hidden : d.inter;
  v4_pack_f8_kernel<<<1184, 256, 0, stream>>>(static_cast<const uint8_t*>(weight),
                                              static_cast<const uint8_t*>(scale),
                                              static_cast<uint8_t*>(packed) + b.shared_off,
                                              d.n_shared, R, K, b);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Token rows -> each chunk's B blocks
// ---------------------------------------------------------------------------
struct V4ScatterParams {
  const uint8_t* xq;      // [M, H] e4m3 token rows
  const float* xs;        // [M, H/128] their power-of-two scales
  const int32_t* perm;
  const int32_t* n_chunks;
  const int4* chunk_info;
  uint8_t* xb;            // [max_chunks][H/128][kV4BBytes]
  int H, k, P;
};

// CTA (group of 8 K blocks, chunk), 256 threads: per K block 16 rows x 8 units of
// 16 bytes into the canonical B layout (unused rows zero), then the scale chunk
// (token i's e8m0 at byte i*16 + j, j = 0..3, the other rows 1.0).
__global__ void __launch_bounds__(256) v4_scatter_kernel(const __grid_constant__ V4ScatterParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.y;
  if (c >= *p.n_chunks) return;
  const int4 ci = p.chunk_info[c];
  const int KB = p.H / 128, kb0 = blockIdx.x * 8, nt = ci.z;
  for (int u = threadIdx.x; u < 8 * (128 + 32); u += blockDim.x) {
    const int kb = kb0 + u / 160, w = u % 160;
    if (kb >= KB) continue;
    uint8_t* blk = p.xb + (static_cast<size_t>(c) * KB + kb) * kV4BBytes;
    if (w < 128) {
      const int i = w / 8, cc = w % 8;   // row, K-chunk
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (i < nt) {
        const int pos = ci.y + i;
        const int t = pos < p.P ? __ldg(&p.perm[pos]) / p.k : pos - p.P;
        v = __ldg(reinterpret_cast<const uint4*>(p.xq + static_cast<size_t>(t) * p.H + kb * 128 + cc * 16));
      }
      *reinterpret_cast<uint4*>(blk + cc * 256 + (i >> 3) * 128 + (i & 7) * 16) = v;
    } else {
      const int i = w - 128;   // scale chunk line
      uint32_t b = 0x7F7F7F7Fu;
      if (i < nt && i < kV4Chunk) {
        const int pos = ci.y + i;
        const int t = pos < p.P ? __ldg(&p.perm[pos]) / p.k : pos - p.P;
        const uint32_t e = (__float_as_uint(__ldg(&p.xs[static_cast<size_t>(t) * KB + kb])) >> 23) & 0xFFu;
        b = e * 0x01010101u;
      }
      *reinterpret_cast<uint4*>(blk + kV4BTile + i * 16) = make_uint4(b, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    }
  }
}

// ---------------------------------------------------------------------------
// The expert kernel
// ---------------------------------------------------------------------------
constexpr int kV4RawStages = 4;
constexpr int kV4Slots = 2;                 // accumulator slots (items in flight)
constexpr int kV4SlotCols = 64;             // issuer p's 32 columns at p*32: gate +0, up +16
constexpr int kV4SfBase = kV4Slots * kV4SlotCols;
constexpr int kV4SfCols = 16;               // per X slot: A tile 0 [0,4), tile 1 [4,8), B [8,12)
constexpr int kV4ExpWarps = 8;
constexpr int kV4ExpBase = 7;               // first expander warp
constexpr int kV4Threads = (kV4ExpBase + kV4ExpWarps) * 32;   // 480
static_assert(kV4SfBase + 2 * kV4SfCols <= 256, "tensor memory budget");
static_assert(kV4Stage % 128 == 0, "stage alignment");

struct V4Params {
  const uint8_t* w13;
  const uint8_t* w2;
  V4Bank b13, b2;
  int El;                   // local routed experts; bank expert El is the shared one
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
  // expert cache (slots > 0): routed expert e of the plan is read from slot
  // slot_of[e]; the shared expert follows the `slots` routed slots
  const int32_t* slot_of;
  int slots;
};

__host__ __device__ inline size_t v4_smem_bytes() {
  return static_cast<size_t>(kV4RawStages + 2) * kV4Stage + align_up(kV4BBytes, 128) + 4 * kV4Chunk * 4 +
         (2 * kV4RawStages + 4 + 2 * kV4Slots + 1) * 8 + 16;
}

__device__ __forceinline__ uint32_t idesc_mxf8_e4m3(int N, int sf_id) {
  uint32_t d = 0;
  d |= static_cast<uint32_t>(sf_id & 3) << 4;     // B scale factor id
  // A and B format e4m3 = 0, both K-major
  d |= static_cast<uint32_t>((N >> 3) & 0x3F) << 17;
  d |= 1u << 23;                                  // scale format: ue8m0
  d |= static_cast<uint32_t>(128 >> 4) << 24;     // M = 128
  d |= static_cast<uint32_t>(sf_id & 3) << 29;    // A scale factor id
  return d;
}

// D(tmem) (+)= A(smem) x B(smem)^T, e4m3 operands with one e8m0 scale per 32 K
// on both, read from tensor memory (byte sf_id of each scale word).
__device__ __forceinline__ void mma_mxf8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(sfa_tmem),
      "r"(sfb_tmem)
      : "memory");
}

__global__ void __launch_bounds__(kV4Threads, 1) v4_moe_kernel(const __grid_constant__ V4Params p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  constexpr int SR = kV4RawStages;
  uint8_t* raw = sm;
  uint8_t* xr = sm + SR * kV4Stage;
  uint8_t* hst = xr + 2 * kV4Stage;                                       // down B block staging
  float* red = reinterpret_cast<float*>(hst + align_up(kV4BBytes, 128));  // [4 warps][16 tokens]
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(red + 4 * kV4Chunk);
  uint64_t* raw_empty = raw_full + SR;
  uint64_t* x_full = raw_empty + SR;
  uint64_t* x_empty = x_full + 2;
  uint64_t* acc_full = x_empty + 2;
  uint64_t* acc_empty = acc_full + kV4Slots;
  uint64_t* epi_done = acc_empty + kV4Slots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SR; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kV4ExpWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&x_full[s], kV4ExpWarps);
      mbar_init(&x_empty[s], 1);
    }
    for (int b = 0; b < kV4Slots; ++b) {
      mbar_init(&acc_full[b], 2);    // both issuers committed
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
        const V4Bank& B = t.gu ? p.b13 : p.b2;
        const bool f8 = e >= p.El;
        const size_t blk = f8 ? B.f8_block : B.fp4_block;
        int es = e;
        size_t shared_off = B.shared_off;
        if (p.slots > 0) {
          // a slot outside the cache (the host's table is wrong) reads slot 0, recorded
          es = f8 ? 0 : __ldg(&p.slot_of[e]);
          if (es < 0 || es >= p.slots) {
            atomicOr(p.err, kErrBadIndex);
            es = 0;
          }
          shared_off = static_cast<size_t>(p.slots) * B.fp4_expert;
        }
        const uint8_t* a = (t.gu ? p.w13 : p.w2) +
                           (f8 ? shared_off + static_cast<size_t>(e - p.El) * B.f8_expert
                               : static_cast<size_t>(es) * B.fp4_expert) +
                           static_cast<size_t>(t.mt) * B.KB * blk;
        const uint8_t* b = (t.gu ? p.xb : p.hb) + static_cast<size_t>(t.chunk) * B.KB * kV4BBytes;
        const uint32_t abytes = static_cast<uint32_t>(blk);
        int kb = 0;
        if (!t.gu) {
          // A down item's weights do not depend on the chunk's gate/up items: its
          // first stages are requested before the wait, only the B blocks after it
          const int npre = B.KB < SR ? B.KB : SR;
          for (; kb < npre; ++kb) {
            const uint32_t s = (ks + kb) % SR, use = (ks + kb) / SR;
            if (use > 0 && !mbar_wait_bounded(&raw_empty[s], (use - 1) & 1)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&raw_full[s], abytes + kV4BBytes);
            bulk_g2s_hint(raw + s * kV4Stage, a + static_cast<size_t>(kb) * abytes, abytes, &raw_full[s], wpol);
          }
          if (!wait_counter_geq(&p.chunk_done[t.chunk], NI)) ok = false;
          fence_proxy_async_global();
          for (int j = 0; j < kb; ++j) {   // (issued also after a failed wait: the phases complete)
            const uint32_t s = (ks + j) % SR;
            bulk_g2s(raw + s * kV4Stage + kV4BOff, b + static_cast<size_t>(j) * kV4BBytes, kV4BBytes,
                     &raw_full[s]);
          }
          ks += kb;
        }
        for (; ok && kb < B.KB; ++kb, ++ks) {
          const uint32_t s = ks % SR, use = ks / SR;
          if (use > 0 && !mbar_wait_bounded(&raw_empty[s], (use - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&raw_full[s], abytes + kV4BBytes);
          bulk_g2s_hint(raw + s * kV4Stage, a + static_cast<size_t>(kb) * abytes, abytes, &raw_full[s], wpol);
          bulk_g2s(raw + s * kV4Stage + kV4BOff, b + static_cast<size_t>(kb) * kV4BBytes, kV4BBytes,
                   &raw_full[s]);
        }
      }
      __syncwarp();
    }
    if (lane == 0) {
      for (uint32_t s = 0; s < SR && s < ks; ++s) {   // copies in flight land before exit
        const uint32_t last = ((ks - 1 - s) / SR) * SR + s;
        if (!mbar_wait_bounded(&raw_full[s], (last / SR) & 1)) ok = false;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
  } else if (warp >= kV4ExpBase) {
    // ---------------- expanders: raw slot -> X slot ----------------
    const int et = threadIdx.x - kV4ExpBase * 32, nth = kV4ExpWarps * 32;
    bool ok = true;
    uint32_t ks = 0;
    for (; ok && cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const bool f8 = __ldg(&p.chunk_info[t.chunk].x) >= p.El;
      const int nk = t.gu ? KB1 : KB2, tiles = t.gu ? 2 : 1;
      for (int kb = 0; kb < nk; ++kb, ++ks) {
        const uint32_t rs = ks % SR, xs = ks & 1u;
        ok = mbar_wait_bounded(&raw_full[rs], (ks / SR) & 1) &&
             (ks < 2 || mbar_wait_bounded(&x_empty[xs], ((ks >> 1) - 1) & 1));
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const uint8_t* src = raw + rs * kV4Stage;
        uint8_t* dst = xr + xs * kV4Stage;
        if (f8) {
          for (int u = et; u < tiles * (kV4XTile / 16); u += nth)
            *reinterpret_cast<uint4*>(dst + u * 16) = *reinterpret_cast<const uint4*>(src + u * 16);
        } else {
          for (int u = et; u < tiles * (kV4Fp4Tile / 16); u += nth) {
            const int tt = u / (kV4Fp4Tile / 16), v = u % (kV4Fp4Tile / 16);
            const uint4 w = *reinterpret_cast<const uint4*>(src + tt * kV4RawTile + v * 16);
            uint4 o0, o1;
            e2m1x8_to_e4m3(w.x, o0.x, o0.y);
            e2m1x8_to_e4m3(w.y, o0.z, o0.w);
            e2m1x8_to_e4m3(w.z, o1.x, o1.y);
            e2m1x8_to_e4m3(w.w, o1.z, o1.w);
            uint8_t* d = dst + tt * kV4XTile + v * 32;
            *reinterpret_cast<uint4*>(d) = o0;
            *reinterpret_cast<uint4*>(d + 16) = o1;
          }
          for (int u = et; u < tiles * (kV4Sf / 16); u += nth) {
            const int tt = u / (kV4Sf / 16), v = u % (kV4Sf / 16);
            *reinterpret_cast<uint4*>(dst + tt * kV4XTile + kV4F8Tile + v * 16) =
                *reinterpret_cast<const uint4*>(src + tt * kV4RawTile + kV4Fp4Tile + v * 16);
          }
        }
        for (int u = et; u < kV4BBytes / 16; u += nth)
          *reinterpret_cast<uint4*>(dst + kV4BOff + u * 16) =
              *reinterpret_cast<const uint4*>(src + kV4BOff + u * 16);
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");   // visible to the tensor core
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&x_full[xs]);
          mbar_arrive(&raw_empty[rs]);
        }
      }
    }
    if (!ok && lane == 0) atomicOr(p.err, kErrWaitTimeout);
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issuers (K blocks with ks % 2 == par, X slot par) ----------------
    const uint32_t par = warp - 1;
    bool ok = true;
    uint32_t ks = 0, su = 0;
    const uint32_t idesc[4] = {idesc_mxf8_e4m3(kV4Chunk, 0), idesc_mxf8_e4m3(kV4Chunk, 1),
                               idesc_mxf8_e4m3(kV4Chunk, 2), idesc_mxf8_e4m3(kV4Chunk, 3)};
    uint8_t* xs_base = xr + par * kV4Stage;
    const uint64_t a0 = tc::smem_desc_kmajor(xs_base, 2048, 128);
    const uint64_t b0 = tc::smem_desc_kmajor(xs_base + kV4BOff, 256, 128);
    const uint64_t cp0 = tc::smem_desc_kmajor(xs_base, 0, 128);
    const uint32_t sfc = tbase + kV4SfBase + par * kV4SfCols;
    // the whole warp walks the items and waits (operands stay warp-uniform); one
    // elected lane issues the tcgen05 ops
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const int nk = t.gu ? KB1 : KB2, tiles = t.gu ? 2 : 1;
      const uint32_t slot = su % kV4Slots;
      if (ok && su >= kV4Slots)
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&acc_empty[slot], ((su / kV4Slots) - 1) & 1));
      const uint32_t d = tbase + slot * kV4SlotCols + par * 32;
      bool fresh = true;   // the next MMA starts this issuer's half of the slot
      for (int kb = 0; kb < nk; ++kb, ++ks) {
        if ((ks & 1u) != par || !ok) continue;
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&x_full[par], (ks >> 1) & 1));
        if (!ok) continue;
        tc::fence_after_sync();
        if (elect_one()) {
          tc::copy_sf_chunk_desc(sfc, cp0 + (kV4F8Tile >> 4));
          if (tiles == 2) tc::copy_sf_chunk_desc(sfc + 4, cp0 + ((kV4XTile + kV4F8Tile) >> 4));
          tc::copy_sf_chunk_desc(sfc + 8, cp0 + ((kV4BOff + kV4BTile) >> 4));
#pragma unroll
          for (int j = 0; j < 4; ++j) {   // K = 32 per MMA: K-chunks 2j, 2j+1
            const uint32_t hi = static_cast<uint32_t>(j) << 30;
            for (int tt = 0; tt < tiles; ++tt)
              mma_mxf8(d + tt * kV4Chunk, a0 + ((tt * kV4XTile + j * 4096) >> 4), b0 + ((j * 512) >> 4),
                       idesc[j], (sfc + tt * 4) | hi, (sfc + 8) | hi, !fresh || j > 0);
          }
          tc::commit_to(&x_empty[par]);
        }
        __syncwarp();
        fresh = false;
      }
      if (elect_one()) tc::commit_to(&acc_full[slot]);   // (also with no K block of this issuer)
      __syncwarp();
      ++su;
    }
    if (lane == 0) {
      // tensor memory goes back only after the epilogue read its last slot
      if (!mbar_wait_bounded(epi_done, 0)) ok = false;
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
    if (warp == 1) {
      tc::fence_after_sync();
      tc::tmem_dealloc(tbase, 256);
    }
  } else {
    // ---------------- epilogue (TMEM lane quadrant = warp % 4) ----------------
    const int q = warp & 3;
    const int r = 32 * q + lane;   // row of the 128-row block
    bool ok = true;
    uint32_t ks = 0, su = 0;
    for (; cur.valid(); cur.next()) {
      const TcItem t = cur.t;
      const int4 ci = __ldg(&p.chunk_info[t.chunk]);
      const int pos0 = ci.y, nt = ci.z;
      const int nk = t.gu ? KB1 : KB2;
      const uint32_t ks0 = ks;
      ks += nk;
      const uint32_t slot = su % kV4Slots;
      if (ok && !mbar_wait_bounded(&acc_full[slot], (su / kV4Slots) & 1)) ok = false;
      tc::fence_after_sync();
      float accg[kV4Chunk], accu[kV4Chunk];
#pragma unroll
      for (int i = 0; i < kV4Chunk; ++i) accg[i] = accu[i] = 0.f;
      const uint32_t ta = tbase + slot * kV4SlotCols + ((32u * q) << 16);
      // both issuers' halves (a single K block: only its issuer's)
      const int h0 = nk > 1 ? 0 : static_cast<int>(ks0 & 1u), h1 = nk > 1 ? 2 : h0 + 1;
      for (int hf = h0; hf < h1; ++hf) {
        uint32_t vg[16], vu[16];
        tc::tmem_ld16(ta + hf * 32, vg);
        if (t.gu) tc::tmem_ld16(ta + hf * 32 + kV4Chunk, vu);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < kV4Chunk; ++i) {
          accg[i] = __fadd_rn(accg[i], __uint_as_float(vg[i]));
          if (t.gu) accu[i] = __fadd_rn(accu[i], __uint_as_float(vu[i]));
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[slot]);
      ++su;
      if (!ok) {
#pragma unroll
        for (int i = 0; i < kV4Chunk; ++i) accg[i] = accu[i] = 0.f;
      }
      if (t.gu) {
        // SwiGLU row r of the chunk's tokens (fp4_gemm outputs are bf16), then the
        // ue8m0 act_quant of the 128-block straight into the chunk's down B block
        float h[kV4Chunk];
#pragma unroll
        for (int i = 0; i < kV4Chunk; ++i) {
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
        for (int i = 0; i < kV4Chunk; ++i) {
          const float a = v4_warp_max(fabsf(h[i]));
          if (lane == 0) red[q * kV4Chunk + i] = a;
        }
        named_barrier_sync(1, 128);
        int e_mine = 0;
#pragma unroll
        for (int i = 0; i < kV4Chunk; ++i) {
          const float a = fmaxf(fmaxf(red[i], red[kV4Chunk + i]),
                                fmaxf(red[2 * kV4Chunk + i], red[3 * kV4Chunk + i]));
          const int e = ue8m0_exp(a, kV4Inv448);
          if (i == (r & (kV4Chunk - 1))) e_mine = e;
          hst[(r >> 4) * 256 + (i >> 3) * 128 + (i & 7) * 16 + (r & 15)] =
              static_cast<uint8_t>(to_e4m3(__fmul_rn(h[i], exp2_int(-e))));
        }
        if (r < 32) {   // scale chunk: token r's e8m0 (rows past the chunk: 1.0)
          const uint32_t b = r < kV4Chunk ? static_cast<uint32_t>(e_mine + 127) * 0x01010101u : 0x7F7F7F7Fu;
          *reinterpret_cast<uint4*>(hst + kV4BTile + r * 16) = make_uint4(b, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
        }
        named_barrier_sync(1, 128);
        uint8_t* tile = p.hb + (static_cast<size_t>(t.chunk) * KB2 + t.mt) * kV4BBytes;
        *reinterpret_cast<uint4*>(tile + r * 16) = *reinterpret_cast<const uint4*>(hst + r * 16);
        if (r < 32)
          *reinterpret_cast<uint4*>(tile + kV4BTile + r * 16) =
              *reinterpret_cast<const uint4*>(hst + kV4BTile + r * 16);
        fence_proxy_async_global();
        __threadfence();
        named_barrier_sync(1, 128);
        if (r == 0) atomicAdd(&p.chunk_done[t.chunk], 1);
      } else {
        const int col = t.mt * 128 + r;
#pragma unroll
        for (int i = 0; i < kV4Chunk; ++i) {
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

int launch_v4_experts(const flyai_moe_desc& d, int M, const flyai_moe_weights& w, void* y,
                      uint16_t* rows, const Fp8Workspace& ws, cudaStream_t stream, cudaEvent_t ev0,
                      cudaEvent_t ev1, const int32_t* slot_of, int slots) {
  if (M == 0) return FLYAI_OK;
  const int P = M * d.top_k;
  V4ScatterParams sp{ws.xq, ws.xs, ws.perm, ws.n_chunks, ws.chunk_info, ws.xb, d.hidden, d.top_k, P};
  if (v4_launch(v4_scatter_kernel, dim3((d.hidden / 128 + 7) / 8, f8_max_chunks(d, M)), 256, 0, stream,
                true, sp) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();

  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem = v4_smem_bytes();
  if (smem > static_cast<size_t>(max_smem)) return FLYAI_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(v4_moe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  V4Params prm{};
  prm.w13 = static_cast<const uint8_t*>(w.w13);
  prm.w2 = static_cast<const uint8_t*>(w.w2);
  prm.b13 = v4_bank(d, FLYAI_PROJ_W13);
  prm.b2 = v4_bank(d, FLYAI_PROJ_W2);
  prm.El = d.expert_end - d.expert_begin;
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
  prm.slot_of = slot_of;
  prm.slots = slot_of ? slots : 0;
  if (ev0 && ev1 && cudaEventRecord(ev0, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  if (v4_launch(v4_moe_kernel, dim3(sms), kV4Threads, smem, stream, true, prm) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  note_launch();
  if (ev0 && ev1 && cudaEventRecord(ev1, stream) != cudaSuccess) return FLYAI_ERR_CUDA;
  return y ? launch_fp8_combine(d, M, rows, y, ws, stream, false) : FLYAI_OK;
}

}  // namespace flyai
