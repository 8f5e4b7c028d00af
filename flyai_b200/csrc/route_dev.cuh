// Device pieces of the GPT-OSS routing shared by the route kernels (route.cu),
// the fused verify layer (tc_experts.cu) and the combine kernels (combine.cu):
// exact bf16 router logits, torch-identical top-k with the bf16 softmax over the
// selected logits, and a token's slots in ascending expert id (the order of the
// reference's index_add_ loop).
//
// Reference: transformers/models/gpt_oss/modeling_gpt_oss.py:117-131
// (GptOssTopKRouter.forward) and :96-112 (the expert loop's index_add_).
#pragma once
#include "common.cuh"
#include "torch_topk.cuh"

namespace flyai {

// ---------------------------------------------------------------------------
// 1) logits = round_bf16(x . W_r^T + b): one warp per (token, expert).
// bf16*bf16 products are exact in fp32; summing them in fp64 makes the sum
// exact to far below one bf16 ulp, so the single rounding reproduces the
// reference CPU F.linear (which rounds once after fp32 accumulation) except
// where that fp32 accumulation itself strays across a rounding boundary.
// ---------------------------------------------------------------------------
__device__ inline float logit_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
                            const uint16_t* __restrict__ br, int m, int e, int H) {
  const int lane = threadIdx.x & 31;
  const uint16_t* xr = x + static_cast<size_t>(m) * H;
  const uint16_t* w = wr + static_cast<size_t>(e) * H;
  double acc = 0.0;
  for (int k0 = lane * 8; k0 < H; k0 += 256) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + k0);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + k0);
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x0 = __uint_as_float(xs[i] << 16), x1 = __uint_as_float(xs[i] & 0xFFFF0000u);
      const float w0 = __uint_as_float(ws[i] << 16), w1 = __uint_as_float(ws[i] & 0xFFFF0000u);
      acc += static_cast<double>(__fmul_rn(x0, w0));
      acc += static_cast<double>(__fmul_rn(x1, w1));
    }
  }
  acc = warp_sum_f64(acc);
  const double b = br ? static_cast<double>(bf16_bits_to_float(br[e])) : 0.0;
  return bf16r(__double2float_rn(acc + b));
}

// ---------------------------------------------------------------------------
// 2) torch CPU topk (sorted=True for GPT-OSS), via torch_topk.cuh's
// restatement of libstdc++'s selection, run by one lane on a shared-memory copy
// of the row when the fast path below cannot decide.
// ---------------------------------------------------------------------------

// Orderable key of a bf16-valued fp32 logit and its expert index: a larger
// value gives a larger key, equal values the lower index (-0 counts as +0, as
// torch's comparison does).  Values differ iff the keys' upper halves differ.
__device__ __forceinline__ uint32_t topk_key(float v, int j) {
  uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (b & 0xFFFF0000u) | (0xFFFFu - static_cast<uint32_t>(j));
}

// One warp selects one token.  Fast path: when the k+1 largest values are
// strictly decreasing (and nothing is NaN) the answer is unique -- the k
// largest in descending order -- and is found with k+1 rounds of a warp
// max-reduction over (value, index) keys.  Any tie or NaN falls back to the
// libstdc++ restatement: torch_topk_warp (the introselect with warp-parallel
// partitions) followed by std::sort's insertion sort of the first k-1 on one
// lane -- torch.topk(sorted=True) -- given kTopkWarpScratch bytes of
// warp-private shared memory in topk_scratch and a row of at most
// kTopkWarpMaxN; else torch_topk_serial on one lane.  The softmax runs on lanes
// 0..k-1 with the reference's fp32 sum order.
__device__ inline void select_softmax_token(const float* __restrict__ lr, KV* row, int m, int E, int k,
                                     int32_t* __restrict__ ids, float* __restrict__ wts,
                                     int32_t* __restrict__ ids_out, uint16_t* __restrict__ wts_out,
                                     void* topk_scratch = nullptr) {
  const int lane = threadIdx.x & 31;
  bool nan_seen = false;
  for (int j = lane; j < E; j += 32) {
    const float v = lr[j];
    row[j] = KV{v, j};
    nan_seen |= isnan(v);
  }
  __syncwarp();
  const bool any_nan = __any_sync(0xffffffffu, nan_seen);

  const int want = (k < E) ? k + 1 : k;
  int my_i = 0;          // lane r < k: index of the r-th selected expert
  bool distinct = !any_nan;
  if (distinct) {
    // lanes own j = lane + 32*t; 'taken' bit t marks an element already chosen
    uint32_t taken = 0, prev = 0xFFFFFFFFu;
#pragma unroll
    for (int r = 0; r < kMaxTopK + 1; ++r) {
      if (r >= want) break;
      uint32_t best = 0;
      for (int t = 0, j = lane; j < E; ++t, j += 32)
        if (!((taken >> t) & 1u)) best = max(best, topk_key(row[j].v, j));
      const uint32_t w = __reduce_max_sync(0xffffffffu, best);
      const int bi = static_cast<int>(0xFFFFu - (w & 0xFFFFu));
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      if (r == lane) my_i = bi;
      distinct &= (w >> 16) < (prev >> 16);
      prev = w;
    }
  }
  if (!distinct) {
    if (topk_scratch && E <= kTopkWarpMaxN) {
      torch_topk_warp(row, E, k, topk_scratch);   // leaves sorted=False's order
      if (lane == 0 && k * 64 > E) kv_insertion_sort(row, 0, k - 1);
    } else if (lane == 0) {
      torch_topk_serial(row, E, k, true);
    }
    __syncwarp();
    if (lane < k) my_i = row[lane].i;
    __syncwarp();
  }
  // softmax over the k selected bf16 logits in fp32, rounded to bf16
  // (torch.nn.functional.softmax(top, dim=1, dtype=bfloat16)): lane r owns slot r
  const float my_v = lane < k ? lr[my_i] : -INFINITY;
  float mx = my_v;
  for (int r = 1; r < k; ++r) mx = fmaxf(mx, __shfl_sync(0xffffffffu, my_v, r));
  mx = __shfl_sync(0xffffffffu, lane == 0 ? mx : 0.f, 0);
  const float ex = lane < k ? expf(__fsub_rn(my_v, mx)) : 0.f;
  float s = 0.f;
  for (int r = 0; r < k; ++r) s = __fadd_rn(s, __shfl_sync(0xffffffffu, ex, r));
  if (lane < k) {
    const float w = bf16r(__fdiv_rn(ex, s));
    const size_t p = static_cast<size_t>(m) * k + lane;
    ids[p] = my_i;
    wts[p] = w;
    if (ids_out) ids_out[p] = my_i;
    if (wts_out) wts_out[p] = float_to_bf16_bits(w);
  }
  __syncwarp();
}

// The token's k slots in ascending expert id (ids of one token are distinct).
__device__ __forceinline__ void slots_by_expert(const int32_t* __restrict__ ids, int m, int k,
                                                int* order) {
  int eid[kMaxTopK];
  for (int s = 0; s < k; ++s) {
    order[s] = s;
    eid[s] = ids[m * k + s];
  }
  for (int i = 1; i < k; ++i) {
    const int o = order[i], v = eid[i];
    int j = i;
    while (j > 0 && eid[j - 1] > v) {
      eid[j] = eid[j - 1];
      order[j] = order[j - 1];
      --j;
    }
    eid[j] = v;
    order[j] = o;
  }
}

}  // namespace flyai
