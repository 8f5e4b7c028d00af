#pragma once
// torch's CPU topk order, restated for the device.
//
// Every reference router in scope selects experts with torch.topk on CPU.  torch
// (aten/src/ATen/native/cpu/SortingKernel.cpp topk_impl_loop) builds (value,
// index) pairs and runs std::partial_sort(q, q+k, q+n, greater) when
// 64*k <= n, else std::nth_element(q, q+k-1, q+n, greater) followed, when
// sorted, by std::sort(q, q+k-1, greater); greater(x, y) = (isnan(x) &&
// !isnan(y)) || x > y on the values.  With sorted=False (DeepSeek-V3's
// KimiMoEGate, vendor/kimi_k3_ref/modeling_kimi_linear.py:727-739; MiniMax-M2's
// MiniMaxM2TopKRouter) the returned order is whatever libstdc++'s introselect
// leaves in q[0..k), so reproducing the reference's ids slot by slot means
// reproducing that algorithm.  The serial routines below restate libstdc++'s
// published __introselect, __move_median_to_first, __unguarded_partition,
// __insertion_sort and the heap routines step for step (one lane, shared
// memory); torch_topk_warp runs the same introselect with one warp, computing
// each Hoare partition in parallel (see kv_partition_warp).
#include <cstdint>

namespace flyai {

struct KV {
  float v;
  int i;
};

__device__ __forceinline__ bool kv_gt(const KV& x, const KV& y) {
  return (isnan(x.v) && !isnan(y.v)) || x.v > y.v;
}

__device__ inline void kv_insertion_sort(KV* a, int f, int l) {
  if (f == l) return;
  for (int i = f + 1; i < l; ++i) {
    KV v = a[i];
    if (kv_gt(v, a[f])) {
      for (int j = i; j > f; --j) a[j] = a[j - 1];
      a[f] = v;
    } else {
      int j = i, n = i - 1;
      while (kv_gt(v, a[n])) {
        a[j] = a[n];
        j = n;
        --n;
      }
      a[j] = v;
    }
  }
}

__device__ __forceinline__ void kv_swap(KV* a, int i, int j) {
  KV t = a[i];
  a[i] = a[j];
  a[j] = t;
}

// The position whose element __move_median_to_first(r, x, y, z) swaps into r.
__device__ __forceinline__ int kv_median_of(const KV* a, int x, int y, int z) {
  if (kv_gt(a[x], a[y])) {
    if (kv_gt(a[y], a[z])) return y;
    if (kv_gt(a[x], a[z])) return z;
    return x;
  }
  if (kv_gt(a[x], a[z])) return x;
  if (kv_gt(a[y], a[z])) return z;
  return y;
}

__device__ inline void kv_move_median_to_first(KV* a, int r, int x, int y, int z) {
  kv_swap(a, r, kv_median_of(a, x, y, z));
}

__device__ inline int kv_unguarded_partition(KV* a, int f, int l, int p) {
  while (true) {
    while (kv_gt(a[f], a[p])) ++f;
    --l;
    while (kv_gt(a[p], a[l])) --l;
    if (!(f < l)) return f;
    kv_swap(a, f, l);
    ++f;
  }
}

__device__ inline void kv_adjust_heap(KV* a, int first, int hole, int len, KV value) {
  const int top = hole;
  int second = hole;
  while (second < (len - 1) / 2) {
    second = 2 * (second + 1);
    if (kv_gt(a[first + second], a[first + second - 1])) --second;
    a[first + hole] = a[first + second];
    hole = second;
  }
  if ((len & 1) == 0 && second == (len - 2) / 2) {
    second = 2 * (second + 1);
    a[first + hole] = a[first + second - 1];
    hole = second - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && kv_gt(a[first + parent], value)) {
    a[first + hole] = a[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  a[first + hole] = value;
}

__device__ inline void kv_heap_select(KV* a, int f, int m, int l) {
  const int n = m - f;
  if (n >= 2) {
    for (int parent = (n - 2) / 2;; --parent) {
      kv_adjust_heap(a, f, parent, n, a[f + parent]);
      if (parent == 0) break;
    }
  }
  for (int i = m; i < l; ++i) {
    if (kv_gt(a[i], a[f])) {
      KV v = a[i];
      a[i] = a[f];
      kv_adjust_heap(a, f, 0, n, v);
    }
  }
}

__device__ inline void kv_sort_heap(KV* a, int f, int l) {
  while (l - f > 1) {
    --l;
    KV v = a[l];
    a[l] = a[f];
    kv_adjust_heap(a, f, 0, l - f, v);
  }
}

__device__ __forceinline__ int ilog2_floor(int n) { return 31 - __clz(n); }

// Leaves torch.topk(values, k, sorted)'s index order in a[0..k).  One thread.
__device__ inline void torch_topk_serial(KV* a, int n, int k, bool sorted) {
  if (k * 64 <= n) {
    kv_heap_select(a, 0, k, n);
    kv_sort_heap(a, 0, k);
    return;
  }
  int f = 0, l = n;
  const int nth = k - 1;
  int depth = 2 * ilog2_floor(n);
  while (l - f > 3) {
    if (depth == 0) {
      kv_heap_select(a, f, nth + 1, l);
      kv_swap(a, f, nth);
      goto selected;
    }
    --depth;
    {
      const int mid = f + (l - f) / 2;
      kv_move_median_to_first(a, f, f + 1, mid, l - 1);
      const int cut = kv_unguarded_partition(a, f + 1, l, f);
      if (cut <= nth) f = cut;
      else l = cut;
    }
  }
  kv_insertion_sort(a, f, l);
selected:
  if (sorted) kv_insertion_sort(a, 0, k - 1);
}

// Rows up to this many elements go through torch_topk_warp.
constexpr int kTopkWarpMaxN = 512;

// __unguarded_partition(a, F0, L0, p) by one warp, same result.  Sequentially
// the left scan stops at "left stoppers" (!greater(a[j], pivot)) and the right
// scan at "right stoppers" (!greater(pivot, a[j])); every swap exchanges the
// i-th left stopper counted from F0 with the i-th right stopper counted down
// from L0, until the two meet.  Swapped elements are never examined again and
// each scan stops at the latest on the element the other scan swapped in, so
// with nL(q) = left stoppers before q and nR(q) = right stoppers after q (all
// in the array as it is when the partition starts): a left stopper swaps iff
// nR > nL, a right stopper iff nL > nR, partner = the right stopper whose nR
// equals the left stopper's nL, and with s swaps the scan ends at
// cut = min(s-th left stopper, (s-1)-th right stopper).  rpos: 256 shorts of
// warp-private shared memory.  All lanes return the cut.
__device__ inline int kv_partition_warp(KV* a, int F0, int L0, int p, uint32_t* msk, int16_t* rpos) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u, gtm = ~lt & ~(1u << lane);
  const KV P = a[p];
  const int nc = (L0 - F0 + 31) >> 5;
  for (int c = 0; c < nc; ++c) {
    const int pos = F0 + (c << 5) + lane;
    bool ls = false, rs = false;
    if (pos < L0) {
      const KV x = a[pos];
      ls = !kv_gt(x, P);
      rs = !kv_gt(P, x);
    }
    const uint32_t bl = __ballot_sync(0xffffffffu, ls), br = __ballot_sync(0xffffffffu, rs);
    if (lane == 0) {
      msk[c] = bl;
      msk[16 + c] = br;
    }
  }
  __syncwarp();
  int tot_r = 0;
  for (int c = 0; c < nc; ++c) tot_r += __popc(msk[16 + c]);
  int below_l = 0, above_r = tot_r, swaps = 0;
  uint32_t my_swaps = 0;
  for (int c = 0; c < nc; ++c) {
    const uint32_t L = msk[c], R = msk[16 + c];
    above_r -= __popc(R);
    const int nl = below_l + __popc(L & lt), nr = above_r + __popc(R & gtm);
    const bool is_l = (L >> lane) & 1u, is_r = (R >> lane) & 1u;
    const bool sw_l = is_l && nr > nl;
    if (is_r && nl > nr) rpos[nr] = static_cast<int16_t>(F0 + (c << 5) + lane);
    if (sw_l) my_swaps |= 1u << c;
    swaps += __popc(__ballot_sync(0xffffffffu, sw_l));
    below_l += __popc(L);
  }
  __syncwarp();
  int cand = L0;
  below_l = 0;
  for (int c = 0; c < nc; ++c) {
    const uint32_t L = msk[c];
    const int nl = below_l + __popc(L & lt), pos = F0 + (c << 5) + lane;
    if ((my_swaps >> c) & 1u) kv_swap(a, pos, rpos[nl]);
    if (((L >> lane) & 1u) && nl == swaps) cand = pos;
    below_l += __popc(L);
  }
  if (swaps > 0) cand = min(cand, static_cast<int>(rpos[swaps - 1]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
  __syncwarp();
  return cand;
}

// torch.topk(values, k, sorted=False)'s order in a[0..k), by one warp: the
// introselect loop of torch_topk_serial with its partitions run by
// kv_partition_warp; the heap paths (64*k <= n, depth limit) and the final
// insertion sort of at most three elements run on lane 0.  n <= kTopkWarpMaxN.
// scratch: warp-private shared memory of kTopkWarpScratch bytes, 4-aligned.
constexpr int kTopkWarpScratch = 32 * 4 + 256 * 2;
__device__ inline void torch_topk_warp(KV* a, int n, int k, void* scratch) {
  const int lane = threadIdx.x & 31;
  uint32_t* msk = static_cast<uint32_t*>(scratch);
  int16_t* rpos = reinterpret_cast<int16_t*>(msk + 32);
  __syncwarp();
  if (k * 64 <= n) {
    if (lane == 0) {
      kv_heap_select(a, 0, k, n);
      kv_sort_heap(a, 0, k);
    }
    __syncwarp();
    return;
  }
  int f = 0, l = n;
  const int nth = k - 1;
  int depth = 2 * ilog2_floor(n);
  while (l - f > 3) {
    if (depth == 0) {
      if (lane == 0) {
        kv_heap_select(a, f, nth + 1, l);
        kv_swap(a, f, nth);
      }
      __syncwarp();
      return;
    }
    --depth;
    const int mid = f + (l - f) / 2;
    const int med = kv_median_of(a, f + 1, mid, l - 1);
    __syncwarp();
    if (lane == 0) kv_swap(a, f, med);
    __syncwarp();
    const int cut = kv_partition_warp(a, f + 1, l, f, msk, rpos);
    if (cut <= nth) f = cut;
    else l = cut;
  }
  if (lane == 0) kv_insertion_sort(a, f, l);
  __syncwarp();
}

}  // namespace flyai
