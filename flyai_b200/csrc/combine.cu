// Weighted combine of the MXFP4 layers.  GPT-OSS: y[t] = bf16 fold of the
// token's k weighted expert rows in ascending expert id with a bf16 rounding
// after every add -- the order and rounding of the reference's index_add_ loop
// (transformers/models/gpt_oss/modeling_gpt_oss.py:96-112).  One CTA per
// (token, 2048 output columns), launched with programmatic dependent launch
// behind the expert kernel.
#include "common.cuh"
#include "route.cuh"
#include "route_dev.cuh"

namespace flyai {

// Columns [o, o + 8) of token m: every slot's 8 values loaded before the folds.
__device__ __forceinline__ void fold_rows(const uint16_t* __restrict__ rows, const int* order,
                                          int m, int k, int H, bool live, uint16_t* __restrict__ y) {
  for (int o = (blockIdx.y * blockDim.x + threadIdx.x) * 8; o < H; o += gridDim.y * blockDim.x * 8) {
    uint32_t v[kMaxTopK][4];
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s)
      if (s < k && live) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(
            rows + (static_cast<size_t>(m) * k + order[s]) * H + o);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[s][j] = __ldcg(src + j);
      }
    uint32_t out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int s = 0; s < kMaxTopK; ++s)
        if (s < k && live) {
          a0 = bf16r(__fadd_rn(a0, __uint_as_float(v[s][j] << 16)));
          a1 = bf16r(__fadd_rn(a1, __uint_as_float(v[s][j] & 0xFFFF0000u)));
        }
      out[j] = static_cast<uint32_t>(float_to_bf16_bits(a0)) |
               (static_cast<uint32_t>(float_to_bf16_bits(a1)) << 16);
    }
    uint32_t* dst = reinterpret_cast<uint32_t*>(y + static_cast<size_t>(m) * H + o);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = out[j];
  }
}

__global__ void __launch_bounds__(256) combine_kernel(const uint16_t* __restrict__ pair_out,
                                                      const int32_t* __restrict__ ids, int k,
                                                      int H, uint16_t* __restrict__ y) {
  pdl_wait();   // the expert kernel's pair rows are complete
  int order[kMaxTopK];
  slots_by_expert(ids, blockIdx.x, k, order);
  fold_rows(pair_out, order, blockIdx.x, k, H, true, y);
}

// Kimi-K3 (FLYAI_ACT_SITU): y[t] = bf16 of the fp32 sum over the k slots, in slot
// order, of (bf16 w2 row) x (fp32 routing weight) -- moe_infer's
// new_x.view(T, k, H).type(fp32).mul_(w).sum(dim=1).type(bf16)
// (vendor/kimi_k3_ref/modeling_kimi_linear.py:868-874).  The pair rows are unweighted.
__global__ void __launch_bounds__(256) combine_slots_kernel(const uint16_t* __restrict__ pair_out,
                                                            const float* __restrict__ wts, int k,
                                                            int H, uint16_t* __restrict__ y) {
  pdl_wait();
  const int m = blockIdx.x;
  float w[kMaxTopKExternal];
#pragma unroll
  for (int s = 0; s < kMaxTopKExternal; ++s) w[s] = s < k ? __ldg(&wts[m * k + s]) : 0.f;
  for (int o = (blockIdx.y * blockDim.x + threadIdx.x) * 8; o < H; o += gridDim.y * blockDim.x * 8) {
    uint4 v[kMaxTopKExternal];
#pragma unroll
    for (int s = 0; s < kMaxTopKExternal; ++s)
      if (s < k)
        v[s] = __ldcg(reinterpret_cast<const uint4*>(pair_out + (static_cast<size_t>(m) * k + s) * H + o));
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxTopKExternal; ++s) {
      if (s < k) {
        const uint32_t u[4] = {v[s].x, v[s].y, v[s].z, v[s].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = __fmul_rn(__uint_as_float(u[j] << 16), w[s]);
          const float hi = __fmul_rn(__uint_as_float(u[j] & 0xFFFF0000u), w[s]);
          acc[2 * j] = s == 0 ? lo : __fadd_rn(acc[2 * j], lo);
          acc[2 * j + 1] = s == 0 ? hi : __fadd_rn(acc[2 * j + 1], hi);
        }
      }
    }
    uint4 out;
    out.x = float_to_bf16_bits(acc[0]) | (static_cast<uint32_t>(float_to_bf16_bits(acc[1])) << 16);
    out.y = float_to_bf16_bits(acc[2]) | (static_cast<uint32_t>(float_to_bf16_bits(acc[3])) << 16);
    out.z = float_to_bf16_bits(acc[4]) | (static_cast<uint32_t>(float_to_bf16_bits(acc[5])) << 16);
    out.w = float_to_bf16_bits(acc[6]) | (static_cast<uint32_t>(float_to_bf16_bits(acc[7])) << 16);
    *reinterpret_cast<uint4*>(y + static_cast<size_t>(m) * H + o) = out;
  }
}

// Expert-parallel combine: wait (bounded, ~2 s) until every rank raised its flag
// in this rank's mailbox to the call's epoch, then fold as combine_kernel does.
// A rank whose expert kernel gave up on a wait raises its failure word to the
// epoch before its flag; then, as on expiry, the fold is skipped (y = 0) and the
// workspace error word gets kErrWaitTimeout.
__global__ void __launch_bounds__(256) combine_ep_kernel(const uint16_t* __restrict__ rows,
                                                         const uint32_t* flags, int world,
                                                         uint32_t epoch, const int32_t* __restrict__ ids,
                                                         int k, int H, uint16_t* __restrict__ y,
                                                         int32_t* err) {
  __shared__ int ready;
  pdl_wait();
  if (threadIdx.x == 0) {
    bool good = true;
    const uint64_t t0 = global_ns();
    for (int r = 0; r < world && good; ++r) {
      while (true) {
        uint32_t f;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(f) : "l"(flags + r) : "memory");
        if (static_cast<int32_t>(f - epoch) >= 0) break;
        if (global_ns() - t0 > 2000000000ull) {
          good = false;
          break;
        }
        __nanosleep(64);
      }
      if (good) {
        uint32_t fail;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n"
                     : "=r"(fail)
                     : "l"(flags + kEpFailWord + r)
                     : "memory");
        if (fail == epoch) good = false;
      }
    }
    if (!good) atomicOr(err, kErrWaitTimeout);
    ready = good;
  }
  __syncthreads();
  int order[kMaxTopK];
  slots_by_expert(ids, blockIdx.x, k, order);
  fold_rows(rows, order, blockIdx.x, k, H, ready != 0, y);
}

static cudaError_t launch_fold(const flyai_moe_desc& d, int M, cudaStream_t stream, void (*kern)(),
                               void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, (d.hidden + 2047) / 2048);   // 8 columns per thread
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kern), args);
}

int launch_combine_ep(const flyai_moe_desc& d, int M, const flyai_moe_ep_peers& ep, void* y,
                      const Workspace& ws, cudaStream_t stream) {
  if (M == 0) return FLYAI_OK;
  const size_t rows_bytes = static_cast<size_t>(d.max_tokens) * d.top_k * d.hidden * 2;
  const uint8_t* mb = static_cast<const uint8_t*>(ep.mailbox[ep.rank]);
  const uint16_t* rows = reinterpret_cast<const uint16_t*>(mb + kEpFlagBytes + (ep.epoch & 1) * rows_bytes);
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(mb);
  int world = ep.world, k = d.top_k, H = d.hidden;
  uint32_t epoch = ep.epoch;
  const int32_t* ids = ws.ids;
  uint16_t* yo = static_cast<uint16_t*>(y);
  int32_t* err = ws.err;
  void* args[] = {&rows, &flags, &world, &epoch, &ids, &k, &H, &yo, &err};
  const cudaError_t st = launch_fold(d, M, stream, reinterpret_cast<void (*)()>(combine_ep_kernel), args);
  note_launch();
  return st == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

int launch_combine(const flyai_moe_desc& d, int M, const uint16_t* pair_out, void* y,
                   const Workspace& ws, cudaStream_t stream) {
  if (M == 0) return FLYAI_OK;
  const int32_t* ids = ws.ids;
  const float* wts = ws.wts;
  int k = d.top_k, H = d.hidden;
  uint16_t* yo = static_cast<uint16_t*>(y);
  void* args[] = {&pair_out, &ids, &k, &H, &yo};
  void* args_slots[] = {&pair_out, &wts, &k, &H, &yo};
  const cudaError_t st =
      d.activation == FLYAI_ACT_SITU
          ? launch_fold(d, M, stream, reinterpret_cast<void (*)()>(combine_slots_kernel), args_slots)
          : launch_fold(d, M, stream, reinterpret_cast<void (*)()>(combine_kernel), args);
  note_launch();
  return st == cudaSuccess ? FLYAI_OK : FLYAI_ERR_CUDA;
}

}  // namespace flyai
