// extern "C" boundary: validation, workspace planning and launch sequencing.
// Every entry point returns a status code; nothing aborts.
#include <atomic>
#include <cstring>

#include "common.cuh"
#include "fp8_moe.cuh"
#include "route.cuh"
#include "tc_bank.cuh"

namespace flyai {

static std::atomic<int64_t> g_launches{0};
void note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

static bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// The FP8 and NVFP4 layers share the routing plan, workspace and combine
// (fp8_moe.cu); their expert kernels differ.
static bool is_fp8(const flyai_moe_desc& d) {
  return d.format == FLYAI_FMT_FP8_BLOCK || d.format == FLYAI_FMT_NVFP4 ||
         d.format == FLYAI_FMT_FP4_W4A8;
}

static int check_desc(const flyai_moe_desc* d) {
  if (!d) return FLYAI_ERR_INVALID_ARG;
  if (d->abi_version != FLYAI_MOE_ABI_VERSION) return FLYAI_ERR_ABI;
  for (int i = 0; i < 4; ++i)
    if (d->reserved[i] != 0) return FLYAI_ERR_INVALID_ARG;
  if (d->num_experts < 1 || d->num_experts > 1024) return FLYAI_ERR_INVALID_ARG;
  const int max_k = d->gating == FLYAI_GATE_EXTERNAL ? kMaxTopKExternal : kMaxTopK;
  if (d->top_k < 1 || d->top_k > max_k || d->top_k > d->num_experts)
    return FLYAI_ERR_INVALID_ARG;
  if (d->hidden < 32 || d->inter < 32) return FLYAI_ERR_INVALID_ARG;
  if (d->hidden % 32 || d->inter % 32) return FLYAI_ERR_ALIGNMENT;
  if (d->expert_begin < 0 || d->expert_end > d->num_experts || d->expert_begin > d->expert_end)
    return FLYAI_ERR_INVALID_ARG;
  if (d->max_tokens < 0) return FLYAI_ERR_INVALID_ARG;
  if (d->format == FLYAI_FMT_MXFP4) {
    // GPT-OSS (SwiGLU) routed here, or routed by the caller (token-sharded expert
    // parallel: the pairs another rank sent); Kimi-K3 (situ, routed by the caller)
    const bool ext = d->gating == FLYAI_GATE_EXTERNAL;
    const bool k3 = ext && d->activation == FLYAI_ACT_SITU;
    if (!ext && d->gating != FLYAI_GATE_SOFTMAX_TOPK) return FLYAI_ERR_UNSUPPORTED;
    if (!k3 && d->activation != FLYAI_ACT_GPTOSS_SWIGLU) return FLYAI_ERR_UNSUPPORTED;
    // the tcgen05 kernels: K-tiles of 64, one tensor-memory accumulator row block
    if (d->hidden % 64 || d->inter % 64) return FLYAI_ERR_ALIGNMENT;
    if (d->hidden > kTcMaxK || d->inter > kTcMaxK) return FLYAI_ERR_UNSUPPORTED;
    if (d->n_group != 0 || d->topk_group != 0 || d->route_scale != 0.f || d->n_shared != 0)
      return FLYAI_ERR_INVALID_ARG;
    if (k3) {
      // beta > 0, linear_beta >= 0 (0 = None); the verify-size kernels only
      if (!(d->swiglu_alpha > 0.f) || !(d->swiglu_limit >= 0.f)) return FLYAI_ERR_INVALID_ARG;
      if (d->max_tokens >= kTcPrefillMinTokens) return FLYAI_ERR_UNSUPPORTED;
      return FLYAI_OK;
    }
    if (!(d->swiglu_limit > 0.f) || !(d->swiglu_alpha > 0.f)) return FLYAI_ERR_INVALID_ARG;
    return FLYAI_OK;
  }
  if (d->format == FLYAI_FMT_FP8_BLOCK) {
    if (d->gating != FLYAI_GATE_SIGMOID_GROUP) return FLYAI_ERR_UNSUPPORTED;
    if (d->activation != FLYAI_ACT_SILU) return FLYAI_ERR_UNSUPPORTED;
    if (d->hidden % kF8Blk || d->inter % kF8Blk) return FLYAI_ERR_ALIGNMENT;
    if (d->num_experts % 32 || d->num_experts > kF8MaxExperts) return FLYAI_ERR_UNSUPPORTED;
    if (d->n_group < 1 || d->n_group > 32 || d->num_experts % d->n_group || d->topk_group < 1 ||
        d->topk_group > d->n_group)
      return FLYAI_ERR_INVALID_ARG;
    if (d->top_k > d->topk_group * (d->num_experts / d->n_group)) return FLYAI_ERR_INVALID_ARG;
    if (!(d->route_scale > 0.f) || d->n_shared < 0 || d->n_shared > 1) return FLYAI_ERR_INVALID_ARG;
    if (!(d->swiglu_limit >= 0.f) || d->swiglu_alpha != 0.f) return FLYAI_ERR_INVALID_ARG;
    if (d->max_tokens > kF8MaxTokens) return FLYAI_ERR_UNSUPPORTED;
    return FLYAI_OK;
  }
  if (d->format == FLYAI_FMT_FP4_W4A8) {
    if (d->gating != FLYAI_GATE_SQRTSOFTPLUS) return FLYAI_ERR_UNSUPPORTED;
    if (d->activation != FLYAI_ACT_SILU) return FLYAI_ERR_UNSUPPORTED;
    if (d->hidden % 128 || d->inter % 128) return FLYAI_ERR_ALIGNMENT;
    if (d->num_experts % 32 || d->num_experts > kF8MaxExperts) return FLYAI_ERR_UNSUPPORTED;
    if (d->n_group != 1 || d->topk_group != 1) return FLYAI_ERR_INVALID_ARG;
    if (!(d->route_scale > 0.f) || d->n_shared < 0 || d->n_shared > 1) return FLYAI_ERR_INVALID_ARG;
    if (!(d->swiglu_limit >= 0.f) || d->swiglu_alpha != 0.f) return FLYAI_ERR_INVALID_ARG;
    if (d->max_tokens > kF8MaxTokens) return FLYAI_ERR_UNSUPPORTED;
    return FLYAI_OK;
  }
  if (d->format == FLYAI_FMT_NVFP4) {
    if (d->gating != FLYAI_GATE_SIGMOID_BF16) return FLYAI_ERR_UNSUPPORTED;
    if (d->activation != FLYAI_ACT_SILU_BF16) return FLYAI_ERR_UNSUPPORTED;
    if (d->hidden % 128 || d->inter % 128) return FLYAI_ERR_ALIGNMENT;
    if (d->num_experts % 32 || d->num_experts > kF8MaxExperts) return FLYAI_ERR_UNSUPPORTED;
    if (d->n_group != 1 || d->topk_group != 1 || !(d->route_scale > 0.f) || d->n_shared != 0)
      return FLYAI_ERR_INVALID_ARG;
    if (d->swiglu_limit != 0.f || d->swiglu_alpha != 0.f) return FLYAI_ERR_INVALID_ARG;
    if (d->max_tokens > kNvPfMaxTokens) return FLYAI_ERR_UNSUPPORTED;   // > 64: prefill path
    return FLYAI_OK;
  }
  return FLYAI_ERR_UNSUPPORTED;
}


// The FP8 layer computes on one GPU holding every routed expert (a partial
// range is only meaningful for packing a slice of the bank).
static int check_fp8_compute(const flyai_moe_desc& d) {
  return (d.expert_begin == 0 && d.expert_end == d.num_experts) ? FLYAI_OK : FLYAI_ERR_UNSUPPORTED;
}

static size_t workspace_total(const flyai_moe_desc& d) {
  return is_fp8(d) ? carve_fp8_workspace(d, d.max_tokens, nullptr).total
                   : carve_workspace(d, d.max_tokens, nullptr).total;
}

static int check_tokens(const flyai_moe_desc* d, int32_t M) {
  if (M < 0 || M > d->max_tokens) return FLYAI_ERR_INVALID_ARG;
  return FLYAI_OK;
}

static int check_workspace(const flyai_moe_desc* d, void* ws, size_t bytes) {
  if (!ws || bytes < workspace_total(*d)) return FLYAI_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return FLYAI_ERR_ALIGNMENT;
  return FLYAI_OK;
}

static int check_weights(const flyai_moe_desc* d, const flyai_moe_weights* w, bool need_router,
                         bool need_experts) {
  if (!w) return FLYAI_ERR_INVALID_ARG;
  if (need_router) {
    if (!w->router_w) return FLYAI_ERR_INVALID_ARG;
    if (!aligned(w->router_w, 16)) return FLYAI_ERR_ALIGNMENT;
  }
  if (need_experts && d->expert_end > d->expert_begin) {
    if (!w->w13 || !w->w2) return FLYAI_ERR_INVALID_ARG;
    if (!aligned(w->w13, 16) || !aligned(w->w2, 16)) return FLYAI_ERR_ALIGNMENT;
    if ((w->w13_bias && !aligned(w->w13_bias, 4)) || (w->w2_bias && !aligned(w->w2_bias, 4)))
      return FLYAI_ERR_ALIGNMENT;
  }
  return FLYAI_OK;
}

static std::atomic<cudaEvent_t> g_prof_start{nullptr}, g_prof_stop{nullptr};

// Expert projections of the FP8 / NVFP4 layers on the plan their route left in
// the workspace; NVFP4 batches above kF8MaxTokens take the prefill kernel.
static int launch_layer_experts(const flyai_moe_desc& d, int M, const void* x,
                                const flyai_moe_weights& w, void* y, uint16_t* rows,
                                const Fp8Workspace& fw, cudaStream_t s) {
  if (d.format == FLYAI_FMT_NVFP4) {
    if (M > kF8MaxTokens)
      return launch_nvp_experts(d, M, w, y, rows, fw, s, g_prof_start.load(), g_prof_stop.load());
    return launch_nv4_experts(d, M, x, w, y, rows, fw, s, g_prof_start.load(), g_prof_stop.load());
  }
  if (d.format == FLYAI_FMT_FP4_W4A8)
    return launch_v4_experts(d, M, w, y, rows, fw, s, g_prof_start.load(), g_prof_stop.load());
  return launch_fp8_experts(d, M, x, w, y, rows, fw, s, g_prof_start.load(), g_prof_stop.load());
}

static int launch_layer_route(const flyai_moe_desc& d, int M, const void* x,
                              const flyai_moe_weights& w, float* logits, int32_t* topk_ids,
                              float* topk_weights, const Fp8Workspace& fw, cudaStream_t s,
                              const void* logits_in = nullptr) {
  if (d.format == FLYAI_FMT_NVFP4 && M > kF8MaxTokens)
    return launch_nvp_route(d, M, x, w, logits, topk_ids, topk_weights, fw, s, logits_in);
  return launch_fp8_route(d, M, x, w, logits, topk_ids, topk_weights, fw, s, nullptr, nullptr, 0,
                          logits_in);
}

// Expert projections: the tcgen05 block-scaled kernels (every MXFP4 descriptor
// check_desc accepts; the bank was packed in their layout).
static int launch_experts(const flyai_moe_desc& d, int M, const void* x, bool x_split,
                          const flyai_moe_weights& w, uint16_t* pair_out, bool zero_pairs,
                          const Workspace& ws, cudaStream_t s, void* y_fold = nullptr,
                          bool* folded = nullptr) {
  const cudaEvent_t e0 = g_prof_start.load(), e1 = g_prof_stop.load();
  if (e0 && e1 && cudaEventRecord(e0, s) != cudaSuccess) return FLYAI_ERR_CUDA;
  const int st = launch_tc_experts(d, M, x, x_split, w, pair_out, zero_pairs, ws, s, y_fold, folded);
  if (st == FLYAI_OK && e0 && e1 && cudaEventRecord(e1, s) != cudaSuccess) return FLYAI_ERR_CUDA;
  return st;
}

}  // namespace flyai

using namespace flyai;

#define FLYAI_TRY(expr)            \
  do {                             \
    const int _s = (expr);         \
    if (_s != FLYAI_OK) return _s; \
  } while (0)

extern "C" {

int flyai_moe_abi_version(void) { return FLYAI_MOE_ABI_VERSION; }

const char* flyai_moe_strerror(int status) {
  switch (status) {
    case FLYAI_OK: return "ok";
    case FLYAI_ERR_INVALID_ARG: return "invalid argument";
    case FLYAI_ERR_UNSUPPORTED: return "unsupported format/gating/activation combination";
    case FLYAI_ERR_ALIGNMENT: return "alignment requirement violated";
    case FLYAI_ERR_WORKSPACE: return "workspace missing or too small";
    case FLYAI_ERR_CUDA: return "CUDA launch or runtime error";
    case FLYAI_ERR_ABI: return "descriptor ABI version mismatch";
    default: return "unknown status";
  }
}

int flyai_moe_check_desc(const flyai_moe_desc* desc) { return check_desc(desc); }

int64_t flyai_moe_launch_count(void) { return g_launches.load(); }

int flyai_moe_set_profile_events(void* start, void* stop) {
  g_prof_start.store(static_cast<cudaEvent_t>(start));
  g_prof_stop.store(static_cast<cudaEvent_t>(stop));
  return FLYAI_OK;
}

int flyai_moe_packed_bytes(const flyai_moe_desc* desc, int32_t proj, size_t* bytes) {
  FLYAI_TRY(check_desc(desc));
  if (!bytes || (proj != FLYAI_PROJ_W13 && proj != FLYAI_PROJ_W2)) return FLYAI_ERR_INVALID_ARG;
  *bytes = desc->format == FLYAI_FMT_NVFP4     ? nv4_packed_bytes(*desc, proj)
           : desc->format == FLYAI_FMT_FP4_W4A8 ? v4_packed_bytes(*desc, proj)
           : is_fp8(*desc)                 ? fp8_packed_bytes(*desc, proj)
                                           : tc_packed_bytes(*desc, proj);
  return FLYAI_OK;
}

int flyai_moe_pack_mxfp4(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                         const void* scales, void* packed, void* stream) {
  FLYAI_TRY(check_desc(desc));
  if (proj != FLYAI_PROJ_W13 && proj != FLYAI_PROJ_W2) return FLYAI_ERR_INVALID_ARG;
  if (is_fp8(*desc)) return FLYAI_ERR_UNSUPPORTED;   // flyai_moe_pack_fp8
  if (desc->expert_end == desc->expert_begin) return FLYAI_OK;
  if (!blocks || !scales || !packed) return FLYAI_ERR_INVALID_ARG;
  if (!aligned(blocks, 16) || !aligned(packed, 16)) return FLYAI_ERR_ALIGNMENT;
  return launch_tc_pack(*desc, proj, blocks, scales, packed, static_cast<cudaStream_t>(stream));
}

int flyai_moe_pack_fp8(const flyai_moe_desc* desc, int32_t proj, const void* weight,
                       const void* scale, void* packed, void* stream) {
  FLYAI_TRY(check_desc(desc));
  if (proj != FLYAI_PROJ_W13 && proj != FLYAI_PROJ_W2) return FLYAI_ERR_INVALID_ARG;
  if (desc->format != FLYAI_FMT_FP8_BLOCK) return FLYAI_ERR_UNSUPPORTED;
  if (desc->expert_end - desc->expert_begin + desc->n_shared == 0) return FLYAI_OK;
  if (!weight || !scale || !packed) return FLYAI_ERR_INVALID_ARG;
  if (!aligned(weight, 16) || !aligned(packed, 16) || !aligned(scale, 4)) return FLYAI_ERR_ALIGNMENT;
  return launch_fp8_pack(*desc, proj, weight, scale, packed, static_cast<cudaStream_t>(stream));
}

int flyai_moe_pack_fp4(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                       const void* scales, void* packed, void* stream) {
  FLYAI_TRY(check_desc(desc));
  if (proj != FLYAI_PROJ_W13 && proj != FLYAI_PROJ_W2) return FLYAI_ERR_INVALID_ARG;
  if (desc->format != FLYAI_FMT_FP4_W4A8) return FLYAI_ERR_UNSUPPORTED;
  if (desc->expert_end == desc->expert_begin) return FLYAI_OK;
  if (!blocks || !scales || !packed) return FLYAI_ERR_INVALID_ARG;
  if (!aligned(blocks, 16) || !aligned(packed, 16) || !aligned(scales, 4)) return FLYAI_ERR_ALIGNMENT;
  return launch_v4_pack_fp4(*desc, proj, blocks, scales, packed, static_cast<cudaStream_t>(stream));
}

int flyai_moe_pack_shared_fp8(const flyai_moe_desc* desc, int32_t proj, const void* weight,
                              const void* scale, void* packed, void* stream) {
  FLYAI_TRY(check_desc(desc));
  if (proj != FLYAI_PROJ_W13 && proj != FLYAI_PROJ_W2) return FLYAI_ERR_INVALID_ARG;
  if (desc->format != FLYAI_FMT_FP4_W4A8) return FLYAI_ERR_UNSUPPORTED;
  if (desc->n_shared == 0) return FLYAI_OK;
  if (!weight || !scale || !packed) return FLYAI_ERR_INVALID_ARG;
  if (!aligned(weight, 16) || !aligned(packed, 16)) return FLYAI_ERR_ALIGNMENT;
  return launch_v4_pack_shared(*desc, proj, weight, scale, packed, static_cast<cudaStream_t>(stream));
}

static int pack_nvfp4(const flyai_moe_desc* desc, int32_t proj, const void* blocks, const void* scales,
                      const void* global_scale, void* packed, void* stream, bool swizzled) {
  FLYAI_TRY(check_desc(desc));
  if (proj != FLYAI_PROJ_W13 && proj != FLYAI_PROJ_W2) return FLYAI_ERR_INVALID_ARG;
  if (desc->format != FLYAI_FMT_NVFP4) return FLYAI_ERR_UNSUPPORTED;
  if (desc->expert_end - desc->expert_begin + desc->n_shared == 0) return FLYAI_OK;
  if (!blocks || !scales || !global_scale || !packed) return FLYAI_ERR_INVALID_ARG;
  if (!aligned(blocks, 16) || !aligned(packed, 16) || !aligned(global_scale, 4))
    return FLYAI_ERR_ALIGNMENT;
  return launch_nv4_pack(*desc, proj, blocks, scales, global_scale, packed,
                         static_cast<cudaStream_t>(stream), swizzled);
}

int flyai_moe_pack_nvfp4(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                         const void* scales, const void* global_scale, void* packed, void* stream) {
  return pack_nvfp4(desc, proj, blocks, scales, global_scale, packed, stream, false);
}

int flyai_moe_pack_nvfp4_swizzled(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                                  const void* scales, const void* global_scale, void* packed,
                                  void* stream) {
  return pack_nvfp4(desc, proj, blocks, scales, global_scale, packed, stream, true);
}

int flyai_moe_workspace_bytes(const flyai_moe_desc* desc, size_t* bytes) {
  FLYAI_TRY(check_desc(desc));
  if (!bytes) return FLYAI_ERR_INVALID_ARG;
  *bytes = workspace_total(*desc);
  return FLYAI_OK;
}

int flyai_moe_route(const flyai_moe_desc* desc, int32_t M, const void* x,
                    const flyai_moe_weights* w, void* logits, int32_t* topk_ids,
                    void* topk_weights, void* workspace, size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  if (desc->gating == FLYAI_GATE_EXTERNAL) return FLYAI_ERR_UNSUPPORTED;   // flyai_moe_route_ids
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, true, false));
  if (M > 0 && !x) return FLYAI_ERR_INVALID_ARG;
  if (x && !aligned(x, 16)) return FLYAI_ERR_ALIGNMENT;
  if (is_fp8(*desc)) {   // partial expert ranges route too (expert parallel)
    if (!w->router_b || !aligned(w->router_b, 4)) return FLYAI_ERR_INVALID_ARG;
    const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
    return launch_layer_route(*desc, M, x, *w, static_cast<float*>(logits), topk_ids,
                              static_cast<float*>(topk_weights), fw, static_cast<cudaStream_t>(stream));
  }
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  return launch_route(*desc, M, x, *w, logits, topk_ids, topk_weights, ws,
                      static_cast<cudaStream_t>(stream));
}

int flyai_moe_route_hash(const flyai_moe_desc* desc, int32_t M, const void* x, const int32_t* input_ids,
                         const int32_t* tid2eid, int32_t vocab, const flyai_moe_weights* w, void* logits,
                         int32_t* topk_ids, void* topk_weights, void* workspace,
                         size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, true, false));
  if (desc->gating != FLYAI_GATE_SQRTSOFTPLUS) return FLYAI_ERR_UNSUPPORTED;
  if (M > 0 && (!x || !input_ids || !tid2eid)) return FLYAI_ERR_INVALID_ARG;
  if (vocab < 1) return FLYAI_ERR_INVALID_ARG;
  if (x && !aligned(x, 16)) return FLYAI_ERR_ALIGNMENT;
  if ((input_ids && !aligned(input_ids, 4)) || (tid2eid && !aligned(tid2eid, 4))) return FLYAI_ERR_ALIGNMENT;
  if (!w->router_b || !aligned(w->router_b, 4)) return FLYAI_ERR_INVALID_ARG;
  const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
  return launch_fp8_route(*desc, M, x, *w, static_cast<float*>(logits), topk_ids,
                          static_cast<float*>(topk_weights), fw, static_cast<cudaStream_t>(stream),
                          tid2eid, input_ids, vocab);
}

int flyai_moe_route_logits(const flyai_moe_desc* desc, int32_t M, const void* x,
                           const void* router_logits, const flyai_moe_weights* w, int32_t* topk_ids,
                           void* topk_weights, void* workspace, size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, true, false));
  if (desc->gating != FLYAI_GATE_SIGMOID_BF16) return FLYAI_ERR_UNSUPPORTED;
  if (M > 0 && (!x || !router_logits)) return FLYAI_ERR_INVALID_ARG;
  if ((x && !aligned(x, 16)) || (router_logits && !aligned(router_logits, 16))) return FLYAI_ERR_ALIGNMENT;
  if (!w->router_b || !aligned(w->router_b, 4)) return FLYAI_ERR_INVALID_ARG;
  const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
  return launch_layer_route(*desc, M, x, *w, nullptr, topk_ids, static_cast<float*>(topk_weights), fw,
                            static_cast<cudaStream_t>(stream), router_logits);
}

int flyai_moe_route_ids(const flyai_moe_desc* desc, int32_t M, const int32_t* topk_ids,
                        const float* topk_weights, void* workspace, size_t workspace_bytes,
                        void* stream) {
  FLYAI_TRY(check_desc(desc));
  if (desc->gating != FLYAI_GATE_EXTERNAL) return FLYAI_ERR_UNSUPPORTED;
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  if (M > 0 && (!topk_ids || !topk_weights)) return FLYAI_ERR_INVALID_ARG;
  if ((topk_ids && !aligned(topk_ids, 4)) || (topk_weights && !aligned(topk_weights, 4)))
    return FLYAI_ERR_ALIGNMENT;
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  return launch_route_ids(*desc, M, topk_ids, topk_weights, ws, static_cast<cudaStream_t>(stream));
}

int flyai_moe_read_plan(const flyai_moe_desc* desc, int32_t M, const void* workspace,
                        size_t workspace_bytes, int32_t* counts, int32_t* offsets, int32_t* perm,
                        void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, const_cast<void*>(workspace), workspace_bytes));
  void* base = const_cast<void*>(workspace);
  const int32_t *w_counts, *w_offsets, *w_perm;
  if (is_fp8(*desc)) {
    const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, base);
    w_counts = fw.counts, w_offsets = fw.offsets, w_perm = fw.perm;
  } else {
    const Workspace ws = carve_workspace(*desc, desc->max_tokens, base);
    w_counts = ws.counts, w_offsets = ws.offsets, w_perm = ws.perm;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t El = desc->expert_end - desc->expert_begin;
  const size_t P = static_cast<size_t>(M) * desc->top_k;
  if (counts && El && cudaMemcpyAsync(counts, w_counts, El * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (offsets && cudaMemcpyAsync(offsets, w_offsets, (El + 1) * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (perm && P && cudaMemcpyAsync(perm, w_perm, P * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  return FLYAI_OK;
}

int flyai_moe_read_error(const flyai_moe_desc* desc, const void* workspace,
                         size_t workspace_bytes, int32_t* out, int32_t clear, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_workspace(desc, const_cast<void*>(workspace), workspace_bytes));
  if (!out) return FLYAI_ERR_INVALID_ARG;
  void* base = const_cast<void*>(workspace);
  int32_t *err, *dbg;
  if (is_fp8(*desc)) {
    const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, base);
    err = fw.err, dbg = fw.dbg;
  } else {
    const Workspace ws = carve_workspace(*desc, desc->max_tokens, base);
    err = ws.err, dbg = ws.dbg;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(out, err, 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(out + 1, dbg, 32, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return FLYAI_ERR_CUDA;
  if (clear && (cudaMemsetAsync(err, 0, 4, s) != cudaSuccess ||
                cudaMemsetAsync(dbg, 0, 32, s) != cudaSuccess))
    return FLYAI_ERR_CUDA;
  return FLYAI_OK;
}

int flyai_moe_experts_pairs(const flyai_moe_desc* desc, int32_t M, const void* x,
                            const flyai_moe_weights* w, void* pair_out, void* workspace,
                            size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, false, true));
  if (M > 0 && (!x || !pair_out)) return FLYAI_ERR_INVALID_ARG;
  if (is_fp8(*desc)) {
    if ((x && !aligned(x, 16)) || (pair_out && !aligned(pair_out, 16))) return FLYAI_ERR_ALIGNMENT;
    if (M == 0) return FLYAI_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
    // rows of other shards' experts (and of the shared expert off its shard) stay zero
    if (cudaMemsetAsync(pair_out, 0, layer_pair_rows(*desc, M) * desc->hidden * 2, s) != cudaSuccess)
      return FLYAI_ERR_CUDA;
    return launch_layer_experts(*desc, M, x, *w, nullptr, static_cast<uint16_t*>(pair_out), fw, s);
  }
  if ((x && !aligned(x, 16)) || (pair_out && !aligned(pair_out, 16))) return FLYAI_ERR_ALIGNMENT;
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  return launch_experts(*desc, M, x, false, *w, static_cast<uint16_t*>(pair_out), true, ws,
                        static_cast<cudaStream_t>(stream));
}

int flyai_moe_combine(const flyai_moe_desc* desc, int32_t M, const void* pair_out, void* y,
                      void* workspace, size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  if (M > 0 && (!pair_out || !y)) return FLYAI_ERR_INVALID_ARG;
  if (is_fp8(*desc)) {
    if ((pair_out && !aligned(pair_out, 16)) || (y && !aligned(y, 16))) return FLYAI_ERR_ALIGNMENT;
    const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
    return launch_fp8_combine(*desc, M, static_cast<const uint16_t*>(pair_out), y, fw,
                              static_cast<cudaStream_t>(stream), desc->format == FLYAI_FMT_NVFP4);
  }
  if ((pair_out && !aligned(pair_out, 4)) || (y && !aligned(y, 4))) return FLYAI_ERR_ALIGNMENT;
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  return launch_combine(*desc, M, static_cast<const uint16_t*>(pair_out), y, ws,
                        static_cast<cudaStream_t>(stream));
}

int flyai_moe_experts(const flyai_moe_desc* desc, int32_t M, const void* x,
                      const flyai_moe_weights* w, void* y, void* workspace,
                      size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, false, true));
  if (M > 0 && (!x || !y)) return FLYAI_ERR_INVALID_ARG;
  if ((x && !aligned(x, 16)) || (y && !aligned(y, 4))) return FLYAI_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (is_fp8(*desc)) {
    FLYAI_TRY(check_fp8_compute(*desc));
    if (y && !aligned(y, 16)) return FLYAI_ERR_ALIGNMENT;
    const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
    return launch_layer_experts(*desc, M, x, *w, y, fw.rows, fw, s);
  }
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  const bool partial = (desc->expert_end - desc->expert_begin) != desc->num_experts;
  bool folded = false;
  FLYAI_TRY(launch_experts(*desc, M, x, false, *w, ws.pair_out, partial, ws, s,
                           partial ? nullptr : y, &folded));
  return folded ? FLYAI_OK : launch_combine(*desc, M, ws.pair_out, y, ws, s);
}

int flyai_moe_experts_slots(const flyai_moe_desc* desc, int32_t M, const void* x,
                            const flyai_moe_weights* w, const int32_t* slot_of, int32_t slots,
                            void* y, void* workspace, size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  if (desc->format != FLYAI_FMT_FP4_W4A8) return FLYAI_ERR_UNSUPPORTED;
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, false, true));
  FLYAI_TRY(check_fp8_compute(*desc));
  if (slots < 1 || !slot_of) return FLYAI_ERR_INVALID_ARG;
  if (M > 0 && (!x || !y)) return FLYAI_ERR_INVALID_ARG;
  if ((x && !aligned(x, 16)) || (y && !aligned(y, 16)) || !aligned(slot_of, 4))
    return FLYAI_ERR_ALIGNMENT;
  const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
  return launch_v4_experts(*desc, M, *w, y, fw.rows, fw, static_cast<cudaStream_t>(stream),
                           g_prof_start.load(), g_prof_stop.load(), slot_of, slots);
}

int flyai_moe_forward(const flyai_moe_desc* desc, int32_t M, const void* x,
                      const flyai_moe_weights* w, void* y, int32_t* topk_ids,
                      void* topk_weights, void* workspace, size_t workspace_bytes,
                      void* stream) {
  FLYAI_TRY(check_desc(desc));
  // caller-routed layers: flyai_moe_route_ids + flyai_moe_experts
  if (desc->gating == FLYAI_GATE_EXTERNAL) return FLYAI_ERR_UNSUPPORTED;
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, true, true));
  if (M > 0 && (!x || !y)) return FLYAI_ERR_INVALID_ARG;
  if ((x && !aligned(x, 16)) || (y && !aligned(y, 4))) return FLYAI_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (is_fp8(*desc)) {
    FLYAI_TRY(check_fp8_compute(*desc));
    if (!w->router_b || !aligned(w->router_b, 4)) return FLYAI_ERR_INVALID_ARG;
    if (y && !aligned(y, 16)) return FLYAI_ERR_ALIGNMENT;
    const Fp8Workspace fw = carve_fp8_workspace(*desc, desc->max_tokens, workspace);
    FLYAI_TRY(launch_layer_route(*desc, M, x, *w, nullptr, topk_ids,
                                 static_cast<float*>(topk_weights), fw, s));
    return launch_layer_experts(*desc, M, x, *w, y, fw.rows, fw, s);
  }
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  if (tc_fused_supported(*desc, M)) {   // verify size: the layer is one launch
    const cudaEvent_t e0 = g_prof_start.load(), e1 = g_prof_stop.load();
    if (e0 && e1 && cudaEventRecord(e0, s) != cudaSuccess) return FLYAI_ERR_CUDA;
    FLYAI_TRY(launch_tc_forward(*desc, M, x, *w, y, topk_ids, topk_weights, ws, s));
    if (e0 && e1 && cudaEventRecord(e1, s) != cudaSuccess) return FLYAI_ERR_CUDA;
    return FLYAI_OK;
  }
  FLYAI_TRY(launch_route(*desc, M, x, *w, nullptr, topk_ids, topk_weights, ws, s));
  const bool partial = (desc->expert_end - desc->expert_begin) != desc->num_experts;
  bool folded = false;
  FLYAI_TRY(launch_experts(*desc, M, x, true, *w, ws.pair_out, partial, ws, s,
                           partial ? nullptr : y, &folded));
  return folded ? FLYAI_OK : launch_combine(*desc, M, ws.pair_out, y, ws, s);
}

static size_t ep_rows_bytes(const flyai_moe_desc& d) {
  return static_cast<size_t>(d.max_tokens) * d.top_k * d.hidden * 2;
}

int flyai_moe_ep_mailbox_bytes(const flyai_moe_desc* desc, size_t* bytes) {
  FLYAI_TRY(check_desc(desc));
  if (!bytes) return FLYAI_ERR_INVALID_ARG;
  *bytes = kEpFlagBytes + 2 * ep_rows_bytes(*desc);
  return FLYAI_OK;
}

int flyai_moe_ep_alloc(size_t bytes, void** mailbox) {
  if (!mailbox || bytes < static_cast<size_t>(kEpFlagBytes)) return FLYAI_ERR_INVALID_ARG;
  if (cudaMalloc(mailbox, bytes) != cudaSuccess) return FLYAI_ERR_CUDA;
  if (cudaMemset(*mailbox, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(*mailbox);
    *mailbox = nullptr;
    return FLYAI_ERR_CUDA;
  }
  return FLYAI_OK;
}

int flyai_moe_ep_free(void* mailbox) {
  return (mailbox && cudaFree(mailbox) != cudaSuccess) ? FLYAI_ERR_CUDA : FLYAI_OK;
}

int flyai_moe_ipc_get_handle(void* mailbox, void* handle64) {
  if (!mailbox || !handle64) return FLYAI_ERR_INVALID_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, mailbox) != cudaSuccess) return FLYAI_ERR_CUDA;
  memcpy(handle64, &h, sizeof(h));
  return FLYAI_OK;
}

int flyai_moe_ipc_open(const void* handle64, void** mailbox) {
  if (!mailbox || !handle64) return FLYAI_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return cudaIpcOpenMemHandle(mailbox, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? FLYAI_OK
             : FLYAI_ERR_CUDA;
}

int flyai_moe_ipc_close(void* mailbox) {
  return (mailbox && cudaIpcCloseMemHandle(mailbox) != cudaSuccess) ? FLYAI_ERR_CUDA : FLYAI_OK;
}

static int check_ep(const flyai_moe_desc* desc, int32_t M, const flyai_moe_ep_peers* ep) {
  if (!ep || ep->world < 2 || ep->world > FLYAI_MOE_EP_MAX_RANKS || ep->rank < 0 ||
      ep->rank >= ep->world || ep->epoch == 0 || ep->reserved != 0)
    return FLYAI_ERR_INVALID_ARG;
  for (int r = 0; r < ep->world; ++r)
    if (!ep->mailbox[r] || !aligned(ep->mailbox[r], 256)) return FLYAI_ERR_INVALID_ARG;
  // peer-memory exchange exists for the GPT-OSS MXFP4 tcgen05 verify kernel only
  if (is_fp8(*desc) || M >= kTcPrefillMinTokens || desc->gating == FLYAI_GATE_EXTERNAL)
    return FLYAI_ERR_UNSUPPORTED;
  return FLYAI_OK;
}

int flyai_moe_experts_ep(const flyai_moe_desc* desc, int32_t M, const void* x,
                         const flyai_moe_weights* w, const flyai_moe_ep_peers* peers,
                         void* workspace, size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, false, true));
  FLYAI_TRY(check_ep(desc, M, peers));
  if (M > 0 && !x) return FLYAI_ERR_INVALID_ARG;
  if (x && !aligned(x, 16)) return FLYAI_ERR_ALIGNMENT;
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaEvent_t e0 = g_prof_start.load(), e1 = g_prof_stop.load();
  if (e0 && e1 && cudaEventRecord(e0, s) != cudaSuccess) return FLYAI_ERR_CUDA;
  const int st = launch_tc_experts(*desc, M, x, false, *w, nullptr, false, ws, s, nullptr, nullptr,
                                   peers);
  if (st == FLYAI_OK && e0 && e1 && cudaEventRecord(e1, s) != cudaSuccess) return FLYAI_ERR_CUDA;
  return st;
}

int flyai_moe_forward_ep(const flyai_moe_desc* desc, int32_t M, const void* x,
                         const flyai_moe_weights* w, const flyai_moe_ep_peers* peers, int32_t* topk_ids,
                         void* topk_weights, void* workspace, size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_weights(desc, w, true, true));
  FLYAI_TRY(check_ep(desc, M, peers));
  if (M > 0 && !x) return FLYAI_ERR_INVALID_ARG;
  if (x && !aligned(x, 16)) return FLYAI_ERR_ALIGNMENT;
  if (!tc_fused_supported(*desc, M, true)) return FLYAI_ERR_UNSUPPORTED;
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaEvent_t e0 = g_prof_start.load(), e1 = g_prof_stop.load();
  if (e0 && e1 && cudaEventRecord(e0, s) != cudaSuccess) return FLYAI_ERR_CUDA;
  FLYAI_TRY(launch_tc_forward(*desc, M, x, *w, nullptr, topk_ids, topk_weights, ws, s, peers));
  if (e0 && e1 && cudaEventRecord(e1, s) != cudaSuccess) return FLYAI_ERR_CUDA;
  return FLYAI_OK;
}

int flyai_moe_combine_ep(const flyai_moe_desc* desc, int32_t M, const flyai_moe_ep_peers* peers,
                         void* y, void* workspace, size_t workspace_bytes, void* stream) {
  FLYAI_TRY(check_desc(desc));
  FLYAI_TRY(check_tokens(desc, M));
  FLYAI_TRY(check_workspace(desc, workspace, workspace_bytes));
  FLYAI_TRY(check_ep(desc, M, peers));
  if (M > 0 && !y) return FLYAI_ERR_INVALID_ARG;
  if (y && !aligned(y, 4)) return FLYAI_ERR_ALIGNMENT;
  const Workspace ws = carve_workspace(*desc, desc->max_tokens, workspace);
  return launch_combine_ep(*desc, M, *peers, y, ws, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
