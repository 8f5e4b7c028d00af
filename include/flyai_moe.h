/*
 * flyai_moe.h -- C ABI of the B200 (sm_100a) quantized MoE expert forward.
 *
 * One MoE layer = router top-k + gating -> token->expert histogram and
 * permutation -> quantized gate/up projection with clamped SwiGLU -> down
 * projection -> weighted combine.  Every entry point is stream-ordered, does
 * no host synchronisation and no allocation (the caller passes a workspace
 * sized by flyai_moe_workspace_bytes), and returns 0 or a negative
 * FLYAI_ERR_* code.  Nothing here aborts or traps on bad input.
 *
 * Reference interfaces these entry points replace (paths inside the FlyAI
 * project; "transformers/" = the HuggingFace package the reference loads):
 *   - GptOssMLP.forward(hidden) -> (out, router_scores)
 *       transformers/models/gpt_oss/modeling_gpt_oss.py:140-146
 *     (router :117-131, experts :69-114), loaded by phase0/pipeline.py:126-182
 *     with the packed MXFP4 layout pinned by phase0/mxfp4_guard.py:223-276;
 *   - the hub MXFP4 forward mlp_forward / Mxfp4GptOssExperts.forward
 *       transformers/integrations/mxfp4.py:389-411, 493-511;
 *   - MoE.forward / Gate.forward / Expert.forward of the DeepSeek reference
 *       vendor/deepseek_v4_ref/inference/model.py:569-649;
 *   - KimiMoEGate.forward (DeepSeek-V3 grouped sigmoid gate)
 *       vendor/kimi_k3_ref/modeling_kimi_linear.py:703-759;
 *   - KimiSparseMoeBlock.moe_infer (Kimi-K3 MXFP4 experts with `situ`)
 *       vendor/kimi_k3_ref/modeling_kimi_linear.py:841-875, served on the GPU by
 *       engines/kimi_k3/k3_moe_mxfp4.py:258-412.
 */
#ifndef FLYAI_MOE_H
#define FLYAI_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FLYAI_API __attribute__((visibility("default")))
#else
#define FLYAI_API
#endif

#define FLYAI_MOE_ABI_VERSION 1

/* status codes */
#define FLYAI_OK                 0
#define FLYAI_ERR_INVALID_ARG   -1  /* null pointer, bad enum, inconsistent sizes   */
#define FLYAI_ERR_UNSUPPORTED   -2  /* valid but not implemented combination        */
#define FLYAI_ERR_ALIGNMENT     -3  /* pointer or dimension breaks an alignment rule */
#define FLYAI_ERR_WORKSPACE     -4  /* workspace missing or smaller than required    */
#define FLYAI_ERR_CUDA          -5  /* a CUDA launch or runtime call failed          */
#define FLYAI_ERR_ABI           -6  /* descriptor abi_version mismatch               */

/* weight formats */
#define FLYAI_FMT_MXFP4          1  /* e2m1 nibbles (low nibble = even K) + e8m0 scale per 32 K */
#define FLYAI_FMT_FP8_BLOCK      2  /* e4m3 weights + one fp32 scale per 128x128 block; activations
                                       quantised to e4m3 per 1x128 with an fp32 scale (DeepSeek fp8
                                       Linear: vendor/deepseek_v4_ref/inference/model.py:114-124) */
#define FLYAI_FMT_NVFP4          3  /* e2m1 nibbles (low nibble = even K) + e4m3 scale per 16 K + one
                                       fp32 global scale per tensor (ModelOpt NVFP4, the M2.5
                                       checkpoint format loaded at engines/minimax_m25/m25_stage.py:288-311) */
#define FLYAI_FMT_FP4_W4A8       4  /* DeepSeek-V4 (V4-Flash config: expert_dtype fp4, dtype fp8, scale_fmt
                                       ue8m0): routed experts e2m1 (low nibble = even K) + one e8m0 scale
                                       per 32 K; the shared expert e4m3 + one e8m0 scale per 128x128 block;
                                       activations quantised to e4m3 per 1x128 with power-of-two scales
                                       (vendor/deepseek_v4_ref/inference/model.py:114-158, 592-649) */

/* gating functions */
#define FLYAI_GATE_SOFTMAX_TOPK  1  /* GPT-OSS: bf16 logits = xW^T+b, torch.topk, softmax over the k */
#define FLYAI_GATE_SIGMOID_GROUP 2  /* DeepSeek-V3: fp32 logits, sigmoid, + correction bias for the
                                       choice only, per-group sum of the top-2, top topk_group groups,
                                       top-k inside them, unbiased scores renormalised / (sum + 1e-20)
                                       and x route_scale (modeling_kimi_linear.py:703-759);
                                       router_b = fp32 [E] correction bias, weights fp32 */
#define FLYAI_GATE_SIGMOID_BF16  3  /* MiniMax-M2: bf16 logits = F.linear(x, W) on bf16, sigmoid in fp32,
                                       + correction bias for the choice, top-k, unbiased scores / sum,
                                       x route_scale (transformers/models/minimax_m2/modeling_minimax_m2.py
                                       MiniMaxM2TopKRouter; routed_scaling_factor as m25_stage.py:234-235
                                       passes it to FusedMoE); router_b = fp32 [E] bias, weights fp32 */
#define FLYAI_GATE_SQRTSOFTPLUS  4  /* DeepSeek-V4 Gate.forward (model.py:569-589): fp32 logits of bf16 x
                                       and W, sqrt(softplus), + bias for the choice only, torch.topk
                                       (sorted; torch's CPU order among ties) -- or tid2eid[input_ids] on
                                       a hash-routed layer (flyai_moe_route_hash) --, the unbiased scores
                                       / their sum x route_scale; router_b = fp32 [E], weights fp32 */
#define FLYAI_GATE_EXTERNAL      5  /* Kimi-K3: the caller's router chose the experts -- the seam is
                                       moe_infer(x, topk_ids, topk_weight) (engines/kimi_k3/
                                       k3_moe_mxfp4.py:405-412, vendor/kimi_k3_ref/modeling_kimi_linear.py:
                                       841-875), ids and weights from its KimiMoEGate -- or, with
                                       FLYAI_ACT_GPTOSS_SWIGLU, the (row, expert, weight) pairs another
                                       rank sent for this rank's experts (token-sharded expert parallel);
                                       they enter through flyai_moe_route_ids.  MXFP4 only */

/* expert activations */
#define FLYAI_ACT_GPTOSS_SWIGLU  1  /* interleaved gate/up, clamp(limit), gate*sigmoid(alpha*gate)*(up+1) */
#define FLYAI_ACT_SILU           2  /* gate rows [0,I) (w1), up rows [I,2I) (w3): silu(gate)*up in fp32,
                                       times the routing weight, to bf16 (model.py:599-611, limit 0) */
#define FLYAI_ACT_SILU_BF16      3  /* gate rows [0,I), up rows [I,2I): bf16 silu(gate) * up, down, then
                                       x routing weight (fp32) to bf16, bf16 index_add in ascending
                                       expert id (modeling_minimax_m2.py MiniMaxM2Experts.forward) */
#define FLYAI_ACT_SITU           4  /* Kimi-K3 `situ` (modeling_kimi_linear.py:64-80, 242-268): w1 (gate)
                                       and w3 (up) rows as bf16 Linear outputs, in fp32
                                       beta*tanh(g/beta)*sigmoid(g) * linear_beta*tanh(u/linear_beta) (u
                                       alone when linear_beta is 0), to bf16; w2 to bf16; the fold is the
                                       fp32 sum over the k slots in slot order of row x routing weight, to
                                       bf16 (moe_infer, :841-875).  swiglu_alpha = beta (> 0),
                                       swiglu_limit = linear_beta (>= 0); W13 blocks are [w1; w3]; top_k
                                       up to 16; max_tokens up to 64 (larger batches in 64-token calls) */

/* which projection a packed bank holds */
#define FLYAI_PROJ_W13           0  /* gate/up: rows = 2*inter (interleaved gate,up), K = hidden */
#define FLYAI_PROJ_W2            1  /* down:    rows = hidden,                       K = inter  */

typedef struct flyai_moe_desc {
  int32_t abi_version;    /* = FLYAI_MOE_ABI_VERSION                                   */
  int32_t format;         /* FLYAI_FMT_*                                               */
  int32_t gating;         /* FLYAI_GATE_*                                              */
  int32_t activation;     /* FLYAI_ACT_*                                               */
  int32_t num_experts;    /* E (global)                                                */
  int32_t top_k;          /* k, 1..8                                                   */
  int32_t hidden;         /* H, multiple of 32                                         */
  int32_t inter;          /* I, multiple of 32                                         */
  int32_t expert_begin;   /* experts this process computes: [begin, end)               */
  int32_t expert_end;     /*   (0, E) on one GPU; a contiguous shard under EP          */
  int32_t max_tokens;     /* upper bound on num_tokens the workspace is sized for:     */
                          /*   <= 64 for FP8_BLOCK and FP4_W4A8, <= 8192 for NVFP4      */
                          /*   (calls above 64 tokens take its prefill kernels), any    */
                          /*   for MXFP4                                                */
  float swiglu_limit;     /* GPT-OSS 7.0 (FLYAI_ACT_SILU: 0 = no clamp; SITU: linear_beta) */
  float swiglu_alpha;     /* GPT-OSS 1.702 (FLYAI_ACT_SILU: unused, 0; SITU: beta)       */
  int32_t n_group;        /* FLYAI_GATE_SIGMOID_GROUP: expert groups (1 = ungrouped)   */
  int32_t topk_group;     /*   groups kept, 1..n_group                                 */
  float route_scale;      /*   routed_scaling_factor (DeepSeek-V3 2.5)                 */
  int32_t n_shared;       /* always-on shared experts, 0 or 1 (FLYAI_FMT_FP8_BLOCK)    */
  int32_t reserved[4];    /* must be zero; the four fields above are zero for MXFP4    */
} flyai_moe_desc;

/* Device pointers of one layer.  w13/w2 are banks produced by flyai_moe_pack_mxfp4
 * (a tiled relayout of the reference's [E, R, K/32, 16] blocks + [E, R, K/32]
 * scales) or flyai_moe_pack_fp8; biases stay in the reference's row order.
 * FLYAI_GATE_SIGMOID_GROUP: router_b is the fp32 [E] e_score_correction_bias;
 * FLYAI_FMT_FP8_BLOCK takes no expert biases (NULL). */
typedef struct flyai_moe_weights {
  const void* router_w;   /* bf16 [E, H]                        */
  const void* router_b;   /* bf16 [E]                           */
  const void* w13;        /* packed bank, FLYAI_PROJ_W13        */
  const void* w13_bias;   /* float32 [E, 2I] or NULL            */
  const void* w2;         /* packed bank, FLYAI_PROJ_W2         */
  const void* w2_bias;    /* float32 [E, H]  or NULL            */
} flyai_moe_weights;

/* Library identity. */
FLYAI_API int flyai_moe_abi_version(void);
FLYAI_API const char* flyai_moe_strerror(int status);

/* Validate a descriptor (no device work). */
FLYAI_API int flyai_moe_check_desc(const flyai_moe_desc* desc);

/* Bytes of one packed projection bank for all E experts.
 * Replaces the storage of Mxfp4GptOssExperts.gate_up_proj / down_proj
 * (transformers/integrations/mxfp4.py:365-383; guard phase0/mxfp4_guard.py:223-276). */
FLYAI_API int flyai_moe_packed_bytes(const flyai_moe_desc* desc, int32_t proj, size_t* bytes);

/* Load-time relayout of the reference's MXFP4 storage into the kernel bank.
 * blocks: uint8 [E, R, K/32, 16]; scales: uint8 [E, R, K/32]; packed: flyai_moe_packed_bytes.
 * W13 rows: GPT-OSS's interleaved gate_up_proj; FLYAI_ACT_SITU: w1's rows then w3's (the
 * checkpoint's weight_packed / weight_scale of each, e2m1 low nibble first, e8m0 per 32).
 * Replaces the reference's load-time handling of the same tensors
 * (transformers/integrations/mxfp4.py:279-330 dequantises them instead). */
FLYAI_API int flyai_moe_pack_mxfp4(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                         const void* scales, void* packed, void* stream);

/* Load-time relayout of DeepSeek fp8 expert weights into the kernel bank.
 * weight: e4m3 [El + n_shared, R, K] (the experts of [expert_begin, expert_end)
 * followed by the shared expert), scale: fp32 [El + n_shared, R/128, K/128] -- the
 * reference's Linear.weight / Linear.scale pair (model.py:143-147) with K and R
 * multiples of 128.  FLYAI_PROJ_W13 rows are [w1; w3] stacked (R = 2I, gate rows
 * first), FLYAI_PROJ_W2 rows are w2 (R = H, K = I).  packed: flyai_moe_packed_bytes. */
FLYAI_API int flyai_moe_pack_fp8(const flyai_moe_desc* desc, int32_t proj, const void* weight,
                                 const void* scale, void* packed, void* stream);

/* Load-time relayout of NVFP4 expert weights (ModelOpt: weight uint8 [.., R, K/2],
 * weight_scale e4m3 [.., R, K/16], weight_scale_2 fp32 per tensor) into the kernel
 * bank.  blocks/scales cover the experts of [expert_begin, expert_end) then the
 * shared ones; global_scale is fp32 [El + n_shared] for FLYAI_PROJ_W2 and
 * [El + n_shared, 2] (w1's, w3's) for FLYAI_PROJ_W13, whose rows are [w1; w3]
 * stacked (R = 2I).  K and R multiples of 128.  packed: flyai_moe_packed_bytes. */
FLYAI_API int flyai_moe_pack_nvfp4(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                                   const void* scales, const void* global_scale, void* packed,
                                   void* stream);
/* Same, with the scales in the block-scale layout vLLM swizzles a loaded NVFP4
 * layer into for the CUTLASS / FlashInfer kernels (vllm/model_executor/layers/
 * quantization/utils/nvfp4_utils.py swizzle_blockscale): per expert the [R, K/16]
 * matrix padded to [roundup(R, 128), roundup(K/16, 4)] and stored as
 * [R'/128][C'/4][32][4][4] -- for banks taken from a layer vLLM already loaded. */
FLYAI_API int flyai_moe_pack_nvfp4_swizzled(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                                            const void* scales, const void* global_scale, void* packed,
                                            void* stream);

/* Load-time relayout of DeepSeek-V4 fp4 routed experts into the kernel bank
 * (FLYAI_FMT_FP4_W4A8).  blocks: uint8 [El, R, K/2] packed e2m1 (the checkpoint's
 * float4_e2m1fn_x2 weight, low nibble = even K), scales: uint8 [El, R, K/32] e8m0
 * (its float8_e8m0fnu scale) for the experts of [expert_begin, expert_end);
 * FLYAI_PROJ_W13 rows are [w1; w3] stacked (R = 2I), FLYAI_PROJ_W2 rows are w2.
 * Replaces the per-expert fp4 Linear storage of vendor/deepseek_v4_ref/inference/
 * model.py:133-139 and the bank relayout of engines/deepseek_v4/v4_moe_grouped.py:
 * 376-550.  packed: flyai_moe_packed_bytes (routed experts, then the shared one). */
FLYAI_API int flyai_moe_pack_fp4(const flyai_moe_desc* desc, int32_t proj, const void* blocks,
                                 const void* scales, void* packed, void* stream);

/* The DeepSeek-V4 shared expert into the same bank (after the routed experts):
 * weight e4m3 [n_shared, R, K], scale uint8 [n_shared, R/128, K/128] e8m0 (an fp8
 * Linear of a "scale_dtype fp8" checkpoint, model.py:140-145). */
FLYAI_API int flyai_moe_pack_shared_fp8(const flyai_moe_desc* desc, int32_t proj, const void* weight,
                                        const void* scale, void* packed, void* stream);

/* Workspace bytes for calls with up to desc->max_tokens tokens.  The layout
 * depends only on the descriptor, so one workspace serves every call with
 * num_tokens <= max_tokens.  Zero-fill a workspace once before its first use:
 * its first 276 bytes are counters the kernels keep and restore to zero after
 * every call (also when the workspace is reused with another descriptor). */
FLYAI_API int flyai_moe_workspace_bytes(const flyai_moe_desc* desc, size_t* bytes);

/* Router: logits (bf16 [M, E], may be NULL), topk_ids (int32 [M, k]) and
 * topk_weights (bf16 [M, k]) exactly as GptOssTopKRouter.forward returns them
 * (modeling_gpt_oss.py:125-131), plus the expert histogram and the stable
 * token->expert permutation, which it leaves in the workspace for
 * flyai_moe_experts.  Outputs may be NULL when only the workspace is needed. */
FLYAI_API int flyai_moe_route(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                    const flyai_moe_weights* w, void* logits, int32_t* topk_ids,
                    void* topk_weights, void* workspace, size_t workspace_bytes, void* stream);

/* Router of a hash-routed DeepSeek-V4 layer (layer_id < n_hash_layers): the gate's
 * scores as flyai_moe_route computes them, but the experts of token t are
 * tid2eid[input_ids[t]] (int32 [vocab, k] and int32 [M], device memory) instead of
 * the top-k (model.py:581-582); an expert may repeat within a token, and the fold
 * then keeps only its last slot, as the reference's y[idx] += does
 * (engines/deepseek_v4/v4_moe_grouped.py:623-631).  An input id or table entry
 * out of range sets bit 2 of the error word (flyai_moe_read_error) and reads 0.
 * FLYAI_GATE_SQRTSOFTPLUS descriptors only; then flyai_moe_experts as usual. */
FLYAI_API int flyai_moe_route_hash(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                                   const int32_t* input_ids, const int32_t* tid2eid, int32_t vocab,
                                   const flyai_moe_weights* w, void* logits, int32_t* topk_ids,
                                   void* topk_weights, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* Router of a MiniMax-M2 layer from logits the caller computed: the M2.5 stage
 * computes rl = F.linear(h, gate) (bf16 [M, E]) and hands (h, rl) to its FusedMoE
 * (engines/minimax_m25/m25_stage.py:412-416); this selects from rl -- sigmoid,
 * correction bias, top-k, renormalise -- and builds the plan and token rows as
 * flyai_moe_route does.  FLYAI_GATE_SIGMOID_BF16 descriptors; then
 * flyai_moe_experts. */
FLYAI_API int flyai_moe_route_logits(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                                     const void* router_logits, const flyai_moe_weights* w,
                                     int32_t* topk_ids, void* topk_weights, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* Routing chosen by the caller (FLYAI_GATE_EXTERNAL): topk_ids int32 [M, k] and
 * topk_weights fp32 [M, k] (device) as the reference's gate returned them -- the
 * moe_infer(x, topk_ids, topk_weight) seam of Kimi-K3 (engines/kimi_k3/
 * k3_moe_mxfp4.py:405-412).  Leaves the ids, weights, expert histogram and stable
 * permutation in the workspace for flyai_moe_experts (or _experts_pairs).  An id
 * outside [0, E) is read as 0 and sets bit 2 of the error word. */
FLYAI_API int flyai_moe_route_ids(const flyai_moe_desc* desc, int32_t num_tokens,
                                  const int32_t* topk_ids, const float* topk_weights,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* DeepSeek-V4 routed experts from an expert cache (the reference's RAM expert
 * tier, engines/deepseek_v4/v4_hybrid.py:113-160 / v4_expert_cache.py: the routed
 * experts live in host memory and only a fixed set of device slots holds weights).
 * FLYAI_FMT_FP4_W4A8 only; as flyai_moe_experts after flyai_moe_route /
 * flyai_moe_route_hash, but w->w13 / w->w2 are cache banks laid out as the bank of
 * a descriptor whose expert range holds `slots` experts (flyai_moe_packed_bytes of
 * that descriptor): slot s at s times one expert's packed bytes, the shared expert
 * after the last slot.  slot_of (int32 [expert_end - expert_begin], device) gives
 * the slot of every routed expert; every expert the routing picked must be in a
 * slot (one that is not, or a slot outside [0, slots), reads slot 0 and sets bit 2
 * of the error word).  Output identical to flyai_moe_experts on the full bank. */
FLYAI_API int flyai_moe_experts_slots(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                                      const flyai_moe_weights* w, const int32_t* slot_of,
                                      int32_t slots, void* y, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* Copy the routing plan flyai_moe_route left in the workspace: counts (int32
 * [El]) and exclusive offsets (int32 [El+1]) of this shard's experts, and the
 * permutation (int32 [M*k]): position p holds the flat pair index token*k+slot,
 * grouped by ascending expert and ascending flat index inside an expert -- the
 * stable argsort of the flat ids that the reference's GPU routing uses to gather
 * rows (transformers/integrations/mxfp4.py:473).  Any output may be NULL. */
FLYAI_API int flyai_moe_read_plan(const flyai_moe_desc* desc, int32_t num_tokens, const void* workspace,
                        size_t workspace_bytes, int32_t* counts, int32_t* offsets,
                        int32_t* perm, void* stream);

/* Copy the error word kernels leave in the workspace (bit 1: a bounded wait gave
 * up; bit 2: a bad index -- a self-check enabled with FLYAI_MOE_CHECK=1, or a
 * hash-routing input id or table entry out of range) and 8 words of detail into out (device, int32 [9]); clear != 0 resets
 * them.  Kernels never hang or trap on these conditions: they record and return. */
FLYAI_API int flyai_moe_read_error(const flyai_moe_desc* desc, const void* workspace,
                                   size_t workspace_bytes, int32_t* out, int32_t clear,
                                   void* stream);

/* Routed experts + combine on the routing left in the workspace by flyai_moe_route:
 * y (bf16 [M, H]) = GptOssExperts.forward(x, ids, weights) (modeling_gpt_oss.py:88-114).
 * With a partial expert range, y holds only this shard's experts; use
 * flyai_moe_experts_pairs + flyai_moe_combine around the exchange instead. */
FLYAI_API int flyai_moe_experts(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                      const flyai_moe_weights* w, void* y, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Expert-parallel halves of flyai_moe_experts.  _pairs writes the weighted
 * per-(token, slot) expert outputs of this shard's experts into pair_out
 * (bf16 [M*k, H]; rows of other shards' experts are zeroed), so a sum over
 * ranks (NCCL all-reduce) rebuilds every row exactly; _combine then folds each
 * token's k rows in ascending expert id with bf16 rounding after each add, the
 * order of the reference's index_add_ loop (modeling_gpt_oss.py:96-112).
 * FLYAI_FMT_FP8_BLOCK / FLYAI_FMT_NVFP4: pair_out has M*k + M*n_shared rows
 * (flat pair t*k+slot, then the shared expert's row of token t at M*k + t,
 * written by the shard with expert_begin 0); the fold is the layer's own
 * (fp32 + shared expert, or bf16).  Those formats take partial expert ranges
 * only in flyai_moe_route / _experts_pairs / _combine. */
FLYAI_API int flyai_moe_experts_pairs(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                            const flyai_moe_weights* w, void* pair_out, void* workspace,
                            size_t workspace_bytes, void* stream);
FLYAI_API int flyai_moe_combine(const flyai_moe_desc* desc, int32_t num_tokens, const void* pair_out,
                      void* y, void* workspace, size_t workspace_bytes, void* stream);

/* Expert parallel over NVLink peer memory (the reference's expert-sharded MoE +
 * all_reduce, vendor/deepseek_v4_ref/inference/model.py:640-647, with the
 * exchange fused into the expert kernel).  Every rank owns one mailbox
 * (flyai_moe_ep_alloc, sized by flyai_moe_ep_mailbox_bytes): 256 bytes of flag
 * words, then two buffers of [max_tokens*k, H] bf16 pair rows used by
 * alternating calls.  The mailboxes are shared once with CUDA IPC
 * (flyai_moe_ipc_get_handle on the owner, flyai_moe_ipc_open on every other
 * rank, with that rank's device current).  Per call, after flyai_moe_route on
 * the same tokens: flyai_moe_experts_ep writes each weighted pair row of this
 * rank's experts into every rank's mailbox and then raises this rank's flag in
 * every mailbox to `epoch`; flyai_moe_combine_ep waits (bounded, ~2 s, error
 * word bit 1 on expiry) until every rank's flag in the own mailbox reached
 * `epoch` and folds the rows in ascending expert id.  `epoch` starts at 1 and
 * grows by one per call, identically on every rank.  Only the tcgen05 verify
 * path (num_tokens <= 64) supports it: other cases return FLYAI_ERR_UNSUPPORTED
 * (use flyai_moe_experts_pairs + an all-reduce + flyai_moe_combine). */
#define FLYAI_MOE_EP_MAX_RANKS 8
typedef struct flyai_moe_ep_peers {
  int32_t world;                              /* ranks, 2..8                         */
  int32_t rank;                               /* this rank                           */
  uint32_t epoch;                             /* call number, from 1                 */
  int32_t reserved;                           /* must be zero                        */
  void* mailbox[FLYAI_MOE_EP_MAX_RANKS];      /* rank r's mailbox as mapped here      */
} flyai_moe_ep_peers;
FLYAI_API int flyai_moe_ep_mailbox_bytes(const flyai_moe_desc* desc, size_t* bytes);
FLYAI_API int flyai_moe_ep_alloc(size_t bytes, void** mailbox);   /* cudaMalloc + zero, set-up only */
FLYAI_API int flyai_moe_ep_free(void* mailbox);
FLYAI_API int flyai_moe_ipc_get_handle(void* mailbox, void* handle64);
FLYAI_API int flyai_moe_ipc_open(const void* handle64, void** mailbox);
FLYAI_API int flyai_moe_ipc_close(void* mailbox);
FLYAI_API int flyai_moe_experts_ep(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                                   const flyai_moe_weights* w, const flyai_moe_ep_peers* peers,
                                   void* workspace, size_t workspace_bytes, void* stream);
/* Expert-parallel counterpart of flyai_moe_forward at verify sizes (1..64
 * tokens, at most 256 pairs): ONE cooperative launch per rank routes every token
 * over all experts (the same ids and weights on every rank), runs this rank's
 * experts (desc's expert range) and stores their weighted pair rows into every
 * rank's mailbox, then raises this rank's flag to `epoch` -- the routing and
 * exchange of flyai_moe_route + flyai_moe_experts_ep in one kernel.  Tokens are
 * replicated: every rank passes the same x, as in the reference's
 * expert-sharded MoE (model.py:620-647).  Follow with flyai_moe_combine_ep.
 * topk_ids / topk_weights (bf16) may be NULL.  Other shapes return
 * FLYAI_ERR_UNSUPPORTED. */
FLYAI_API int flyai_moe_forward_ep(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                                   const flyai_moe_weights* w, const flyai_moe_ep_peers* peers,
                                   int32_t* topk_ids, void* topk_weights, void* workspace,
                                   size_t workspace_bytes, void* stream);
FLYAI_API int flyai_moe_combine_ep(const flyai_moe_desc* desc, int32_t num_tokens,
                                   const flyai_moe_ep_peers* peers, void* y, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* The whole layer: route + experts.  GptOssMLP.forward(hidden) -> (out, router_scores)
 * (modeling_gpt_oss.py:140-146): y = out, topk_weights = router_scores.
 * MXFP4 layers of 1..64 tokens with at most 256 (token, slot) pairs on a GPU
 * holding every expert run as ONE cooperative launch (routing, experts and the
 * fold into y; one CTA per SM, which must all be resident: on a GPU whose SMs
 * are partly held by other work the launch fails with FLYAI_ERR_CUDA instead of
 * waiting); that path leaves topk ids/weights in the workspace but not the
 * histogram and permutation flyai_moe_read_plan returns after flyai_moe_route. */
FLYAI_API int flyai_moe_forward(const flyai_moe_desc* desc, int32_t num_tokens, const void* x,
                      const flyai_moe_weights* w, void* y, int32_t* topk_ids,
                      void* topk_weights, void* workspace, size_t workspace_bytes,
                      void* stream);

/* No-allocation variant of flyai_moe_forward.  No counterpart in the reference:
 * it exists for callers that cannot supply device memory -- a host reaching this
 * library over an FFI (cgo, JNI, N-API) with no CUDA allocator of its own, or a
 * serving loop whose memory budget is fixed at start-up.  The layer's
 * intermediate data lives in a static device array of
 * FLYAI_MOE_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * the process exits; nothing is allocated.  Descriptors whose workspace
 * (flyai_moe_workspace_bytes) exceeds that size are refused with
 * FLYAI_ERR_WORKSPACE.  All calls on a device share the one array: calls that
 * overlap on the GPU race, so order them on one stream.  The array's address
 * belongs to a CUDA context: every call outside stream capture looks it up
 * (cudaGetSymbolAddress) for the calling thread's current context and records
 * it; a call made while its stream is being captured uses the recorded address,
 * so make one uncaptured call on that context first (a context destroyed and
 * recreated, e.g. by cudaDeviceReset, needs its own).  Device error bits (a
 * bounded wait that gave up) land in the array and cannot be read on this path:
 * use flyai_moe_forward with a workspace and flyai_moe_read_error to observe
 * them.  Same outputs as flyai_moe_forward. */
#define FLYAI_MOE_NOALLOC_SCRATCH_BYTES (8u << 20)
FLYAI_API int flyai_moe_forward_noalloc(const flyai_moe_desc* desc, int32_t num_tokens,
                                        const void* x, const flyai_moe_weights* w, void* y,
                                        int32_t* topk_ids, void* topk_weights, void* stream);

/* Read back how many kernels the library launched since load (for launch accounting). */
FLYAI_API int64_t flyai_moe_launch_count(void);

/* Measurement hook (no reference counterpart): when both are non-null, every
 * later expert-kernel launch of this process records `start` (a cudaEvent_t)
 * just before it and `stop` just after it, on the launch stream, so a caller
 * can time the dominant kernel alone.  Pass nulls to switch it off. */
FLYAI_API int flyai_moe_set_profile_events(void* start, void* stop);

/* ---- Dense FP8 linear ----------------------------------------------------------
 * y = linear(x, W) for an e4m3 weight W [N, K] with one scale per 128x128 block
 * (vendor/deepseek_v4_ref/inference/model.py:114-124 `linear` on a float8_e4m3fn
 * weight: act_quant of x per 1x128, then fp8_gemm, kernel.py:203-274), at the
 * decode / verify sizes the reference's GEMV lever serves
 * (engines/deepseek_v4/v4_fp8_gemv.py:178-262 fp8_gemm_tiled_kernel and its
 * dispatch).  x bf16 [M, K], y bf16 [M, N]; N and K multiples of 128.
 * Per element: acc = D_kb * (s_x * s_w) + acc in fp32 over ascending 128-wide K
 * blocks (D_kb the block's e4m3 dot product), rounded once to bf16. */
#define FLYAI_LIN_SCALE_F32   0  /* weight scales fp32 [N/128, K/128]                          */
#define FLYAI_LIN_SCALE_E8M0  1  /* weight scales e8m0 bytes [N/128, K/128] (float8_e8m0fnu)   */
#define FLYAI_LIN_FMT_AMAX    0  /* activation scale amax/448 (scale_fmt None)                 */
#define FLYAI_LIN_FMT_UE8M0   1  /* activation scale 2^ceil(log2(amax/448)) (scale_fmt "ue8m0") */

/* Bytes of the packed weight bank of an [N, K] weight. */
FLYAI_API int flyai_fp8_linear_bank_bytes(int32_t N, int32_t K, size_t* bytes);
/* Pack weight (e4m3 [N, K], 16-byte aligned) and its scales (scale_dtype
 * FLYAI_LIN_SCALE_*) into bank, at load time (the reference's Linear holds
 * weight + weight.scale, model.py:127-158).  Banks of weights that read the same
 * x concatenate: the bank of [w1; w3] is the bank of w1 followed by that of w3. */
FLYAI_API int flyai_fp8_linear_pack(int32_t N, int32_t K, const void* weight, const void* scale,
                                    int32_t scale_dtype, void* bank, void* stream);
/* Workspace bytes for calls of up to max_tokens rows.  Zero-fill it once before
 * its first use; int32 word 0 is the error word (bit 1: a bounded wait gave up),
 * which calls set and never clear. */
FLYAI_API int flyai_fp8_linear_workspace_bytes(int32_t max_tokens, int32_t N, int32_t K,
                                               size_t* bytes);
/* y = linear(x, W) for num_tokens rows (two kernel launches per 64 rows),
 * scale_fmt FLYAI_LIN_FMT_*; x 16-byte and workspace 256-byte aligned. */
FLYAI_API int flyai_fp8_linear(int32_t num_tokens, int32_t N, int32_t K, const void* x,
                               const void* bank, int32_t scale_fmt, void* y, void* workspace,
                               size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLYAI_MOE_H */
