#pragma once
#include "common.cuh"

namespace flyai {

int launch_route(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                 void* logits_out, int32_t* ids_out, void* wts_out, const Workspace& ws,
                 cudaStream_t stream);
// Routing the caller chose (FLYAI_GATE_EXTERNAL): ids and weights into the
// workspace, an id outside [0, E) read as 0 with kErrBadIndex, then the plan.
int launch_route_ids(const flyai_moe_desc& d, int M, const int32_t* ids, const float* wts,
                     const Workspace& ws, cudaStream_t stream);

// Tensor-core (tcgen05 kind::mxf4) expert path: every MXFP4 descriptor the ABI
// accepts (hidden and inter multiples of 64, at most kTcMaxK); the bank layout is
// the tile layout of tc_experts.cu.
bool tc_supported(const flyai_moe_desc& d);
size_t tc_packed_bytes(const flyai_moe_desc& d, int proj);
int launch_tc_pack(const flyai_moe_desc& d, int proj, const void* blocks, const void* scales,
                   void* packed, cudaStream_t stream);
// x_split: the route step of this call already wrote ws.x_terms / ws.x_sf from x.
// ep != null: expert parallel over peer memory (verify sizes only; the caller checks).
int launch_tc_experts(const flyai_moe_desc& d, int M, const void* x, bool x_split,
                      const flyai_moe_weights& w, uint16_t* pair_out, bool zero_pairs,
                      const Workspace& ws, cudaStream_t stream, void* y_fold = nullptr,
                      bool* folded = nullptr, const flyai_moe_ep_peers* ep = nullptr);
// The whole verify-size layer in one launch (routing in the expert kernel's
// prologue, the fold into y in its down epilogue): batches of 1..64 tokens with
// at most 256 (token, slot) pairs on a GPU holding every expert.  With ep, the
// same launch for an expert shard: routing of every token over all experts,
// this shard's experts, pair rows stored into every rank's mailbox and this
// rank's flag raised (the fold is launch_combine_ep's).
bool tc_fused_supported(const flyai_moe_desc& d, int M, bool ep = false);
int launch_tc_forward(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                      void* y, int32_t* ids_out, void* wts_out, const Workspace& ws,
                      cudaStream_t stream, const flyai_moe_ep_peers* ep = nullptr);
// Fold rows from this rank's mailbox once every rank's flag reached the epoch.
int launch_combine_ep(const flyai_moe_desc& d, int M, const flyai_moe_ep_peers& ep, void* y,
                      const Workspace& ws, cudaStream_t stream);

// Prefill-size batches (M >= kTcPrefillMinTokens): 16-token chunks, activation
// terms streamed with the weights (tc_prefill.cu).  Routing already done.
int launch_tc_prefill(const flyai_moe_desc& d, int M, const void* x, const flyai_moe_weights& w,
                      uint16_t* pair_out, const Workspace& ws, cudaStream_t stream);

int launch_combine(const flyai_moe_desc& d, int M, const uint16_t* pair_out, void* y,
                   const Workspace& ws, cudaStream_t stream);

}  // namespace flyai
