// flyai_moe_forward_noalloc: the whole MoE layer without any caller-supplied
// or library-allocated device memory beyond the inputs and outputs.
//
// Who needs this: hosts that cannot give the library device memory -- e.g. a
// Go/Java/Node program that reaches this library over cgo/JNI/N-API and has no
// CUDA allocator of its own to size and pass a workspace, or a serving loop whose
// device-memory budget is fixed at start-up and may not allocate per request.
// For them the intermediate data of a layer call (router logits, routing plan,
// SwiGLU activations, per-(token, slot) expert rows) lives in one file-scope
// __device__ array that is part of this library's module image: every GPU that
// loads the library holds it for the life of the process, and nothing here ever
// calls cudaMalloc, cudaFree or an allocating library routine.
//
// Rules of use:
//   * Limit: the descriptor's workspace (the same bytes flyai_moe_workspace_bytes
//     reports, which grow with max_tokens, num_experts, top_k, hidden and inter)
//     must fit in FLYAI_MOE_NOALLOC_SCRATCH_BYTES; larger descriptors are refused
//     with FLYAI_ERR_WORKSPACE before any device work.
//   * One array per device, shared by every call: calls that overlap on the GPU
//     (different streams, or threads issuing concurrently without ordering) race
//     on it and corrupt each other's results.  Order them on one stream.
//   * The array keeps the previous call's contents.  Each call writes every
//     region before reading it, and the one region that must start at zero (the
//     pair rows of other shards' experts under a partial expert range) is
//     cleared by the call itself.
//   * The array's device address belongs to a CUDA context.  Every call made
//     outside stream capture looks it up again (cudaGetSymbolAddress) for the
//     context current on the calling thread and records it per context; a call
//     issued while its stream is being captured into a CUDA graph uses the
//     recorded address, so make one call on that context before capturing.  A
//     context that was destroyed and recreated (cudaDeviceReset, or a host that
//     manages its own contexts) gets its own lookup on its first uncaptured call.
//   * Error bits that kernels record (a bounded wait that gave up) land in the
//     array, where no caller can read them: flyai_moe_read_error needs a
//     workspace pointer.  On this path a call that hit such a wait returns
//     FLYAI_OK with a zero output; callers that must observe it use
//     flyai_moe_forward with their own workspace.
#include <mutex>

#include "common.cuh"
#include "route.cuh"

namespace flyai {

// 8 MiB: enough for a verify-size layer (max_tokens 64, 128 experts, top-4,
// hidden = inter = 2880 needs about 5.6 MiB with the e2m1 activation terms of
// the tensor-core path).
static __device__ __align__(256) unsigned char g_noalloc_scratch[FLYAI_MOE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxContexts = 64;
struct CtxAddr {
  void* ctx;
  void* addr;
};
std::mutex g_noalloc_mu;
CtxAddr g_noalloc_cache[kMaxContexts] = {};
int g_noalloc_next = 0;

// cuCtxGetCurrent through the runtime's driver entry point table (the library
// links the static runtime, not libcuda, directly).
using CtxGetCurrentFn = int (*)(void**);
CtxGetCurrentFn ctx_get_current() {
  static const CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  return fn;
}
}  // namespace

// Device address of the scratch array in the calling thread's current context
// (the symbol itself is only a host stand-in, not a device address).
static int noalloc_scratch(cudaStream_t stream, void** out) {
  const CtxGetCurrentFn get_ctx = ctx_get_current();
  void* ctx = nullptr;
  if (!get_ctx || get_ctx(&ctx) != 0) return FLYAI_ERR_CUDA;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  const bool capturing = cudaStreamIsCapturing(stream, &cs) != cudaSuccess ||
                         cs != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  int slot = -1;
  if (ctx)
    for (int i = 0; i < kMaxContexts; ++i)
      if (g_noalloc_cache[i].ctx == ctx) slot = i;
  if (capturing) {
    if (slot < 0) return FLYAI_ERR_CUDA;   // no uncaptured call on this context yet
    *out = g_noalloc_cache[slot].addr;
    return FLYAI_OK;
  }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
    return FLYAI_ERR_CUDA;
  if (!ctx) {   // the lookup made the runtime's primary context current
    if (get_ctx(&ctx) != 0 || !ctx) return FLYAI_ERR_CUDA;
    for (int i = 0; i < kMaxContexts; ++i)
      if (g_noalloc_cache[i].ctx == ctx) slot = i;
  }
  if (slot < 0) {
    slot = g_noalloc_next;
    g_noalloc_next = (g_noalloc_next + 1) % kMaxContexts;
  }
  g_noalloc_cache[slot] = CtxAddr{ctx, p};
  *out = p;
  return FLYAI_OK;
}

}  // namespace flyai

using namespace flyai;

extern "C" int flyai_moe_forward_noalloc(const flyai_moe_desc* desc, int32_t M, const void* x,
                                         const flyai_moe_weights* w, void* y, int32_t* topk_ids,
                                         void* topk_weights, void* stream) {
  const int st = flyai_moe_check_desc(desc);
  if (st != FLYAI_OK) return st;
  if (M < 0 || M > desc->max_tokens) return FLYAI_ERR_INVALID_ARG;
  size_t need = 0;
  if (flyai_moe_workspace_bytes(desc, &need) != FLYAI_OK) return FLYAI_ERR_INVALID_ARG;
  if (need > FLYAI_MOE_NOALLOC_SCRATCH_BYTES) return FLYAI_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int sst = noalloc_scratch(static_cast<cudaStream_t>(stream), &scratch);
  if (sst != FLYAI_OK) return sst;
  // Same validation and launch sequence as flyai_moe_forward, on the static array.
  return flyai_moe_forward(desc, M, x, w, y, topk_ids, topk_weights, scratch,
                           FLYAI_MOE_NOALLOC_SCRATCH_BYTES, stream);
}
