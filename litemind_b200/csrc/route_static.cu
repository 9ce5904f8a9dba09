// route_static.cu -- routing for callers that cannot allocate device memory.
//
// lm_moe_route_static runs the same two kernels as lm_moe_route (router logits,
// then softmax / top-k per token) but needs no context and allocates nothing.
// Its only scratch, the f32 logits of one call, lives in the file-scope device
// array below, which every GPU that loads this library holds until the process
// exits.  Callers that cannot allocate include code running inside a CUDA graph
// capture (cudaMalloc is not a capturable operation), plugins whose host owns all
// device memory through its own pool and forbids the plugin from calling the
// CUDA allocator, and latency-critical paths that must not risk an allocation
// that synchronises the device.
#include <cudaTypedefs.h>

#include <mutex>

#include "moe_internal.h"

namespace lm {
namespace {

constexpr int kStaticLogitsFloats = 262144;  // 1 MiB of f32 logits: tokens * experts
constexpr int kStaticMaxTokens = 2047;       // the warp-per-token logits kernel's range
constexpr int kMaxDevices = 64;

// The scratch.  In host code this name is only a stand-in for the symbol, not a
// device address: it must go through cudaGetSymbolAddress before any kernel sees it.
static __device__ __align__(256) float g_route_scratch[kStaticLogitsFloats];

// The resolved address of the scratch on each device, with the unique id of the
// context it belongs to: after a device reset the module is loaded again into a new
// context (with a new id), and the address is looked up again.
struct ScratchSlot {
    unsigned long long ctx_id = 0;
    float* ptr = nullptr;
};
std::mutex g_setup_mutex;
ScratchSlot g_scratch[kMaxDevices];

// Failures are reported by status code only (see include/litemind_moe.h): the
// entry point keeps no message state of its own.
lm_status static_fail(lm_status code, const char* /*why*/) { return code; }

// cuCtxGetCurrent and cuCtxGetId, fetched through the runtime (the library does not
// link the driver API directly).
struct CtxApi {
    PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    PFN_cuCtxGetId_v12000 get_id = nullptr;
};
const CtxApi& ctx_api() {
    static CtxApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            api.get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            api.get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    });
    return api;
}

// Unique id of this thread's current context, 0 when none is current yet.
unsigned long long current_ctx_id() {
    const CtxApi& api = ctx_api();
    CUcontext cur = nullptr;
    unsigned long long id = 0;
    if (api.get_current == nullptr || api.get_id == nullptr || api.get_current(&cur) != CUDA_SUCCESS ||
        cur == nullptr || api.get_id(cur, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Set-up, once per device (and again after a reset of that device), with the device
// current: resolve the device address of the scratch array.  The first call on a
// device does this; it should come before any stream capture on that device.
lm_status scratch_for_current_device(float** out) {
    int device = -1;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return static_fail(LM_ERR_CUDA, "cudaGetDevice failed");
    if (device < 0 || device >= kMaxDevices) return static_fail(LM_ERR_UNSUPPORTED, "device ordinal out of range");
    const unsigned long long id = current_ctx_id();
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    ScratchSlot& slot = g_scratch[device];
    if (slot.ptr == nullptr || id == 0 || slot.ctx_id != id) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_route_scratch);  // makes the device's context current if needed
        if (e != cudaSuccess || ptr == nullptr) return static_fail(LM_ERR_CUDA, "cudaGetSymbolAddress failed");
        slot.ptr = static_cast<float*>(ptr);
        slot.ctx_id = current_ctx_id();
    }
    *out = slot.ptr;
    return LM_OK;
}

}  // namespace
}  // namespace lm

extern "C" {

lm_status lm_moe_route_static(const float* router, const uint16_t* x, int32_t tokens, int32_t hidden,
                              int32_t experts, int32_t top_k, int32_t norm_topk_prob, float routed_scaling_factor,
                              const float* logit_bias, int32_t* topk_idx, float* topk_w, void* stream) {
    using namespace lm;
    if (tokens < 0 || hidden <= 0 || experts <= 0 || top_k <= 0 || top_k > experts)
        return static_fail(LM_ERR_INVALID_ARGUMENT, "need tokens >= 0, hidden > 0 and 0 < top_k <= experts");
    if (hidden % 8 != 0 || experts > kMaxExperts || top_k > kMaxTopK)
        return static_fail(LM_ERR_UNSUPPORTED, "hidden must be a multiple of 8, experts <= 256, top_k <= 16");
    if (tokens > kStaticMaxTokens || static_cast<int64_t>(tokens) * experts > kStaticLogitsFloats)
        return static_fail(LM_ERR_TOO_MANY_TOKENS,
                           "lm_moe_route_static handles at most 2047 tokens and tokens * experts <= 262144 "
                           "(its fixed 1 MiB scratch); use lm_moe_route for larger batches");
    if (tokens == 0) return LM_OK;
    if (router == nullptr || x == nullptr || topk_idx == nullptr || topk_w == nullptr ||
        (reinterpret_cast<uintptr_t>(x) & 15u) != 0 || (reinterpret_cast<uintptr_t>(router) & 15u) != 0)
        return static_fail(LM_ERR_INVALID_ARGUMENT, "router and x must be 16-byte aligned device pointers");
    float* scratch = nullptr;
    lm_status st = scratch_for_current_device(&scratch);
    if (st != LM_OK) return st;
    RouterParams rp{};
    rp.experts = experts;
    rp.top_k = top_k;
    rp.n_group = 1;
    rp.topk_group = 1;
    rp.group_limited = 0;
    rp.normalize = norm_topk_prob != 0;
    rp.scale = routed_scaling_factor;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Every logit of this call is written before it is read, so nothing in the
    // scratch needs clearing between calls.
    cudaError_t e = launch_router_logits(x, nullptr, router, nullptr, logit_bias, scratch, tokens, hidden, experts, nullptr,
                                         0, s, false);
    if (e == cudaSuccess) e = launch_router_topk(scratch, tokens, rp, topk_idx, topk_w, nullptr, s, false);
    if (e != cudaSuccess) return static_fail(LM_ERR_CUDA, "kernel launch failed");
    return LM_OK;
}

}  // extern "C"
