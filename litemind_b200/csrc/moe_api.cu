// moe_api.cu -- the C ABI of include/litemind_moe.h: context, weight residency,
// and the per-call launch sequence of the MoE path.
//
// Residency replaces the reference's ExpertCache paging (src/ExpertCache.cpp:9-47):
// every expert of every resident layer lives in HBM in the layout the grouped GEMMs
// read, so a forward call never moves weights.  Per layer:
//   w13   gate and up rows interleaved in pairs: logically [segments, 2*inter, hidden]
//   w2    down (the shared FFN split by columns): logically [segments, hidden, inter]
//   router [E, hidden] f32 and its transpose [hidden, E]
// Both weight matrices are stored tile-major: every 128-row x 64-column tile the
// GEMM loads is one contiguous 16 KiB block, tiles ordered (segment, row block,
// column block), so each TMA load reads whole DRAM pages instead of 128-byte pieces
// of 128 rows.
// where segments = the routed experts held on this device + n_shared_experts
// shared splits of width inter (sum over the splits == the reference's one
// shared FFN of width inter * n_shared, src/DeepSeekRunner.cpp:217-222).
// Uploads copy each segment's row-major rows into pinned staging on host threads,
// move them with one DMA and reorder them into tiles on the device (pack_upload).
#include "moe_internal.h"
#include "nccl_dl.h"
#include "ptx.cuh"
#include "host/CopyPool.hpp"
#include "host/SafeTensors.hpp"

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

namespace lm {

struct LayerWeights {
    uint16_t* w13 = nullptr;
    uint16_t* w2 = nullptr;
    float* router = nullptr;
    float* router_t = nullptr;
    float* norm = nullptr;
    uint16_t* router_cat = nullptr;  // [128, 3*hidden] bf16: router = hi + mid + lo, for the tensor-core router
    CUtensorMap map_w13{};
    CUtensorMap map_w2{};
    CUtensorMap map_router{};
    std::vector<uint8_t> expert_loaded;  // per local routed expert
    bool shared_loaded = false;
    bool router_loaded = false;
    bool complete() const {
        return router_loaded && shared_loaded &&
               std::all_of(expert_loaded.begin(), expert_loaded.end(), [](uint8_t v) { return v != 0; });
    }
};

// A dense feed-forward layer (DeepSeek's first layers, src/DeepSeekRunner.cpp:270-271):
// gate/up [inter, hidden] interleaved tile-major like an expert, down [hidden, inter].
struct DenseWeights {
    uint16_t* w13 = nullptr;
    uint16_t* w2 = nullptr;
    float* norm = nullptr;
    int inter = 0;
    CUtensorMap map_w13{};
    CUtensorMap map_w2{};
};

constexpr int kBnChoices[5] = {16, 32, 64, 128, 256};

}  // namespace lm

struct lm_moe_ctx {
    lm_moe_config cfg{};
    int device = 0;
    int sms = 148;
    int rank = 0;
    int nranks = 1;
    // Testing and profiling only (LITEMIND_B200_EP_SINGLE=1 at lm_moe_ep_init): a one-rank
    // expert-parallel context runs the exchange path, NCCL sending to itself, instead of
    // the local path, so that the exchange's kernels run on one GPU.
    bool ep_single = false;
    int first_expert = 0;
    int local_experts = 0;
    int n_seg = 0;
    int routed_cap = 0;  // rows reserved for routed tokens in h (expert-sorted order)
    std::vector<lm::LayerWeights> layers;

    float* logits = nullptr;
    int32_t* topk_idx = nullptr;
    float* topk_w = nullptr;
    int32_t* tile_counts = nullptr;
    int32_t* tile_base = nullptr;
    int32_t* expert_totals = nullptr;
    lm::Schedule* sched = nullptr;
    int32_t* row_token = nullptr;
    float* row_weight = nullptr;
    int32_t* slot_row = nullptr;
    uint16_t* x_perm = nullptr;      // routed token rows in expert-sorted order
    uint16_t* h = nullptr;
    int32_t* status = nullptr;
    int split_max_waves = 4;          // split-K below this many waves of tiles (LITEMIND_B200_SPLIT_WAVES)
    bool fused_decode = true;         // decode sizes on one GPU: one cooperative launch (LITEMIND_B200_FUSED_DECODE=0: off)
    int fused_max_tokens = lm::kDecodeMaxTokens;    // largest batch for it (LITEMIND_B200_FUSED_MAX_TOKENS)
    // Smallest batch the fused kernel gathers token rows for (LITEMIND_B200_FUSED_GATHER_FROM);
    // measured on B200: gather mode is faster from 16 tokens up (T=32: 187 vs 194 us).
    int fused_gather_from = 16;
    // Weight tiles read with an L2 evict-first hint (LITEMIND_B200_FUSED_EVICT_FIRST=0: off):
    // they are read once, and the hint keeps L2 for the rows the kernel re-reads.
    bool fused_evict_first = true;
    // In direct mode the fused kernel brings the shared experts' gate/up weights (known
    // before routing) into L2 while it routes (LITEMIND_B200_FUSED_PREFETCH=0: off).
    // Measured on B200: T=1 51.2 -> 47.0 us, T=8 123.9 -> 118.9 us.  In gather mode the
    // prefetch traffic slows the routing's L2 round trips by more than it saves (T=128:
    // +1 to +3 us), so it is off there; so is prefetching each CTA's share of the routed
    // experts' weights once the schedule exists (T=1: 50 -> 55 us).
    int fused_prefetch = 1;
    unsigned long long* grid_bar = nullptr;  // the fused decode kernel's arrival counters (self-resetting)
    // Testing only (lm_moe_debug_set): arrivals the fused kernel's grid waits expect
    // beyond the grid (so the waits run out), and the bound of those waits (0: 2 s).
    uint32_t debug_grid_extra = 0;
    uint64_t debug_wait_limit_ns = 0;
    unsigned long long* decode_trace = nullptr;  // per-CTA phase stamps of the last fused launch (profiling)
    std::vector<lm::DenseWeights> dense;  // dense feed-forward layers (lm_ffn_*)
    uint16_t* dense_h = nullptr;       // [max_tokens, widest dense inter] SwiGLU outputs
    int dense_h_inter = 0;
    CUtensorMap dense_map_h[5]{};
    lm::Schedule* dense_sched = nullptr;
    float* split_ws = nullptr;        // gate/up split-K partial tiles
    int32_t* split_ticket = nullptr;  // k-blocks done per split tile, zero between uses
    unsigned int* ticket = nullptr;  // [kRouteTickets] last-CTA tickets of the single-launch route kernels
    CUtensorMap map_xperm[5]{};
    CUtensorMap map_h[5]{};

    // Weight upload: rows staged in two pinned buffers, then on the device before
    // packing; the copy threads, the stream and each pinned buffer's DMA event.
    uint16_t* upload_raw = nullptr;
    size_t upload_raw_elems = 0;
    uint16_t* upload_pinned[2]{};
    cudaEvent_t upload_free[2]{};
    int upload_next = 0;
    cudaStream_t upload_stream = nullptr;
    std::unique_ptr<lm::CopyPool> copy_pool;

    // Host-API staging and the decoder sub-layer's normalised activations.
    uint16_t* x_stage = nullptr;
    float* y_stage = nullptr;
    float* bias_stage = nullptr;
    int32_t* status_host = nullptr;  // pinned: the status word read back with y, one sync per host call
    int32_t* status_host_dev = nullptr;  // its device address (the push kernel writes it)
    float* norm_f32 = nullptr;
    uint16_t* norm_bf16 = nullptr;
    cudaStream_t own_stream = nullptr;

    // Expert parallelism (lm_moe_ep_init).
    ncclComm_t comm = nullptr;
    bool ep_aborted = false;  // a peer missed an exchange: the communicator was aborted
    const lm::NcclApi* nccl = nullptr;
    uint16_t* x_recv = nullptr;    // received token rows, (source rank, local expert) segments
    uint16_t* x_sorted = nullptr;  // received rows, expert-major (each expert's rows contiguous)
    int ep_cap = 0;                // > 0: fixed-capacity exchange, rows per (source, destination) block
    uint16_t* x_send = nullptr;    // fixed-capacity send blocks [nranks][ep_cap][hidden]
    int32_t* ep_row_src = nullptr;  // expert-major row -> its source-major row (where its output goes back)
    uint16_t* y_ret = nullptr;     // expert outputs of the received rows (bf16), returned to their ranks
    uint16_t* y_back = nullptr;    // this rank's rows' expert outputs (bf16), in send order
    int32_t* recv_counts = nullptr;  // [nranks, local experts] rows received per source and expert
    lm::Schedule* sched_ep = nullptr;    // [kEpMaxChunks + 1]: one per chunk, then the shared experts'
    lm::Schedule* host_sched = nullptr;  // pinned, same shape
    int ep_chunks = 2;     // local-expert chunks of the host-planned exchange (LITEMIND_B200_EP_CHUNKS; 1: off)
    int ep_nccl_ctas = 32;  // NCCL's CTA cap, and the SMs the chunked GEMMs leave it (LITEMIND_B200_EP_NCCL_CTAS)
    cudaStream_t ep_stream = nullptr;  // the chunked exchange's NCCL stream
    cudaEvent_t ep_ev_ready = nullptr;
    cudaEvent_t ep_ev_back = nullptr;
    cudaEvent_t ep_ev_sent[lm::kEpMaxChunks]{};
    cudaEvent_t ep_ev_done[lm::kEpMaxChunks]{};
    // Profiling: timing events of the chunked exchange's last forward (see
    // lm_moe_profile_ep_timeline) and the times read from them.
    cudaEvent_t ep_tl_events[LM_EP_TIMELINE_MAX + 1]{};
    float ep_timeline[LM_EP_TIMELINE_MAX]{};
    int ep_timeline_chunks = 0;
    int32_t* host_totals = nullptr;      // pinned [E]
    int32_t* host_recv = nullptr;        // pinned [nranks * local experts]
    // Copy-engine exchange (LITEMIND_B200_EP_COPY, host-planned mode, nranks <= 8): every
    // rank's x_perm, y_ret and flag buffer mapped here by IPC; one copy stream per peer.
    bool ep_copy = false;
    uint32_t ep_epoch = 0;
    uint32_t* ep_flags = nullptr;        // this rank's flag slots: [N] rows ready, [kEpMaxChunks][N] outputs ready
    lm::EpPeerFlags ep_peer_flags{};
    uint16_t* ep_peer_xperm[lm::kEpCopyMaxRanks]{};
    uint16_t* ep_peer_yret[lm::kEpCopyMaxRanks]{};
    bool ep_peer_opened[lm::kEpCopyMaxRanks]{};  // IPC mappings to close at destroy
    cudaStream_t ep_copy_stream[lm::kEpCopyMaxRanks]{};
    cudaEvent_t ep_ev_pulled[lm::kEpMaxChunks][lm::kEpCopyMaxRanks]{};
    cudaEvent_t ep_ev_returned[lm::kEpCopyMaxRanks]{};
    int32_t* counts_all = nullptr;       // device [N, E]: every rank's rows per expert
    int32_t* host_counts_all = nullptr;  // pinned copy
    CUtensorMap map_xrecv[5]{};
    CUtensorMap map_xsorted[5]{};

    bool profiling = false;
    cudaEvent_t prof_events[LM_PROFILE_SLOTS + 1]{};
    double prof_ms[LM_PROFILE_SLOTS]{};
    int64_t prof_count[LM_PROFILE_SLOTS]{};
    int prof_last = -1;  // slot of the last recorded event in the current call

    uint64_t resident_bytes = 0;
    uint64_t uploaded_bytes = 0;
    std::string last_error;
    std::vector<void*> allocations;
};

namespace lm {
namespace {

lm_status fail(lm_moe_ctx* ctx, lm_status code, const std::string& message) {
    if (ctx != nullptr) ctx->last_error = message;
    return code;
}

lm_status cuda_fail(lm_moe_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, LM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define LM_CUDA(ctx, expr)                                         \
    do {                                                           \
        const cudaError_t lm_e_ = (expr);                          \
        if (lm_e_ != cudaSuccess) return cuda_fail(ctx, lm_e_, #expr); \
    } while (0)

template <typename T>
lm_status alloc(lm_moe_ctx* ctx, T** ptr, size_t count) {
    void* p = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 256);
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMalloc");
    ctx->allocations.push_back(p);
    *ptr = static_cast<T*>(p);
    return LM_OK;
}

int bn_index(int bn) {
    for (int i = 0; i < 5; ++i)
        if (kBnChoices[i] == bn) return i;
    return -1;
}

// Token-tile width of the grouped GEMMs from the average rows per expert segment.
int choose_bn(int tokens, int top_k, int experts) {
    const long avg = (static_cast<long>(tokens) * top_k + experts - 1) / experts;
    if (avg <= 16) return 16;
    if (avg <= 32) return 32;
    if (avg <= 64) return 64;
    if (avg <= 128) return 128;
    return 256;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The device address of a host buffer when it is page-locked (cudaHostAlloc,
// cudaMallocHost, cudaHostRegister: under unified addressing every page-locked range is
// mapped), else nullptr (pageable memory).
const void* mapped_device_address(const void* host) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, host) != cudaSuccess) {
        cudaGetLastError();  // not a CUDA-known pointer: clear the error, copy instead
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// Whether the placement kernel (one CTA per routing tile) also copies the token rows:
// only past the routed-small path and with at least one tile per two SMs.  Below that
// the separate gather (a CTA per row) copies faster than the placement's few CTAs.
bool place_gathers(const lm_moe_ctx* ctx, int T) { return T > kRouteTile && 2 * T >= kRouteTile * ctx->sms; }

lm_status check_layer(lm_moe_ctx* ctx, int32_t layer) {
    if (layer < 0 || layer >= static_cast<int32_t>(ctx->layers.size()))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "layer index out of range");
    if (!ctx->layers[layer].complete())
        return fail(ctx, LM_ERR_NOT_LOADED, "layer " + std::to_string(layer) + " is not fully uploaded");
    return LM_OK;
}

RouterParams router_params(const lm_moe_config& c) {
    RouterParams rp{};
    rp.experts = c.n_routed_experts;
    rp.top_k = c.num_experts_per_tok;
    int n_group = std::max(c.n_group, 1);
    rp.topk_group = std::max(c.topk_group, 1);
    rp.group_limited = c.topk_method == LM_TOPK_GROUP_LIMITED_GREEDY;
    if (c.n_routed_experts % n_group != 0) {  // src/MoeRouter.cpp:46-51
        rp.group_limited = 0;
        n_group = 1;
    }
    rp.n_group = n_group;
    rp.normalize = c.norm_topk_prob != 0;
    rp.scale = c.routed_scaling_factor;
    return rp;
}

lm_status ensure_layer_buffers(lm_moe_ctx* ctx, int32_t layer) {
    LayerWeights& L = ctx->layers[layer];
    if (L.w13 != nullptr) return LM_OK;
    const lm_moe_config& c = ctx->cfg;
    const size_t H = c.hidden_size, I = c.moe_intermediate_size, E = c.n_routed_experts;
    const size_t segs = ctx->n_seg;
    lm_status st;
    if ((st = alloc(ctx, &L.w13, segs * 2 * I * H)) != LM_OK) return st;
    if ((st = alloc(ctx, &L.w2, segs * H * I)) != LM_OK) return st;
    if ((st = alloc(ctx, &L.router, E * H)) != LM_OK) return st;
    if ((st = alloc(ctx, &L.router_t, E * H)) != LM_OK) return st;
    if ((st = alloc(ctx, &L.norm, H)) != LM_OK) return st;
    if ((st = alloc(ctx, &L.router_cat, 128 * 3 * H)) != LM_OK) return st;
    ctx->resident_bytes += segs * 3 * I * H * 2 + 2 * E * H * 4 + H * 4;
    std::string err;
    // Tile-major storage: a [rows, 64] matrix of 128-row tiles.
    if (!encode_tensor_map_bf16(&L.map_w13, L.w13, segs * 2 * I * H / 64, 64, 128, 64, err) ||
        !encode_tensor_map_bf16(&L.map_w2, L.w2, segs * H * I / 64, 64, 128, 64, err) ||
        !encode_tensor_map_bf16(&L.map_router, L.router_cat, 128, 3 * H, 128, 64, err))
        return fail(ctx, LM_ERR_CUDA, err);
    L.expert_loaded.assign(ctx->local_experts, 0);
    return LM_OK;
}

// One SwiGLU block from host memory into the tile-major w13 / w2.  The host threads
// of a CopyPool copy the three matrices' rows into one of two pinned buffers (down
// rows read with their pitch), one DMA moves the buffer to the device, and
// launch_pack_swiglu reorders the rows there -- the host does no per-element work,
// and the next block's host copy overlaps this one's DMA.  The source is fully read
// on return; the device work completes by finish_uploads.
lm_status pack_upload(lm_moe_ctx* ctx, uint16_t* w13, uint16_t* w2, const uint16_t* gate, const uint16_t* up,
                      const uint16_t* down, size_t I, size_t H, size_t down_pitch) {
    const size_t need = 3 * I * H;
    if (ctx->upload_stream == nullptr) {
        LM_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->upload_stream, cudaStreamNonBlocking));
        for (cudaEvent_t& e : ctx->upload_free) LM_CUDA(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        const unsigned hw = std::thread::hardware_concurrency();
        ctx->copy_pool = std::make_unique<CopyPool>(static_cast<int>(std::clamp(hw, 1u, 8u)));
    }
    cudaStream_t s = ctx->upload_stream;
    if (need > ctx->upload_raw_elems) {
        LM_CUDA(ctx, cudaStreamSynchronize(s));
        if (ctx->upload_raw != nullptr) cudaFree(ctx->upload_raw);
        for (uint16_t*& p : ctx->upload_pinned) {
            if (p != nullptr) cudaFreeHost(p);
            p = nullptr;
        }
        ctx->upload_raw = nullptr;
        ctx->upload_raw_elems = 0;
        LM_CUDA(ctx, cudaMalloc(&ctx->upload_raw, need * sizeof(uint16_t)));
        for (uint16_t*& p : ctx->upload_pinned) LM_CUDA(ctx, cudaMallocHost(&p, need * sizeof(uint16_t)));
        ctx->upload_raw_elems = need;
    }
    const int k = ctx->upload_next;
    ctx->upload_next ^= 1;
    // The buffer's previous DMA must be done before it is refilled.
    LM_CUDA(ctx, cudaEventSynchronize(ctx->upload_free[k]));
    uint16_t* pin = ctx->upload_pinned[k];
    struct Rows {
        uint16_t* dst;
        const uint16_t* src;
        size_t rows, width, pitch;
    };
    const Rows mats[3] = {{pin, gate, I, H, H}, {pin + I * H, up, I, H, H}, {pin + 2 * I * H, down, H, I, down_pitch}};
    // About 1 MiB per piece.
    size_t per[3], pieces[3], total = 0;
    for (int m = 0; m < 3; ++m) {
        per[m] = std::max<size_t>(1, (size_t(1) << 19) / mats[m].width);
        pieces[m] = (mats[m].rows + per[m] - 1) / per[m];
        total += pieces[m];
    }
    ctx->copy_pool->run(static_cast<int>(total), [&](int i) {
        int m = 0;
        size_t j = static_cast<size_t>(i);
        while (j >= pieces[m]) j -= pieces[m++];
        const Rows& R = mats[m];
        const size_t r0 = j * per[m], r1 = std::min(R.rows, r0 + per[m]);
        if (R.pitch == R.width) {
            std::memcpy(R.dst + r0 * R.width, R.src + r0 * R.pitch, (r1 - r0) * R.width * sizeof(uint16_t));
        } else {
            for (size_t r = r0; r < r1; ++r)
                std::memcpy(R.dst + r * R.width, R.src + r * R.pitch, R.width * sizeof(uint16_t));
        }
    });
    LM_CUDA(ctx, cudaMemcpyAsync(ctx->upload_raw, pin, need * sizeof(uint16_t), cudaMemcpyHostToDevice, s));
    LM_CUDA(ctx, cudaEventRecord(ctx->upload_free[k], s));
    uint16_t* rg = ctx->upload_raw;
    LM_CUDA(ctx, launch_pack_swiglu(rg, rg + I * H, rg + 2 * I * H, static_cast<int>(I), static_cast<int>(H), w13, w2,
                                    ctx->sms, s));
    return LM_OK;
}

// Waits for the uploads pack_upload queued (every public upload entry point ends
// here, so weights are in place when it returns); `st` passes through unless it is
// LM_OK and the device work failed.
lm_status finish_uploads(lm_moe_ctx* ctx, lm_status st) {
    if (ctx == nullptr || ctx->upload_stream == nullptr) return st;
    const cudaError_t e = cudaStreamSynchronize(ctx->upload_stream);
    if (st == LM_OK && e != cudaSuccess) return cuda_fail(ctx, e, "weight upload");
    return st;
}

// One SwiGLU block into segment `seg`: gate rows to the even rows of w13, up rows
// to the odd rows, down [hidden, inter] with source row pitch `down_pitch` elements;
// both stored tile-major.
lm_status upload_segment(lm_moe_ctx* ctx, LayerWeights& L, int seg, const uint16_t* gate, const uint16_t* up,
                         const uint16_t* down, size_t down_pitch) {
    const size_t H = ctx->cfg.hidden_size, I = ctx->cfg.moe_intermediate_size;
    lm_status st = pack_upload(ctx, L.w13 + static_cast<size_t>(seg) * 2 * I * H, L.w2 + static_cast<size_t>(seg) * H * I,
                               gate, up, down, I, H, down_pitch);
    if (st != LM_OK) return st;
    ctx->uploaded_bytes += 3 * I * H * 2;
    return LM_OK;
}

lm_status set_device(lm_moe_ctx* ctx) {
    LM_CUDA(ctx, cudaSetDevice(ctx->device));
    return LM_OK;
}

// Profiling: event 0 marks the start of a forward, event slot+1 the end of that
// slot's launch.  Times are attributed from the previous recorded event.
void prof_begin(lm_moe_ctx* ctx, cudaStream_t s) {
    if (!ctx->profiling) return;
    cudaEventRecord(ctx->prof_events[0], s);
    ctx->prof_last = -1;
}
void prof_mark(lm_moe_ctx* ctx, int slot, cudaStream_t s) {
    if (!ctx->profiling) return;
    cudaEventRecord(ctx->prof_events[slot + 1], s);
}
lm_status prof_end(lm_moe_ctx* ctx, const int* slots, int n) {
    if (!ctx->profiling) return LM_OK;
    LM_CUDA(ctx, cudaEventSynchronize(ctx->prof_events[slots[n - 1] + 1]));
    int prev = 0;
    for (int i = 0; i < n; ++i) {
        float ms = 0.0f;
        LM_CUDA(ctx, cudaEventElapsedTime(&ms, ctx->prof_events[prev], ctx->prof_events[slots[i] + 1]));
        ctx->prof_ms[slots[i]] += ms;
        ctx->prof_count[slots[i]] += 1;
        prev = slots[i] + 1;
    }
    return LM_OK;
}

// The shared experts (gate/up [n_shared * I, H], down [H, n_shared * I]), the f32
// router [E, H] in its three device forms, and the block's RMSNorm weight (ones
// when null).
lm_status upload_shared_and_router(lm_moe_ctx* ctx, LayerWeights& L, const float* router, const uint16_t* shared_gate,
                                   const uint16_t* shared_up, const uint16_t* shared_down, const float* norm_weight) {
    const lm_moe_config& c = ctx->cfg;
    const size_t H = c.hidden_size, I = c.moe_intermediate_size, E = c.n_routed_experts;
    lm_status st;
    const size_t S = I * c.n_shared_experts;
    for (int t = 0; t < c.n_shared_experts; ++t) {
        if ((st = upload_segment(ctx, L, ctx->local_experts + t, shared_gate + t * I * H, shared_up + t * I * H,
                                 shared_down + t * I, S)) != LM_OK)
            return st;
    }
    L.shared_loaded = true;
    std::vector<float> transposed(E * H);
    for (size_t e = 0; e < E; ++e)
        for (size_t k = 0; k < H; ++k) transposed[k * E + e] = router[e * H + k];
    LM_CUDA(ctx, cudaMemcpy(L.router, router, E * H * sizeof(float), cudaMemcpyHostToDevice));
    // The f32 router as three bf16 parts (each the rounding of what the previous
    // ones leave), so hi + mid + lo == router exactly and every product with a bf16
    // token is exact in f32 on the tensor cores.
    if (E <= 128) {
        std::vector<uint16_t> cat(128 * 3 * H, 0);
        auto rne = [](float v) -> uint16_t {
            uint32_t b;
            std::memcpy(&b, &v, 4);
            return static_cast<uint16_t>((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
        };
        auto widen = [](uint16_t h) -> float {
            const uint32_t b = static_cast<uint32_t>(h) << 16;
            float v;
            std::memcpy(&v, &b, 4);
            return v;
        };
        for (size_t e = 0; e < E; ++e)
            for (size_t k = 0; k < H; ++k) {
                const float w = router[e * H + k];
                const uint16_t hi = rne(w);
                const float r1 = w - widen(hi);
                const uint16_t mid = rne(r1);
                const float r2 = r1 - widen(mid);
                cat[e * 3 * H + k] = hi;
                cat[e * 3 * H + H + k] = mid;
                cat[e * 3 * H + 2 * H + k] = rne(r2);
            }
        LM_CUDA(ctx, cudaMemcpy(L.router_cat, cat.data(), cat.size() * sizeof(uint16_t), cudaMemcpyHostToDevice));
    }
    LM_CUDA(ctx, cudaMemcpy(L.router_t, transposed.data(), E * H * sizeof(float), cudaMemcpyHostToDevice));
    if (norm_weight != nullptr)
        LM_CUDA(ctx, cudaMemcpy(L.norm, norm_weight, H * sizeof(float), cudaMemcpyHostToDevice));
    else {
        std::vector<float> ones(H, 1.0f);
        LM_CUDA(ctx, cudaMemcpy(L.norm, ones.data(), H * sizeof(float), cudaMemcpyHostToDevice));
    }
    ctx->uploaded_bytes += 2 * E * H * 4;
    L.router_loaded = true;
    return LM_OK;
}

// The expired exchange wait's record in this rank's flag buffer (copy-engine exchange).
uint32_t* ep_diag(lm_moe_ctx* ctx) { return ctx->ep_flags + ep_flag_slots(ctx->nranks) - kEpDiagSlots; }

// A status word the device recorded (already read back): on an error, clear it and
// re-arm every counter an aborted launch may have left short, then report it.
lm_status settle_status(lm_moe_ctx* ctx, int32_t status) {
    if (status != 0) {
        std::string detail;
        if (status == kDevTimeoutExchange && ctx->ep_flags != nullptr) {
            uint32_t d[3] = {0, 0, 0};
            if (cudaMemcpy(d, ep_diag(ctx), sizeof(d), cudaMemcpyDeviceToHost) == cudaSuccess)
                detail = ": flag slot " + std::to_string(d[0]) + " held " + std::to_string(d[1]) + ", epoch " +
                         std::to_string(d[2]) + " was awaited";
        }
        LM_CUDA(ctx, cudaMemset(ctx->status, 0, sizeof(int32_t)));
        // An aborted fused decode launch leaves its grid counters short: restart them.
        LM_CUDA(ctx, cudaMemset(ctx->grid_bar, 0, kDecodeCounters * sizeof(unsigned long long)));
        LM_CUDA(ctx, cudaMemset(ctx->split_ticket, 0, kSplitTickets * sizeof(int32_t)));
        LM_CUDA(ctx, cudaMemset(ctx->ticket, 0, kRouteTickets * sizeof(unsigned int)));
        const char* what = status == kDevBadTile  ? "a tile outside the schedule"
                           : status == kDevBadRow ? "an output row outside its buffer"
                                                  : "a bounded wait expired";
        return fail(ctx, LM_ERR_DEVICE_TIMEOUT,
                    std::string("a kernel stopped on ") + what + " (code " + std::to_string(status) + detail +
                        "); results are invalid");
    }
    return LM_OK;
}

// How long a host wait on expert-parallel work may take before the peers are given up
// on (LM_DEBUG_WAIT_LIMIT_NS shortens it, with the device waits, for tests).
constexpr uint64_t kEpHostLimitNs = 30ull * 1000 * 1000 * 1000;

// Ends expert parallelism on this context: aborts the communicator (which ends any of
// its kernels still waiting for a peer, so `s` drains) and reports LM_ERR_COMM.
lm_status ep_give_up(lm_moe_ctx* ctx, cudaStream_t s, const std::string& why) {
    if (ctx->comm != nullptr) ctx->nccl->CommAbort(ctx->comm);
    ctx->comm = nullptr;
    ctx->ep_aborted = true;
    cudaStreamSynchronize(s);
    cudaGetLastError();
    return fail(ctx, LM_ERR_COMM, why + "; the communicator was aborted");
}

// Waits for stream `s`, which may hold this rank's side of NCCL exchanges.  A peer that
// never takes its side leaves NCCL's kernels waiting for it, and a plain stream
// synchronisation would wait with them for ever.  So the stream is polled against a
// deadline; on expiry the communicator is aborted (which ends its waiting kernels and
// lets the stream drain) and the call fails with LM_ERR_COMM.  Expert parallelism on
// this context is then unusable; the caller destroys it.
lm_status ep_wait_stream(lm_moe_ctx* ctx, cudaStream_t s, const char* what) {
    if (ctx->comm == nullptr) {
        LM_CUDA(ctx, cudaStreamSynchronize(s));
        return LM_OK;
    }
    const uint64_t limit = ctx->debug_wait_limit_ns != 0 ? ctx->debug_wait_limit_ns : kEpHostLimitNs;
    const auto t0 = std::chrono::steady_clock::now();
    std::string why;
    for (int polls = 0;; ++polls) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess) {
            // An exchange whose peer went away can also end early with an error (the data
            // it delivered is not to be used).
            ncclResult_t async = ncclSuccess;
            if (ctx->nccl->CommGetAsyncError(ctx->comm, &async) == ncclSuccess && async != ncclSuccess &&
                async != ncclInProgress) {
                why = std::string(what) + ": the exchange failed (" + ctx->nccl->GetErrorString(async) + ")";
                break;
            }
            return LM_OK;
        }
        if (q != cudaErrorNotReady) return cuda_fail(ctx, q, what);
        const auto waited = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0);
        if (static_cast<uint64_t>(waited.count()) > limit) {
            why = std::string(what) + ": a peer did not take its part in the exchange within " +
                  std::to_string(limit / 1000000) + " ms";
            break;
        }
        // Spin at first (an exchange normally completes within milliseconds), then back off.
        if (polls > 2000) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return ep_give_up(ctx, s, why);
}
}  // namespace
}  // namespace lm

using namespace lm;

extern "C" {

void lm_moe_config_default(lm_moe_config* c) {
    if (c == nullptr) return;
    std::memset(c, 0, sizeof(*c));
    c->hidden_size = 2048;
    c->moe_intermediate_size = 1408;
    c->n_routed_experts = 64;
    c->n_shared_experts = 2;
    c->num_experts_per_tok = 6;
    c->norm_topk_prob = 0;
    c->routed_scaling_factor = 1.0f;
    c->topk_method = LM_TOPK_GREEDY;
    c->n_group = 1;
    c->topk_group = 1;
    c->rms_norm_eps = 1e-6f;
    c->num_layers = 1;
    c->max_tokens = 16384;
}

const char* lm_status_string(lm_status s) {
    switch (s) {
        case LM_OK: return "ok";
        case LM_ERR_INVALID_ARGUMENT: return "invalid argument";
        case LM_ERR_CUDA: return "CUDA error";
        case LM_ERR_NOT_LOADED: return "weights not loaded";
        case LM_ERR_TOO_MANY_TOKENS: return "too many tokens";
        case LM_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case LM_ERR_COMM: return "communication error";
        case LM_ERR_UNSUPPORTED: return "unsupported";
        default: return "unknown status";
    }
}

const char* lm_moe_last_error(const lm_moe_ctx* ctx) {
    return ctx != nullptr ? ctx->last_error.c_str() : context_free_error().c_str();
}

lm_status lm_moe_create(const lm_moe_config* config, int device, lm_moe_ctx** out) {
    if (config == nullptr || out == nullptr) return LM_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    const lm_moe_config& c = *config;
    // Config::validate (src/Config.cpp:156-191) plus what the kernels need.
    if (c.hidden_size <= 0 || c.moe_intermediate_size <= 0 || c.n_routed_experts <= 0 ||
        c.num_experts_per_tok <= 0 || c.num_experts_per_tok > c.n_routed_experts || c.n_shared_experts < 0 ||
        c.num_layers <= 0 || c.max_tokens <= 0)
        return LM_ERR_INVALID_ARGUMENT;
    if (c.hidden_size % 128 != 0 || c.moe_intermediate_size % 64 != 0 || c.n_routed_experts > kMaxExperts ||
        c.num_experts_per_tok > kMaxTopK || c.n_shared_experts > kMaxShared ||
        (c.topk_method == LM_TOPK_GROUP_LIMITED_GREEDY && c.n_group > 32))
        return LM_ERR_UNSUPPORTED;
    if (c.topk_method != LM_TOPK_GREEDY && c.topk_method != LM_TOPK_GROUP_LIMITED_GREEDY)
        return LM_ERR_INVALID_ARGUMENT;

    auto ctx = std::make_unique<lm_moe_ctx>();
    ctx->cfg = c;
    ctx->device = device;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        context_free_error();
        return LM_ERR_CUDA;  // no GPU: there is no CPU fallback
    }
    if (device < 0 || device >= count) return LM_ERR_INVALID_ARGUMENT;
    if (cudaSetDevice(device) != cudaSuccess) return LM_ERR_CUDA;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return LM_ERR_CUDA;
    if (prop.major != 10) return LM_ERR_UNSUPPORTED;  // built for sm_100a only
    ctx->sms = prop.multiProcessorCount;
    if (const char* w = std::getenv("LITEMIND_B200_SPLIT_WAVES")) ctx->split_max_waves = std::max(0, std::atoi(w));
    if (const char* f = std::getenv("LITEMIND_B200_FUSED_DECODE")) ctx->fused_decode = std::atoi(f) != 0;
    if (const char* f = std::getenv("LITEMIND_B200_FUSED_MAX_TOKENS")) ctx->fused_max_tokens = std::atoi(f);
    if (const char* f = std::getenv("LITEMIND_B200_FUSED_GATHER_FROM"))
        ctx->fused_gather_from = std::max(1, std::atoi(f));
    if (const char* f = std::getenv("LITEMIND_B200_FUSED_EVICT_FIRST")) ctx->fused_evict_first = std::atoi(f) != 0;
    if (const char* f = std::getenv("LITEMIND_B200_FUSED_PREFETCH"))
        ctx->fused_prefetch = std::min(1, std::max(0, std::atoi(f)));
    ctx->local_experts = c.n_routed_experts;
    ctx->n_seg = ctx->local_experts + c.n_shared_experts;
    ctx->routed_cap = c.max_tokens * c.num_experts_per_tok;
    ctx->layers.resize(c.num_layers);

    lm_moe_ctx* p = ctx.get();
    const size_t T = c.max_tokens, K = c.num_experts_per_tok, E = c.n_routed_experts, H = c.hidden_size,
                 I = c.moe_intermediate_size;
    const size_t tiles = (T + kRouteTile - 1) / kRouteTile;
    const size_t h_rows = static_cast<size_t>(p->routed_cap) + c.n_shared_experts * T;
    lm_status st;
    if ((st = alloc(p, &p->logits, T * E)) || (st = alloc(p, &p->topk_idx, T * K)) ||
        (st = alloc(p, &p->topk_w, T * K)) || (st = alloc(p, &p->tile_counts, tiles * E)) ||
        (st = alloc(p, &p->tile_base, tiles * E)) || (st = alloc(p, &p->expert_totals, E)) ||
        (st = alloc(p, &p->sched, 1)) || (st = alloc(p, &p->row_token, static_cast<size_t>(p->routed_cap))) ||
        (st = alloc(p, &p->row_weight, static_cast<size_t>(p->routed_cap))) || (st = alloc(p, &p->slot_row, T * K)) ||
        (st = alloc(p, &p->x_perm, static_cast<size_t>(p->routed_cap) * H)) || (st = alloc(p, &p->h, h_rows * I)) ||
        (st = alloc(p, &p->status, 1)) || (st = alloc(p, &p->ticket, kRouteTickets)) ||
        (st = alloc(p, &p->split_ws, kSplitWsBytes / sizeof(float))) ||
        (st = alloc(p, &p->split_ticket, static_cast<size_t>(kSplitTickets))) ||
        (st = alloc(p, &p->grid_bar, kDecodeCounters))) {
        lm_moe_destroy(ctx.release());
        return st;
    }
    if (cudaMemset(p->status, 0, sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(p->ticket, 0, kRouteTickets * sizeof(unsigned int)) != cudaSuccess ||
        cudaMemset(p->expert_totals, 0, E * sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(p->sched, 0, sizeof(Schedule)) != cudaSuccess ||
        cudaMemset(p->split_ws, 0, kSplitWsBytes) != cudaSuccess ||
        cudaMemset(p->split_ticket, 0, kSplitTickets * sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(p->grid_bar, 0, kDecodeCounters * sizeof(unsigned long long)) != cudaSuccess) {
        lm_moe_destroy(ctx.release());
        return LM_ERR_CUDA;
    }
    std::string err;
    for (int i = 0; i < 5; ++i) {
        if (!encode_tensor_map_bf16(&p->map_xperm[i], p->x_perm, p->routed_cap, H, kBnChoices[i], 64, err) ||
            !encode_tensor_map_bf16(&p->map_h[i], p->h, h_rows, I, kBnChoices[i], 64, err)) {
            lm_moe_destroy(ctx.release());
            return LM_ERR_CUDA;
        }
    }
    *out = ctx.release();
    return LM_OK;
}

lm_status lm_moe_destroy(lm_moe_ctx* ctx) {
    if (ctx == nullptr) return LM_OK;
    cudaSetDevice(ctx->device);
    for (void* ptr : ctx->allocations) cudaFree(ptr);
    if (ctx->x_stage) cudaFree(ctx->x_stage);
    if (ctx->y_stage) cudaFree(ctx->y_stage);
    if (ctx->bias_stage) cudaFree(ctx->bias_stage);
    if (ctx->status_host) cudaFreeHost(ctx->status_host);
    if (ctx->norm_f32) cudaFree(ctx->norm_f32);
    if (ctx->norm_bf16) cudaFree(ctx->norm_bf16);
    if (ctx->decode_trace) cudaFree(ctx->decode_trace);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    if (ctx->upload_stream) cudaStreamSynchronize(ctx->upload_stream);
    if (ctx->upload_raw) cudaFree(ctx->upload_raw);
    for (uint16_t* p : ctx->upload_pinned)
        if (p) cudaFreeHost(p);
    for (cudaEvent_t e : ctx->upload_free)
        if (e) cudaEventDestroy(e);
    if (ctx->upload_stream) cudaStreamDestroy(ctx->upload_stream);
    if (ctx->comm != nullptr && ctx->nccl != nullptr) ctx->nccl->CommDestroy(ctx->comm);
    if (ctx->host_sched) cudaFreeHost(ctx->host_sched);
    if (ctx->ep_stream) cudaStreamDestroy(ctx->ep_stream);
    for (cudaEvent_t e : {ctx->ep_ev_ready, ctx->ep_ev_back})
        if (e) cudaEventDestroy(e);
    for (int i = 0; i < kEpMaxChunks; ++i) {
        if (ctx->ep_ev_sent[i]) cudaEventDestroy(ctx->ep_ev_sent[i]);
        if (ctx->ep_ev_done[i]) cudaEventDestroy(ctx->ep_ev_done[i]);
    }
    for (cudaEvent_t e : ctx->ep_tl_events)
        if (e) cudaEventDestroy(e);
    if (ctx->host_totals) cudaFreeHost(ctx->host_totals);
    if (ctx->host_recv) cudaFreeHost(ctx->host_recv);
    if (ctx->host_counts_all) cudaFreeHost(ctx->host_counts_all);
    for (int r = 0; r < kEpCopyMaxRanks; ++r) {
        if (ctx->ep_peer_opened[r]) {
            cudaIpcCloseMemHandle(ctx->ep_peer_xperm[r]);
            cudaIpcCloseMemHandle(ctx->ep_peer_yret[r]);
            cudaIpcCloseMemHandle(ctx->ep_peer_flags.flags[r]);
        }
        if (ctx->ep_copy_stream[r]) cudaStreamDestroy(ctx->ep_copy_stream[r]);
        if (ctx->ep_ev_returned[r]) cudaEventDestroy(ctx->ep_ev_returned[r]);
        for (int k = 0; k < kEpMaxChunks; ++k)
            if (ctx->ep_ev_pulled[k][r]) cudaEventDestroy(ctx->ep_ev_pulled[k][r]);
    }
    for (auto& e : ctx->prof_events)
        if (e) cudaEventDestroy(e);
    delete ctx;
    return LM_OK;
}

static lm_status upload_layer_body(lm_moe_ctx* ctx, int32_t layer, const float* router, const uint16_t* gate,
                              const uint16_t* up, const uint16_t* down, const uint16_t* shared_gate,
                              const uint16_t* shared_up, const uint16_t* shared_down, const float* norm_weight) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (layer < 0 || layer >= static_cast<int32_t>(ctx->layers.size()))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "layer index out of range");
    const lm_moe_config& c = ctx->cfg;
    if (router == nullptr || gate == nullptr || up == nullptr || down == nullptr ||
        (c.n_shared_experts > 0 && (shared_gate == nullptr || shared_up == nullptr || shared_down == nullptr)))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "null weight pointer");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    if ((st = ensure_layer_buffers(ctx, layer)) != LM_OK) return st;
    LayerWeights& L = ctx->layers[layer];
    const size_t H = c.hidden_size, I = c.moe_intermediate_size, E = c.n_routed_experts;
    for (int s = 0; s < ctx->local_experts; ++s) {
        const size_t e = static_cast<size_t>(ctx->first_expert + s);
        if ((st = upload_segment(ctx, L, s, gate + e * I * H, up + e * I * H, down + e * H * I, I)) != LM_OK)
            return st;
        L.expert_loaded[s] = 1;
    }
    return upload_shared_and_router(ctx, L, router, shared_gate, shared_up, shared_down, norm_weight);
}

lm_status lm_moe_upload_layer(lm_moe_ctx* ctx, int32_t layer, const float* router, const uint16_t* gate,
                              const uint16_t* up, const uint16_t* down, const uint16_t* shared_gate,
                              const uint16_t* shared_up, const uint16_t* shared_down, const float* norm_weight) {
    return finish_uploads(
        ctx, upload_layer_body(ctx, layer, router, gate, up, down, shared_gate, shared_up, shared_down, norm_weight));
}


lm_status lm_safetensors_info(const char* path, const char* name, int32_t* dtype, int32_t* ndim, int64_t* shape,
                              uint64_t* offset, uint64_t* nbytes, char* error, int32_t error_len) {
    auto set_error = [&](const std::string& e) {
        if (error != nullptr && error_len > 0) {
            const size_t n = std::min(e.size(), static_cast<size_t>(error_len - 1));
            std::memcpy(error, e.data(), n);
            error[n] = '\0';
        }
    };
    set_error("");
    if (path == nullptr || name == nullptr) {
        set_error("null path or name");
        return LM_ERR_INVALID_ARGUMENT;
    }
    host::StShard shard;
    std::string err;
    if (!shard.open(path, err)) {
        set_error(err);
        return LM_ERR_INVALID_ARGUMENT;
    }
    for (const host::StTensor& t : shard.tensors()) {
        if (t.name != name) continue;
        if (dtype != nullptr) *dtype = static_cast<int32_t>(t.dtype);
        if (ndim != nullptr) *ndim = static_cast<int32_t>(t.shape.size());
        if (shape != nullptr)
            for (size_t i = 0; i < t.shape.size() && i < LM_SAFETENSORS_MAX_DIMS; ++i) shape[i] = t.shape[i];
        if (offset != nullptr) *offset = t.offset;
        if (nbytes != nullptr) *nbytes = t.nbytes;
        if (t.shape.size() > LM_SAFETENSORS_MAX_DIMS) {
            set_error("tensor has more than LM_SAFETENSORS_MAX_DIMS dimensions");
            return LM_ERR_UNSUPPORTED;
        }
        return LM_OK;
    }
    set_error(std::string("no tensor named '") + name + "' in " + path);
    return LM_ERR_NOT_LOADED;
}

static lm_status load_safetensors_body(lm_moe_ctx* ctx, int32_t layer, int32_t checkpoint_layer,
                                  const char* const* shard_paths, int32_t n_shards) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (layer < 0 || layer >= static_cast<int32_t>(ctx->layers.size()))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "layer index out of range");
    if (shard_paths == nullptr || n_shards <= 0 || checkpoint_layer < 0)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "need at least one shard path and a checkpoint layer >= 0");
    std::vector<std::string> paths;
    for (int i = 0; i < n_shards; ++i) {
        if (shard_paths[i] == nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "null shard path");
        paths.emplace_back(shard_paths[i]);
    }
    host::StCheckpoint ck;
    std::string err;
    if (!ck.open(paths, err)) return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    const lm_moe_config& c = ctx->cfg;
    const int64_t H = c.hidden_size, I = c.moe_intermediate_size, E = c.n_routed_experts;
    const int64_t S = I * c.n_shared_experts;
    // Tensor names as DeepSeekRunner::Impl::resolve_layer reads them (src/DeepSeekRunner.cpp:157-224).
    const std::string prefix = "model.layers." + std::to_string(checkpoint_layer) + ".";
    std::vector<float> router, norm;
    if (ck.find(prefix + "mlp.gate.weight") == nullptr && ck.find(prefix + "mlp.gate_proj.weight") != nullptr)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "checkpoint layer " + std::to_string(checkpoint_layer) +
                                                      " is a dense feed-forward layer, not a mixture of experts");
    if (!ck.read_float32(prefix + "mlp.gate.weight", {E, H}, router, err) ||
        !ck.read_float32(prefix + "post_attention_layernorm.weight", {H}, norm, err))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    // Payload pointers of a shard whose header length is odd would be misaligned for
    // 16-bit reads: such tensors are copied out first.
    std::vector<std::vector<uint16_t>> copies;
    auto bf16 = [&](const host::StTensor* t) -> const uint16_t* {
        if ((reinterpret_cast<uintptr_t>(t->data) & 1u) == 0) return reinterpret_cast<const uint16_t*>(t->data);
        copies.emplace_back(t->nbytes / 2);
        std::memcpy(copies.back().data(), t->data, t->nbytes);
        return copies.back().data();
    };
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    if ((st = ensure_layer_buffers(ctx, layer)) != LM_OK) return st;
    LayerWeights& L = ctx->layers[layer];
    for (int s = 0; s < ctx->local_experts; ++s) {
        const std::string ep = prefix + "mlp.experts." + std::to_string(ctx->first_expert + s) + ".";
        const host::StTensor* g = ck.require(ep + "gate_proj.weight", {I, H}, host::StDtype::BF16, err);
        const host::StTensor* u = g ? ck.require(ep + "up_proj.weight", {I, H}, host::StDtype::BF16, err) : nullptr;
        const host::StTensor* d = u ? ck.require(ep + "down_proj.weight", {H, I}, host::StDtype::BF16, err) : nullptr;
        if (d == nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
        copies.clear();
        if ((st = upload_segment(ctx, L, s, bf16(g), bf16(u), bf16(d), static_cast<size_t>(I))) != LM_OK) return st;
        L.expert_loaded[s] = 1;
    }
    const uint16_t *sg = nullptr, *su = nullptr, *sd = nullptr;
    copies.clear();
    if (c.n_shared_experts > 0) {
        const std::string sp = prefix + "mlp.shared_experts.";
        const host::StTensor* g = ck.require(sp + "gate_proj.weight", {S, H}, host::StDtype::BF16, err);
        const host::StTensor* u = g ? ck.require(sp + "up_proj.weight", {S, H}, host::StDtype::BF16, err) : nullptr;
        const host::StTensor* d = u ? ck.require(sp + "down_proj.weight", {H, S}, host::StDtype::BF16, err) : nullptr;
        if (d == nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
        sg = bf16(g);
        su = bf16(u);
        sd = bf16(d);
    }
    return upload_shared_and_router(ctx, L, router.data(), sg, su, sd, norm.data());
}

lm_status lm_moe_load_safetensors(lm_moe_ctx* ctx, int32_t layer, int32_t checkpoint_layer,
                                  const char* const* shard_paths, int32_t n_shards) {
    return finish_uploads(ctx, load_safetensors_body(ctx, layer, checkpoint_layer, shard_paths, n_shards));
}

static lm_status ffn_upload_body(lm_moe_ctx* ctx, int32_t layer, int32_t intermediate, const uint16_t* gate, const uint16_t* up,
                        const uint16_t* down, const float* norm_weight) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    const lm_moe_config& c = ctx->cfg;
    if (layer < 0 || layer > 4096) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "dense layer index out of range");
    if (intermediate <= 0 || intermediate % 64 != 0)
        return fail(ctx, LM_ERR_UNSUPPORTED, "the dense intermediate size must be a positive multiple of 64");
    if (gate == nullptr || up == nullptr || down == nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "null weight");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    if (static_cast<int32_t>(ctx->dense.size()) <= layer) ctx->dense.resize(layer + 1);
    DenseWeights& D = ctx->dense[layer];
    const size_t H = c.hidden_size, I = intermediate;
    if (D.w13 != nullptr && D.inter != intermediate)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "dense layer was uploaded with another intermediate size");
    if (D.w13 == nullptr) {
        if ((st = alloc(ctx, &D.w13, 2 * I * H)) || (st = alloc(ctx, &D.w2, H * I)) || (st = alloc(ctx, &D.norm, H)))
            return st;
        D.inter = intermediate;
        ctx->resident_bytes += 3 * I * H * 2 + H * 4;
        std::string err;
        if (!encode_tensor_map_bf16(&D.map_w13, D.w13, 2 * I * H / 64, 64, 128, 64, err) ||
            !encode_tensor_map_bf16(&D.map_w2, D.w2, H * I / 64, 64, 128, 64, err))
            return fail(ctx, LM_ERR_CUDA, err);
    }
    if (intermediate > ctx->dense_h_inter) {
        // SwiGLU outputs of the widest dense layer for max_tokens rows.
        const size_t rows = c.max_tokens;
        for (auto it = ctx->allocations.begin(); it != ctx->allocations.end(); ++it)
            if (*it == ctx->dense_h) {
                cudaFree(*it);
                ctx->allocations.erase(it);
                break;
            }
        if ((st = alloc(ctx, &ctx->dense_h, rows * I)) != LM_OK) return st;
        if (ctx->dense_sched == nullptr && (st = alloc(ctx, &ctx->dense_sched, 1)) != LM_OK) return st;
        ctx->dense_h_inter = intermediate;
        std::string err;
        for (int i = 0; i < 5; ++i)
            if (!encode_tensor_map_bf16(&ctx->dense_map_h[i], ctx->dense_h, rows, I, kBnChoices[i], 64, err))
                return fail(ctx, LM_ERR_CUDA, err);
    }
    if ((st = pack_upload(ctx, D.w13, D.w2, gate, up, down, I, H, I)) != LM_OK) return st;
    std::vector<float> ones;
    if (norm_weight == nullptr) ones.assign(H, 1.0f);
    LM_CUDA(ctx, cudaMemcpy(D.norm, norm_weight != nullptr ? norm_weight : ones.data(), H * 4, cudaMemcpyHostToDevice));
    ctx->uploaded_bytes += 3 * I * H * 2;
    return LM_OK;
}

lm_status lm_ffn_upload(lm_moe_ctx* ctx, int32_t layer, int32_t intermediate, const uint16_t* gate, const uint16_t* up,
                        const uint16_t* down, const float* norm_weight) {
    return finish_uploads(ctx, ffn_upload_body(ctx, layer, intermediate, gate, up, down, norm_weight));
}

static lm_status ffn_load_safetensors_body(lm_moe_ctx* ctx, int32_t layer, int32_t checkpoint_layer, int32_t intermediate,
                                  const char* const* shard_paths, int32_t n_shards) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (shard_paths == nullptr || n_shards <= 0 || checkpoint_layer < 0)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "need at least one shard path and a checkpoint layer >= 0");
    std::vector<std::string> paths;
    for (int i = 0; i < n_shards; ++i) {
        if (shard_paths[i] == nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "null shard path");
        paths.emplace_back(shard_paths[i]);
    }
    host::StCheckpoint ck;
    std::string err;
    if (!ck.open(paths, err)) return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    const int64_t H = ctx->cfg.hidden_size, I = intermediate;
    // resolve_feed_forward(prefix + "mlp.", intermediate_size) (src/DeepSeekRunner.cpp:157-177, :193-195).
    const std::string prefix = "model.layers." + std::to_string(checkpoint_layer) + ".";
    std::vector<float> norm;
    const host::StTensor* g = ck.require(prefix + "mlp.gate_proj.weight", {I, H}, host::StDtype::BF16, err);
    const host::StTensor* u = g ? ck.require(prefix + "mlp.up_proj.weight", {I, H}, host::StDtype::BF16, err) : nullptr;
    const host::StTensor* d = u ? ck.require(prefix + "mlp.down_proj.weight", {H, I}, host::StDtype::BF16, err) : nullptr;
    if (d == nullptr || !ck.read_float32(prefix + "post_attention_layernorm.weight", {H}, norm, err))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    std::vector<std::vector<uint16_t>> copies;
    auto bf16 = [&](const host::StTensor* t) -> const uint16_t* {
        if ((reinterpret_cast<uintptr_t>(t->data) & 1u) == 0) return reinterpret_cast<const uint16_t*>(t->data);
        copies.emplace_back(t->nbytes / 2);
        std::memcpy(copies.back().data(), t->data, t->nbytes);
        return copies.back().data();
    };
    return lm_ffn_upload(ctx, layer, intermediate, bf16(g), bf16(u), bf16(d), norm.data());
}

lm_status lm_ffn_load_safetensors(lm_moe_ctx* ctx, int32_t layer, int32_t checkpoint_layer, int32_t intermediate,
                                  const char* const* shard_paths, int32_t n_shards) {
    return finish_uploads(ctx,
                          ffn_load_safetensors_body(ctx, layer, checkpoint_layer, intermediate, shard_paths, n_shards));
}

lm_status lm_ffn_forward(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, int32_t tokens, float* y,
                         int32_t accumulate, void* stream) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (layer < 0 || layer >= static_cast<int32_t>(ctx->dense.size()) || ctx->dense[layer].w13 == nullptr)
        return fail(ctx, LM_ERR_NOT_LOADED, "dense layer " + std::to_string(layer) + " is not uploaded");
    if (tokens < 0) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "negative token count");
    if (tokens > ctx->cfg.max_tokens) return fail(ctx, LM_ERR_TOO_MANY_TOKENS, "tokens exceed max_tokens");
    if (tokens == 0) return LM_OK;
    if (x == nullptr || y == nullptr || !aligned16(x) || !aligned16(y))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "x and y must be 16-byte aligned device pointers");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    const DenseWeights& D = ctx->dense[layer];
    const int H = ctx->cfg.hidden_size, I = D.inter, T = tokens;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // One segment of all tokens; 256-wide token tiles would need 256-row weight
    // blocks, which a dense intermediate size need not divide into.
    const int bn = std::min(choose_bn(T, 1, 1), 128);
    const int bi = bn_index(bn);
    prof_begin(ctx, s);
    LM_CUDA(ctx, launch_dense_schedule(ctx->dense_sched, T, bn, 2 * I / 128, H / 128, accumulate ? nullptr : y,
                                       static_cast<int64_t>(T) * H, ctx->sms, s));
    prof_mark(ctx, 3, s);
    CUtensorMap map_x{};
    std::string err;
    if (!encode_tensor_map_bf16(&map_x, x, T, H, bn, 64, err)) return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    GemmArgs args{};
    args.sched = ctx->dense_sched;
    args.x = x;
    args.h = ctx->dense_h;
    args.y = y;
    args.status = ctx->status;
    args.tokens = T;
    args.hidden = H;
    args.inter = I;
    args.n_routed_local = 0;  // the segment reads x, with weight 1, like a shared expert
    args.split_ws = ctx->split_ws;
    args.split_ticket = ctx->split_ticket;
    args.split_ws_floats = static_cast<int32_t>(kSplitWsBytes / sizeof(float));
    args.split_max_waves = ctx->split_max_waves;
    LM_CUDA(ctx, launch_gemm_gate_up(bn, D.map_w13, map_x, map_x, args, ctx->sms, s, true));
    prof_mark(ctx, 5, s);
    LM_CUDA(ctx, launch_gemm_down(bn, D.map_w2, ctx->dense_map_h[bi], args, ctx->sms, s, true));
    prof_mark(ctx, 6, s);
    const int slots[3] = {3, 5, 6};
    return prof_end(ctx, slots, 3);
}

lm_status lm_ffn_block_forward(lm_moe_ctx* ctx, int32_t layer, float* hidden, int32_t tokens, void* stream) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (layer < 0 || layer >= static_cast<int32_t>(ctx->dense.size()) || ctx->dense[layer].w13 == nullptr)
        return fail(ctx, LM_ERR_NOT_LOADED, "dense layer " + std::to_string(layer) + " is not uploaded");
    if (tokens < 0) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "negative token count");
    if (tokens > ctx->cfg.max_tokens) return fail(ctx, LM_ERR_TOO_MANY_TOKENS, "tokens exceed max_tokens");
    if (tokens == 0) return LM_OK;
    if (hidden == nullptr || !aligned16(hidden)) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "hidden must be aligned");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    const lm_moe_config& c = ctx->cfg;
    const size_t T = c.max_tokens, H = c.hidden_size;
    if (ctx->norm_f32 == nullptr) {
        LM_CUDA(ctx, cudaMalloc(&ctx->norm_f32, T * H * sizeof(float)));
        LM_CUDA(ctx, cudaMalloc(&ctx->norm_bf16, T * H * sizeof(uint16_t)));
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // rms_norm, the dense feed-forward, the residual add (src/DeepSeekRunner.cpp:265-271, :290),
    // the add folded into the down projection's accumulation into `hidden`.
    LM_CUDA(ctx, launch_rms_norm_rows(hidden, ctx->norm_f32, ctx->norm_bf16, ctx->dense[layer].norm, tokens,
                                      c.hidden_size, c.rms_norm_eps, s));
    return lm_ffn_forward(ctx, layer, ctx->norm_bf16, tokens, hidden, 1, stream);
}

static lm_status upload_expert_body(lm_moe_ctx* ctx, int32_t layer, int32_t expert, const uint16_t* gate,
                               const uint16_t* up, const uint16_t* down) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (layer < 0 || layer >= static_cast<int32_t>(ctx->layers.size()))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "layer index out of range");
    if (expert < ctx->first_expert || expert >= ctx->first_expert + ctx->local_experts)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "expert is not held by this device");
    if (gate == nullptr || up == nullptr || down == nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "null weight");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    if ((st = ensure_layer_buffers(ctx, layer)) != LM_OK) return st;
    LayerWeights& L = ctx->layers[layer];
    const int s = expert - ctx->first_expert;
    if ((st = upload_segment(ctx, L, s, gate, up, down, ctx->cfg.moe_intermediate_size)) != LM_OK) return st;
    L.expert_loaded[s] = 1;
    return LM_OK;
}

lm_status lm_moe_upload_expert(lm_moe_ctx* ctx, int32_t layer, int32_t expert, const uint16_t* gate,
                               const uint16_t* up, const uint16_t* down) {
    return finish_uploads(ctx, upload_expert_body(ctx, layer, expert, gate, up, down));
}

// Router logits: on the tensor cores for large batches of bf16 tokens, else the
// f32 CUDA-core kernels (which also serve the f32 activations of block_forward).
static lm_status router_logits(lm_moe_ctx* ctx, const LayerWeights& L, const uint16_t* x, const float* x_f32, int32_t T,
                               const float* bias, float* logits, cudaStream_t s, bool pdl, RouterFix* fix) {
    const lm_moe_config& c = ctx->cfg;
    *fix = RouterFix{};
    // Group-limited routing also ranks groups; it keeps the plain f32 logits.
    if (x_f32 == nullptr && T >= 512 && c.n_routed_experts <= 128 && !router_params(c).group_limited) {
        int bn = 16;
        while (bn < 128 && (T + bn - 1) / bn > ctx->sms) bn *= 2;
        CUtensorMap map_x{};
        std::string err;
        if (!encode_tensor_map_bf16(&map_x, x, T, c.hidden_size, bn, 64, err))
            return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
        GemmArgs args{};
        args.status = ctx->status;
        args.tokens = T;
        args.hidden = c.hidden_size;
        args.inter = c.moe_intermediate_size;
        args.logits = logits;
        args.bias = bias;
        args.experts = c.n_routed_experts;
        LM_CUDA(ctx, launch_gemm_router(bn, L.map_router, map_x, args, ctx->sms, s, pdl));
        fix->x = x;
        fix->w = L.router;
        fix->bias = bias;
        fix->hidden = c.hidden_size;
        fix->margin = 2e-5f;  // ten times the largest probability error seen from tensor-core logits
        return LM_OK;
    }
    LM_CUDA(ctx, launch_router_logits(x, x_f32, L.router, L.router_t, bias, logits, T, c.hidden_size,
                                      c.n_routed_experts, ctx->split_ws, kSplitWsBytes, s, pdl));
    return LM_OK;
}

static lm_status route_common(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, const float* x_f32, int32_t T,
                              const float* bias, float* logits, cudaStream_t stream) {
    const lm_moe_config& c = ctx->cfg;
    const LayerWeights& L = ctx->layers[layer];
    lm_status st;
    RouterFix fix;
    if ((st = router_logits(ctx, L, x, x_f32, T, bias, logits, stream, false, &fix)) != LM_OK) return st;
    LM_CUDA(ctx, launch_router_topk(logits, T, router_params(c), ctx->topk_idx, ctx->topk_w, ctx->tile_counts,
                                    stream, true, fix));
    return LM_OK;
}

lm_status lm_moe_route(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, int32_t tokens, const float* logit_bias,
                       int32_t* topk_idx, float* topk_w, float* logits, void* stream) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    lm_status st;
    if ((st = check_layer(ctx, layer)) != LM_OK) return st;
    if (tokens < 0) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "negative token count");
    if (tokens > ctx->cfg.max_tokens) return fail(ctx, LM_ERR_TOO_MANY_TOKENS, "tokens exceed max_tokens");
    if (tokens == 0) return LM_OK;
    if (x == nullptr || topk_idx == nullptr || topk_w == nullptr || !aligned16(x))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "x must be a 16-byte aligned device pointer; outputs non-null");
    if ((st = set_device(ctx)) != LM_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* lg = logits != nullptr ? logits : ctx->logits;
    if ((st = route_common(ctx, layer, x, nullptr, tokens, logit_bias, lg, s)) != LM_OK) return st;
    const lm_moe_config& c = ctx->cfg;
    LM_CUDA(ctx, launch_dispatch_scan(ctx->tile_counts, ctx->tile_base, ctx->expert_totals, ctx->sched, tokens,
                                      c.num_experts_per_tok, c.n_routed_experts, c.n_shared_experts, ctx->first_expert,
                                      ctx->local_experts, ctx->routed_cap, 16, 1, 1, s, true));
    const size_t n = static_cast<size_t>(tokens) * c.num_experts_per_tok;
    LM_CUDA(ctx, cudaMemcpyAsync(topk_idx, ctx->topk_idx, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    LM_CUDA(ctx, cudaMemcpyAsync(topk_w, ctx->topk_w, n * sizeof(float), cudaMemcpyDeviceToDevice, s));
    return LM_OK;
}

lm_status lm_moe_select(lm_moe_ctx* ctx, const float* logits, int32_t tokens, int32_t* topk_idx, float* topk_w,
                        void* stream) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (tokens < 0) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "negative token count");
    if (tokens == 0) return LM_OK;
    if (logits == nullptr || topk_idx == nullptr || topk_w == nullptr)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "null pointer");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    LM_CUDA(ctx, launch_router_topk(const_cast<float*>(logits), tokens, router_params(ctx->cfg), topk_idx, topk_w, nullptr,
                                    static_cast<cudaStream_t>(stream), false));
    return LM_OK;
}

static lm_status forward_impl(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, const float* x_f32, int32_t T,
                              const float* bias, float* y, int32_t accumulate, cudaStream_t s) {
    const lm_moe_config& c = ctx->cfg;
    const LayerWeights& L = ctx->layers[layer];
    const int K = c.num_experts_per_tok, E = c.n_routed_experts, H = c.hidden_size, I = c.moe_intermediate_size;
    const int bn = choose_bn(T, K, E);
    const int bi = bn_index(bn);
    prof_begin(ctx, s);
    int slots[8];
    int n_slots = 0;
    const RouterParams rp = router_params(c);
    float* y_zero = accumulate ? nullptr : y;  // the down GEMM adds into y
    // Decode sizes: the whole layer in one cooperative launch.  Below fused_gather_from
    // tokens every expert reads x itself (direct mode); from there on, routed token rows
    // are gathered in the kernel and tiled 32 at a time (gather mode).
    const bool gather = T >= ctx->fused_gather_from;
    const int fused_bn = gather ? kDecodeColTile : T <= 16 ? 16 : 32;
    const int max_active = std::min(E, T * K);
    const int fused_tiles =
        gather ? (c.n_shared_experts * ((T + kDecodeColTile - 1) / kDecodeColTile) + max_active +
                  (T * K + kDecodeColTile - 1) / kDecodeColTile) * (2 * I / 128)
               : (c.n_shared_experts + max_active) * (2 * I / 128);
    if (ctx->fused_decode && T <= ctx->fused_max_tokens && T <= kDecodeMaxTokens && T * K <= kDecodeMaxRows &&
        ctx->comm == nullptr && (gather || (T <= kDecodeDirectTokens && T * E <= kDecodeMaxLogits)) &&
        fused_tiles <= kSplitTickets &&
        static_cast<size_t>(2) * ctx->sms * 128 * fused_bn * sizeof(float) <= kSplitWsBytes) {
        CUtensorMap map_x{};
        std::string err;
        if (!encode_tensor_map_bf16(&map_x, x, T, H, fused_bn, 64, err)) return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
        DecodeArgs a{};
        a.x = x;
        a.x_f32 = x_f32;
        a.router = L.router;
        a.bias = bias;
        a.y = y;
        a.zero_y = accumulate ? 0 : 1;
        a.tokens = T;
        a.hidden = H;
        a.inter = I;
        a.n_shared = c.n_shared_experts;
        a.rp = rp;
        a.gather = gather ? 1 : 0;
        a.weight_evict_first = ctx->fused_evict_first ? 1 : 0;
        a.logits = ctx->logits;
        a.topk_idx = ctx->topk_idx;
        a.topk_w = ctx->topk_w;
        a.expert_totals = ctx->expert_totals;
        a.row_token = ctx->row_token;
        a.row_weight = ctx->row_weight;
        a.x_perm = ctx->x_perm;
        a.h = ctx->h;
        a.h_shared_base = ctx->routed_cap;
        a.split_ws = ctx->split_ws;
        a.split_ticket = ctx->split_ticket;
        a.grid_bar = ctx->grid_bar;
        a.grid_extra = ctx->debug_grid_extra;
        a.wait_limit_ns = ctx->debug_wait_limit_ns != 0 ? ctx->debug_wait_limit_ns : kWaitLimitNs;
        a.status = ctx->status;
        if (ctx->profiling && ctx->decode_trace == nullptr)
            LM_CUDA(ctx, cudaMalloc(&ctx->decode_trace, static_cast<size_t>(ctx->sms) * kDecodeTraceSlots * 8));
        if (ctx->profiling) LM_CUDA(ctx, cudaMemsetAsync(ctx->decode_trace, 0, static_cast<size_t>(ctx->sms) *
                                                                                   kDecodeTraceSlots * 8, s));
        a.trace = ctx->profiling ? ctx->decode_trace : nullptr;
        if (!gather && ctx->fused_prefetch > 0) {
            // w13 holds the routed experts' segments, then the shared experts' (2*I*H bf16
            // each): the shared ones are needed whatever the routing.
            const uint64_t seg13 = static_cast<uint64_t>(2) * I * H * sizeof(uint16_t);
            a.prefetch_base[0] = reinterpret_cast<const uint8_t*>(L.w13) + ctx->local_experts * seg13;
            a.prefetch_len[0] = (c.n_shared_experts * seg13) & ~uint64_t(4095);
        }
        const int fbi = bn_index(fused_bn);
        LM_CUDA(ctx, launch_moe_decode(fused_bn, L.map_w13, L.map_w2, map_x, ctx->map_xperm[bn_index(kDecodeColTile)],
                                       ctx->map_h[fbi], a, ctx->sms, s));
        prof_mark(ctx, 8, s);
        slots[n_slots++] = 8;
        return prof_end(ctx, slots, n_slots);
    }
    if (T <= kRouteTile) {
        // Decode: logits, top-k, counts, schedule and placement in one launch.
        LM_CUDA(ctx, launch_route_small(x, x_f32, L.router, bias, ctx->logits, T, H, rp, ctx->topk_idx, ctx->topk_w,
                                        ctx->expert_totals, ctx->sched, ctx->row_token, ctx->row_weight,
                                        ctx->slot_row, y_zero, ctx->ticket, c.n_shared_experts, ctx->first_expert,
                                        ctx->local_experts, ctx->routed_cap, bn, 2 * I / 128, H / 128, s, false));
        prof_mark(ctx, 1, s);
        slots[n_slots++] = 1;
    } else if (T <= kRouteMidTokens) {
        // Mid-size batches: the same single launch, over several token blocks.
        LM_CUDA(ctx, launch_route_mid(x, x_f32, L.router, bias, ctx->logits, T, H, rp, ctx->topk_idx, ctx->topk_w,
                                      ctx->expert_totals, ctx->sched, ctx->row_token, ctx->row_weight,
                                      ctx->slot_row, y_zero, ctx->ticket + 1,
                                      reinterpret_cast<uint32_t*>(ctx->tile_counts), c.n_shared_experts,
                                      ctx->first_expert, ctx->local_experts, ctx->routed_cap, bn, 2 * I / 128, H / 128,
                                      s, false));
        prof_mark(ctx, 1, s);
        slots[n_slots++] = 1;
    } else {
        lm_status rst;
        RouterFix fix;
        if ((rst = router_logits(ctx, L, x, x_f32, T, bias, ctx->logits, s, false, &fix)) != LM_OK) return rst;
        prof_mark(ctx, 1, s);
        slots[n_slots++] = 1;
        LM_CUDA(ctx, launch_router_topk(ctx->logits, T, rp, ctx->topk_idx, ctx->topk_w, ctx->tile_counts, s, true, fix));
        prof_mark(ctx, 2, s);
        slots[n_slots++] = 2;
        LM_CUDA(ctx, launch_dispatch_scan(ctx->tile_counts, ctx->tile_base, ctx->expert_totals, ctx->sched, T, K, E,
                                          c.n_shared_experts, ctx->first_expert, ctx->local_experts, ctx->routed_cap,
                                          bn, 2 * I / 128, H / 128, s, true));
        prof_mark(ctx, 3, s);
        slots[n_slots++] = 3;
        // With enough routing tiles the placement also copies the token rows into
        // expert order (each token read once); below that its grid is too small to
        // copy fast and the separate gather runs instead.
        LM_CUDA(ctx, launch_place(ctx->topk_idx, ctx->topk_w, ctx->tile_base, T, H, K, E, ctx->first_expert,
                                  ctx->local_experts, ctx->row_token, ctx->row_weight, ctx->slot_row, y_zero, x,
                                  place_gathers(ctx, T) ? ctx->x_perm : nullptr, s, true));
        prof_mark(ctx, 4, s);
        slots[n_slots++] = 4;
    }
    if (!place_gathers(ctx, T)) {
        LM_CUDA(ctx, launch_gather_rows(x, ctx->row_token, T * K, H, ctx->x_perm, s, true));
        prof_mark(ctx, 0, s);
        slots[n_slots++] = 0;
    }
    // Prefill-sized token tiles run on CTA pairs (256-row weight tiles); each CTA
    // loads half of a token tile, so the token maps' boxes are bn/2 rows.
    const bool pair = bn == 256;
    CUtensorMap map_x{};
    std::string err;
    if (!encode_tensor_map_bf16(&map_x, x, T, H, pair ? bn / 2 : bn, 64, err))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    GemmArgs args{};
    args.sched = ctx->sched;
    args.x = x;
    args.h = ctx->h;
    args.y = y;
    args.row_token = ctx->row_token;
    args.row_weight = ctx->row_weight;
    args.status = ctx->status;
    args.tokens = T;
    args.hidden = H;
    args.inter = I;
    args.n_routed_local = ctx->local_experts;
    args.split_ws = ctx->split_ws;
    args.split_ticket = ctx->split_ticket;
    args.split_ws_floats = static_cast<int32_t>(kSplitWsBytes / sizeof(float));
    args.split_max_waves = ctx->split_max_waves;
    if (pair) {
        const int hi = bn_index(bn / 2);
        LM_CUDA(ctx, launch_gemm_gate_up_pair(bn, L.map_w13, ctx->map_xperm[hi], map_x, args, ctx->sms, s, true));
        prof_mark(ctx, 5, s);
        slots[n_slots++] = 5;
        LM_CUDA(ctx, launch_gemm_down_pair(bn, L.map_w2, ctx->map_h[hi], args, ctx->sms, s, true));
    } else {
        LM_CUDA(ctx, launch_gemm_gate_up(bn, L.map_w13, ctx->map_xperm[bi], map_x, args, ctx->sms, s, true));
        prof_mark(ctx, 5, s);
        slots[n_slots++] = 5;
        LM_CUDA(ctx, launch_gemm_down(bn, L.map_w2, ctx->map_h[bi], args, ctx->sms, s, true));
    }
    prof_mark(ctx, 6, s);
    slots[n_slots++] = 6;
    return prof_end(ctx, slots, n_slots);
}

#define LM_NCCL(ctx, expr)                                                                       \
    do {                                                                                         \
        const ncclResult_t lm_r_ = (expr);                                                       \
        if (lm_r_ != ncclSuccess)                                                                \
            return fail(ctx, LM_ERR_COMM, std::string(#expr) + ": " + ctx->nccl->GetErrorString(lm_r_)); \
    } while (0)

// Expert-parallel forward.  Every rank runs this same sequence of collectives.
// Expert parallelism for small batches: every rank pair exchanges a fixed block of
// ep_cap rows, so the counts travel with the rows in one NCCL group and the receiver
// plans on the device -- no host round trip per layer.  Steps after routing: pack
// rows into destination blocks, exchange counts + rows, sort expert-major, schedule,
// the grouped GEMMs, return the blocks, weighted combine.
static lm_status forward_ep_fixed(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, int32_t T, float* y,
                                  cudaStream_t s, int* slots, int n_slots) {
    const lm_moe_config& c = ctx->cfg;
    const LayerWeights& L = ctx->layers[layer];
    const int K = c.num_experts_per_tok, E = c.n_routed_experts, H = c.hidden_size, I = c.moe_intermediate_size;
    const int N = ctx->nranks, El = ctx->local_experts, cap = ctx->ep_cap;
    const NcclApi& nc = *ctx->nccl;
    LM_CUDA(ctx, launch_ep_pack(x, ctx->row_token, ctx->expert_totals, ctx->slot_row, ctx->x_send, T, K, E, El, cap, H,
                                s, true));
    prof_mark(ctx, 1, s);
    slots[n_slots++] = 1;
    const size_t block = static_cast<size_t>(cap) * H;
    LM_NCCL(ctx, nc.GroupStart());
    for (int d = 0; d < N; ++d) {
        LM_NCCL(ctx, nc.Send(ctx->expert_totals + d * El, El, ncclInt32, d, ctx->comm, s));
        LM_NCCL(ctx, nc.Recv(ctx->recv_counts + d * El, El, ncclInt32, d, ctx->comm, s));
        LM_NCCL(ctx, nc.Send(ctx->x_send + d * block, block, ncclBfloat16, d, ctx->comm, s));
        LM_NCCL(ctx, nc.Recv(ctx->x_recv + d * block, block, ncclBfloat16, d, ctx->comm, s));
    }
    LM_NCCL(ctx, nc.GroupEnd());
    // The receiver does not know its row counts on the host: the GEMM tile width
    // comes from the expected rows per local expert (every rank at T tokens).
    const int bn = std::min(choose_bn(N * std::max(T, 1), K, E), 128);
    const int bi = bn_index(bn);
    LM_CUDA(ctx, launch_ep_sort_rows(ctx->x_recv, ctx->x_sorted, ctx->ep_row_src, ctx->recv_counts, N, El, cap, H, cap,
                                     0, El, s, false));
    LM_CUDA(ctx, launch_ep_schedule(ctx->recv_counts, ctx->sched_ep, N, El, c.n_shared_experts, T, ctx->routed_cap, bn,
                                    2 * I / 128, H / 128, s, true));
    prof_mark(ctx, 7, s);
    slots[n_slots++] = 7;
    CUtensorMap map_x{};
    std::string err;
    if (!encode_tensor_map_bf16(&map_x, T > 0 ? x : ctx->x_perm, std::max(T, 1), H, bn, 64, err))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    GemmArgs args{};
    args.sched = ctx->sched_ep;
    args.x = x;
    args.h = ctx->h;
    args.y = y;
    args.y_rows = ctx->y_ret;
    args.y_rows_map = ctx->ep_row_src;
    args.y_rows_cap = ctx->routed_cap;
    args.status = ctx->status;
    args.tokens = T;
    args.hidden = H;
    args.inter = I;
    args.n_routed_local = El;
    args.split_ws = ctx->split_ws;
    args.split_ticket = ctx->split_ticket;
    args.split_ws_floats = static_cast<int32_t>(kSplitWsBytes / sizeof(float));
    args.split_max_waves = ctx->split_max_waves;
    LM_CUDA(ctx, launch_gemm_gate_up(bn, L.map_w13, ctx->map_xsorted[bi], map_x, args, ctx->sms, s, true));
    prof_mark(ctx, 5, s);
    slots[n_slots++] = 5;
    LM_CUDA(ctx, launch_gemm_down(bn, L.map_w2, ctx->map_h[bi], args, ctx->sms, s, true));
    prof_mark(ctx, 6, s);
    slots[n_slots++] = 6;
    LM_NCCL(ctx, nc.GroupStart());
    for (int d = 0; d < N; ++d) {
        LM_NCCL(ctx, nc.Send(ctx->y_ret + d * block, block, ncclBfloat16, d, ctx->comm, s));
        LM_NCCL(ctx, nc.Recv(ctx->y_back + d * block, block, ncclBfloat16, d, ctx->comm, s));
    }
    LM_NCCL(ctx, nc.GroupEnd());
    LM_CUDA(ctx, launch_ep_combine(y, ctx->y_back, ctx->slot_row, ctx->topk_w, T, K, H, s, false));
    prof_mark(ctx, 4, s);
    slots[n_slots++] = 4;
    return prof_end(ctx, slots, n_slots);
}

static lm_status forward_ep(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, const float* x_f32, int32_t T,
                            const float* bias, float* y, int32_t accumulate, cudaStream_t s) {
    const lm_moe_config& c = ctx->cfg;
    const LayerWeights& L = ctx->layers[layer];
    const int K = c.num_experts_per_tok, E = c.n_routed_experts, H = c.hidden_size, I = c.moe_intermediate_size;
    const int N = ctx->nranks, El = ctx->local_experts;
    if (ctx->ep_aborted)
        return fail(ctx, LM_ERR_COMM, "expert parallelism on this context ended when a peer missed an exchange");
    const NcclApi& nc = *ctx->nccl;
    const RouterParams rp = router_params(c);
    float* y_zero = accumulate ? nullptr : y;
    prof_begin(ctx, s);
    int slots[8];
    int n_slots = 0;
    // 1. Route this rank's tokens over all experts; rows sorted by expert are
    //    sorted by destination rank, so x_perm is the send buffer.
    if (T > 0 && T <= kRouteTile) {
        LM_CUDA(ctx, launch_route_small(x, x_f32, L.router, bias, ctx->logits, T, H, rp, ctx->topk_idx, ctx->topk_w,
                                        ctx->expert_totals, ctx->sched, ctx->row_token, ctx->row_weight,
                                        ctx->slot_row, y_zero, ctx->ticket, 0, 0, E, 0, 16, 1, 1, s, false));
    } else if (T > 0) {
        lm_status rst;
        RouterFix fix;
        if ((rst = router_logits(ctx, L, x, x_f32, T, bias, ctx->logits, s, false, &fix)) != LM_OK) return rst;
        LM_CUDA(ctx, launch_router_topk(ctx->logits, T, rp, ctx->topk_idx, ctx->topk_w, ctx->tile_counts, s, true, fix));
        LM_CUDA(ctx, launch_dispatch_scan(ctx->tile_counts, ctx->tile_base, ctx->expert_totals, ctx->sched, T, K, E,
                                          0, 0, E, 0, 16, 1, 1, s, true));
        // Host-planned exchange: x_perm is the send buffer, filled by the placement
        // when its grid is large enough (see forward_impl), else by the gather below.
        LM_CUDA(ctx, launch_place(ctx->topk_idx, ctx->topk_w, ctx->tile_base, T, H, K, E, 0, E, ctx->row_token,
                                  ctx->row_weight, ctx->slot_row, y_zero, x,
                                  ctx->ep_cap == 0 && place_gathers(ctx, T) ? ctx->x_perm : nullptr, s, true));
    } else {
        LM_CUDA(ctx, cudaMemsetAsync(ctx->expert_totals, 0, E * sizeof(int32_t), s));
    }
    if (ctx->ep_cap > 0) return forward_ep_fixed(ctx, layer, x, T, y, s, slots, n_slots);
    if (T > 0 && !place_gathers(ctx, T))
        LM_CUDA(ctx, launch_gather_rows(x, ctx->row_token, T * K, H, ctx->x_perm, s, true));
    prof_mark(ctx, 1, s);
    slots[n_slots++] = 1;
    // 2. Rows per (destination, expert) to every rank; one host sync to plan.  The
    //    copy-engine exchange needs every rank's counts (where its rows sit in every
    //    peer's buffers): all-gather them, and derive this rank's own slices.
    const int32_t* counts_all = nullptr;  // copy mode: [N, E] rows each rank sends to each expert
    if (ctx->ep_copy) {
        LM_NCCL(ctx, nc.GroupStart());
        for (int d = 0; d < N; ++d) {
            LM_NCCL(ctx, nc.Send(ctx->expert_totals, E, ncclInt32, d, ctx->comm, s));
            LM_NCCL(ctx, nc.Recv(ctx->counts_all + d * E, E, ncclInt32, d, ctx->comm, s));
        }
        LM_NCCL(ctx, nc.GroupEnd());
        LM_CUDA(ctx, cudaMemcpyAsync(ctx->host_counts_all, ctx->counts_all, static_cast<size_t>(N) * E * sizeof(int32_t),
                                     cudaMemcpyDeviceToHost, s));
        if (const lm_status ws = ep_wait_stream(ctx, s, "expert-parallel row counts"); ws != LM_OK) return ws;
        counts_all = ctx->host_counts_all;
        // Every rank's counts locate rows in its own and its peers' buffers: they are
        // checked before any copy uses them (each rank sends at most routed_cap rows).
        for (int r = 0; r < N; ++r) {
            int64_t sum = 0;
            for (int e = 0; e < E; ++e) sum += counts_all[r * E + e] < 0 ? INT32_MAX : counts_all[r * E + e];
            if (sum > ctx->routed_cap)
                return ep_give_up(ctx, s, "expert-parallel row counts: rank " + std::to_string(r) +
                                              "'s do not fit its send buffer");
        }
        for (int e = 0; e < E; ++e) ctx->host_totals[e] = counts_all[ctx->rank * E + e];
        for (int r = 0; r < N; ++r)
            for (int e = 0; e < El; ++e) ctx->host_recv[r * El + e] = counts_all[r * E + ctx->rank * El + e];
        LM_CUDA(ctx, cudaMemcpyAsync(ctx->recv_counts, ctx->host_recv, static_cast<size_t>(N) * El * sizeof(int32_t),
                                     cudaMemcpyHostToDevice, s));
    } else {
        LM_NCCL(ctx, nc.GroupStart());
        for (int d = 0; d < N; ++d) {
            LM_NCCL(ctx, nc.Send(ctx->expert_totals + d * El, El, ncclInt32, d, ctx->comm, s));
            LM_NCCL(ctx, nc.Recv(ctx->recv_counts + d * El, El, ncclInt32, d, ctx->comm, s));
        }
        LM_NCCL(ctx, nc.GroupEnd());
        LM_CUDA(ctx, cudaMemcpyAsync(ctx->host_totals, ctx->expert_totals, E * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                     s));
        LM_CUDA(ctx, cudaMemcpyAsync(ctx->host_recv, ctx->recv_counts, N * El * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                     s));
        if (const lm_status ws = ep_wait_stream(ctx, s, "expert-parallel row counts"); ws != LM_OK) return ws;
        for (int r = 0; r < N; ++r) {  // the receive buffer holds routed_cap rows per source
            int64_t sum = 0;
            for (int e = 0; e < El; ++e)
                sum += ctx->host_recv[r * El + e] < 0 ? INT32_MAX : ctx->host_recv[r * El + e];
            if (sum > ctx->routed_cap)
                return ep_give_up(ctx, s, "expert-parallel row counts: rank " + std::to_string(r) +
                                              "'s do not fit the receive buffer");
        }
    }
    lm_ep_plan total;
    if (lm_moe_ep_plan(N, E, ctx->host_totals, ctx->host_recv, &total) != LM_OK)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "invalid expert-parallel plan");
    // The local experts move in C chunks (lm_moe_ep_chunk_plan).  C = 1: one exchange
    // each way, all on the caller's stream.  C > 1: every chunk's rows go out on the
    // exchange stream at once; the caller's stream runs the shared experts (they need
    // no rows from other ranks), then each chunk's sort and GEMMs as its rows arrive,
    // and each chunk's outputs go back while the next chunk computes.  The GEMMs then
    // leave ep_nccl_ctas SMs to NCCL's kernels (capped to that many CTAs at init).
    const int C = ctx->ep_chunks;
    const bool piped = C > 1;
    // NCCL's kernels run beside the chunked GEMMs and need SMs of their own; copy
    // engines do not.
    const int gemm_sms = piped && !ctx->ep_copy ? std::max(2, (ctx->sms - ctx->ep_nccl_ctas) & ~1) : ctx->sms;
    lm_ep_plan plans[kEpMaxChunks];
    for (int k = 0; k < C; ++k)
        if (lm_moe_ep_chunk_plan(N, E, C, k, ctx->host_totals, ctx->host_recv, &plans[k]) != LM_OK)
            return fail(ctx, LM_ERR_INVALID_ARGUMENT, "invalid expert-parallel plan");
    // Receiver schedules: one segment per local expert (its rows from every source,
    // made contiguous by ep_sort_rows after the dispatch; expert-major over all
    // chunks), then the shared experts -- in chunk 0's schedule when C = 1, else in
    // a schedule of their own (slot C).
    const int bn = choose_bn(total.n_recv, 1, El);  // from the mean rows per local expert
    const int bi = bn_index(bn);
    const int mb1 = 2 * I / 128, mb2 = H / 128;
    int expert_row[kMaxExperts + 1];  // first expert-major row of each local expert
    expert_row[0] = 0;
    for (int e = 0; e < El; ++e) {
        int cnt = 0;
        for (int r = 0; r < N; ++r) cnt += ctx->host_recv[r * El + e];
        expert_row[e + 1] = expert_row[e] + cnt;
    }
    auto build = [&](Schedule& hs, int e_lo, int e_hi, bool shared) {
        int p1 = 0, p2 = 0, seg = 0;
        auto add_segment = [&](int off, int cnt, int wslot) {
            hs.seg_off[seg] = off;
            hs.seg_cnt[seg] = cnt;
            hs.seg_weight[seg] = wslot;
            hs.tiles1[seg] = p1;
            hs.tiles2[seg] = p2;
            const int nb = (cnt + bn - 1) / bn;
            p1 += nb * mb1;
            p2 += nb * mb2;
            ++seg;
        };
        for (int e = e_lo; e < e_hi; ++e) add_segment(expert_row[e], expert_row[e + 1] - expert_row[e], e);
        if (shared)
            for (int j = 0; j < c.n_shared_experts; ++j) add_segment(ctx->routed_cap + j * T, T, El + j);
        hs.tiles1[seg] = p1;
        hs.tiles2[seg] = p2;
        hs.n_seg = seg;
        hs.first_expert = ctx->first_expert;
    };
    int max_group[kEpMaxChunks];
    for (int k = 0; k < C; ++k) {
        const int e_lo = k * El / C, e_hi = (k + 1) * El / C;
        build(ctx->host_sched[k], e_lo, e_hi, !piped);
        max_group[k] = 0;
        for (int r = 0; r < N; ++r)
            for (int e = e_lo; e < e_hi; ++e) max_group[k] = std::max(max_group[k], ctx->host_recv[r * El + e]);
    }
    if (piped) build(ctx->host_sched[C], 0, 0, true);
    const int n_sched = C + (piped ? 1 : 0);
    LM_CUDA(ctx, cudaMemcpyAsync(ctx->sched_ep, ctx->host_sched, n_sched * sizeof(Schedule), cudaMemcpyHostToDevice, s));
    // One NCCL group per chunk and direction: rows out (x_perm -> x_recv) or expert
    // outputs back (y_ret -> y_back, the same offsets reversed).
    auto exchange = [&](int k, bool back, cudaStream_t st) -> lm_status {
        const lm_ep_plan& pk = plans[k];
        LM_NCCL(ctx, nc.GroupStart());
        for (int d = 0; d < N; ++d) {
            uint16_t* out = back ? ctx->y_ret + static_cast<size_t>(pk.recv_offset[d]) * H
                                 : ctx->x_perm + static_cast<size_t>(pk.send_offset[d]) * H;
            uint16_t* in = back ? ctx->y_back + static_cast<size_t>(pk.send_offset[d]) * H
                                : ctx->x_recv + static_cast<size_t>(pk.recv_offset[d]) * H;
            const size_t n_out = static_cast<size_t>(back ? pk.recv_count[d] : pk.send_count[d]) * H;
            const size_t n_in = static_cast<size_t>(back ? pk.send_count[d] : pk.recv_count[d]) * H;
            if (n_out > 0) LM_NCCL(ctx, nc.Send(out, n_out, ncclBfloat16, d, ctx->comm, st));
            if (n_in > 0) LM_NCCL(ctx, nc.Recv(in, n_in, ncclBfloat16, d, ctx->comm, st));
        }
        LM_NCCL(ctx, nc.GroupEnd());
        return LM_OK;
    };
    // 4. Local experts on the received rows, shared experts on this rank's tokens.
    CUtensorMap map_x{};
    std::string err;
    const bool pair = bn == 256;
    // A rank without tokens still serves its experts; its (unread) token map points
    // at a workspace buffer.
    if (!encode_tensor_map_bf16(&map_x, T > 0 ? x : ctx->x_perm, std::max(T, 1), H, pair ? bn / 2 : bn, 64, err))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, err);
    GemmArgs args{};
    args.x = x;
    args.h = ctx->h;
    args.y = y;
    args.y_rows = ctx->y_ret;
    args.y_rows_map = ctx->ep_row_src;
    args.y_rows_cap = ctx->routed_cap;
    args.row_token = ctx->row_token;
    args.row_weight = ctx->row_weight;
    args.status = ctx->status;
    args.tokens = T;
    args.hidden = H;
    args.inter = I;
    args.n_routed_local = El;
    args.split_ws = ctx->split_ws;
    args.split_ticket = ctx->split_ticket;
    args.split_ws_floats = static_cast<int32_t>(kSplitWsBytes / sizeof(float));
    args.split_max_waves = ctx->split_max_waves;
    auto gemms = [&](int slot, bool mark) -> lm_status {
        args.sched = ctx->sched_ep + slot;
        // The kernels take segments [0, n_routed_local) as routed (rows from x_sorted,
        // outputs to y_ret) and the rest as shared (rows from x, outputs into y): the
        // shared experts' own schedule has no routed segment.
        args.n_routed_local = piped && slot == C ? 0 : El;
        if (pair) {
            const int hi = bn_index(bn / 2);
            LM_CUDA(ctx, launch_gemm_gate_up_pair(bn, L.map_w13, ctx->map_xsorted[hi], map_x, args, gemm_sms, s, true));
            if (mark) {
                prof_mark(ctx, 5, s);
                slots[n_slots++] = 5;
            }
            LM_CUDA(ctx, launch_gemm_down_pair(bn, L.map_w2, ctx->map_h[hi], args, gemm_sms, s, true));
        } else {
            LM_CUDA(ctx, launch_gemm_gate_up(bn, L.map_w13, ctx->map_xsorted[bi], map_x, args, gemm_sms, s, true));
            if (mark) {
                prof_mark(ctx, 5, s);
                slots[n_slots++] = 5;
            }
            LM_CUDA(ctx, launch_gemm_down(bn, L.map_w2, ctx->map_h[bi], args, gemm_sms, s, true));
        }
        if (mark) {
            prof_mark(ctx, 6, s);
            slots[n_slots++] = 6;
        }
        return LM_OK;
    };
    auto sort = [&](int k, cudaStream_t st, bool pdl) -> lm_status {
        LM_CUDA(ctx, launch_ep_sort_rows(ctx->x_recv, ctx->x_sorted, ctx->ep_row_src, ctx->recv_counts, N, El,
                                         max_group[k], H, 0, k * El / C, (k + 1) * El / C, st, pdl));
        return LM_OK;
    };
    lm_status st;
    if (ctx->ep_copy) {
        // Copy-engine exchange.  Owner d's receive buffer holds chunk after chunk, source
        // after source within a chunk; rank r's send buffer is sorted by global expert.
        const int me = ctx->rank;
        auto chunk_lo = [&](int k) { return k * El / C; };
        auto rows_to = [&](int r, int d, int k) {  // rows rank r sends to owner d's chunk-k experts
            int n = 0;
            for (int e = chunk_lo(k); e < chunk_lo(k + 1); ++e) n += counts_all[r * E + d * El + e];
            return n;
        };
        auto send_off = [&](int r, int d, int k) {  // where they start in r's send buffer
            int n = 0;
            for (int e = 0; e < d * El + chunk_lo(k); ++e) n += counts_all[r * E + e];
            return n;
        };
        auto recv_off = [&](int d, int r, int k) {  // where they land in d's receive buffer
            int n = 0;
            for (int kk = 0; kk < k; ++kk)
                for (int rr = 0; rr < N; ++rr) n += rows_to(rr, d, kk);
            for (int rr = 0; rr < r; ++rr) n += rows_to(rr, d, k);
            return n;
        };
        const uint32_t epoch = ++ctx->ep_epoch;
        const uint64_t limit = ctx->debug_wait_limit_ns != 0 ? ctx->debug_wait_limit_ns : kWaitLimitNs;
        const size_t row_bytes = static_cast<size_t>(H) * sizeof(uint16_t);
        // Flag slots: [r] rank r's rows are in its send buffer; [N + k N + r] rank r's
        // outputs for chunk k are in its y_ret.
        auto slot_rows = [&](int r) { return r; };
        auto slot_out = [&](int k, int r) { return N + k * N + r; };
        const bool tl = ctx->profiling;
        if (tl && ctx->ep_tl_events[0] == nullptr)
            for (auto& e : ctx->ep_tl_events) LM_CUDA(ctx, cudaEventCreate(&e));
        auto stamp = [&](int i) -> lm_status {
            if (tl) LM_CUDA(ctx, cudaEventRecord(ctx->ep_tl_events[i], s));
            return LM_OK;
        };
        if ((st = stamp(LM_EP_TIMELINE_MAX)) != LM_OK) return st;
        // This rank's rows are in x_perm: every peer may pull its share.
        LM_CUDA(ctx, launch_ep_signal(ctx->ep_peer_flags, me, slot_rows(me), epoch, s));
        for (int k = 0; k < C; ++k) {
            const int n = rows_to(me, me, k);
            if (n > 0)
                LM_CUDA(ctx, cudaMemcpyAsync(ctx->x_recv + static_cast<size_t>(recv_off(me, me, k)) * H,
                                             ctx->x_perm + static_cast<size_t>(send_off(me, me, k)) * H, n * row_bytes,
                                             cudaMemcpyDeviceToDevice, s));
        }
        // Per peer, on its copy stream: wait for its rows, pull them chunk by chunk; then,
        // chunk by chunk, wait for its outputs of this rank's rows and pull those back.
        for (int r = 0; r < N; ++r) {
            if (r == me) continue;
            cudaStream_t cs = ctx->ep_copy_stream[r];
            LM_CUDA(ctx, launch_ep_wait(ctx->ep_flags, slot_rows(r), epoch, ctx->status, ep_diag(ctx), limit, cs));
            for (int k = 0; k < C; ++k) {
                const int n = rows_to(r, me, k);
                if (n > 0)
                    LM_CUDA(ctx, cudaMemcpyAsync(ctx->x_recv + static_cast<size_t>(recv_off(me, r, k)) * H,
                                                 ctx->ep_peer_xperm[r] + static_cast<size_t>(send_off(r, me, k)) * H,
                                                 n * row_bytes, cudaMemcpyDeviceToDevice, cs));
                LM_CUDA(ctx, cudaEventRecord(ctx->ep_ev_pulled[k][r], cs));
            }
            for (int k = 0; k < C; ++k) {
                LM_CUDA(ctx, launch_ep_wait(ctx->ep_flags, slot_out(k, r), epoch, ctx->status, ep_diag(ctx), limit, cs));
                const int n = rows_to(me, r, k);
                if (n > 0)
                    LM_CUDA(ctx, cudaMemcpyAsync(ctx->y_back + static_cast<size_t>(send_off(me, r, k)) * H,
                                                 ctx->ep_peer_yret[r] + static_cast<size_t>(recv_off(r, me, k)) * H,
                                                 n * row_bytes, cudaMemcpyDeviceToDevice, cs));
            }
            LM_CUDA(ctx, cudaEventRecord(ctx->ep_ev_returned[r], cs));
        }
        prof_mark(ctx, 7, s);
        slots[n_slots++] = 7;
        // The shared experts need no peer rows: they run while the first chunk arrives.
        if (piped && (st = gemms(C, false)) != LM_OK) return st;
        if ((st = stamp(C)) != LM_OK) return st;
        for (int k = 0; k < C; ++k) {
            for (int r = 0; r < N; ++r)
                if (r != me) LM_CUDA(ctx, cudaStreamWaitEvent(s, ctx->ep_ev_pulled[k][r], 0));
            if ((st = stamp(k)) != LM_OK) return st;
            if ((st = stamp(C + 1 + k)) != LM_OK) return st;
            if ((st = sort(k, s, false)) != LM_OK) return st;
            if ((st = gemms(k, false)) != LM_OK) return st;
            if ((st = stamp(2 * C + 1 + k)) != LM_OK) return st;
            // This rank's outputs of chunk k are in y_ret: the peers may pull theirs back.
            LM_CUDA(ctx, launch_ep_signal(ctx->ep_peer_flags, me, slot_out(k, me), epoch, s));
            const int n = rows_to(me, me, k);
            if (n > 0)
                LM_CUDA(ctx, cudaMemcpyAsync(ctx->y_back + static_cast<size_t>(send_off(me, me, k)) * H,
                                             ctx->y_ret + static_cast<size_t>(recv_off(me, me, k)) * H, n * row_bytes,
                                             cudaMemcpyDeviceToDevice, s));
        }
        prof_mark(ctx, 5, s);
        slots[n_slots++] = 5;
        for (int r = 0; r < N; ++r)
            if (r != me) LM_CUDA(ctx, cudaStreamWaitEvent(s, ctx->ep_ev_returned[r], 0));
        for (int k = 0; k < C; ++k)
            if ((st = stamp(3 * C + 1 + k)) != LM_OK) return st;
        LM_CUDA(ctx, launch_ep_combine(y, ctx->y_back, ctx->slot_row, ctx->topk_w, T, K, H, s, false));
        if ((st = stamp(4 * C + 1)) != LM_OK) return st;
        prof_mark(ctx, 4, s);
        slots[n_slots++] = 4;
        if ((st = prof_end(ctx, slots, n_slots)) != LM_OK) return st;
        if (tl) {
            for (int i = 0; i <= 4 * C + 1; ++i)
                LM_CUDA(ctx, cudaEventElapsedTime(&ctx->ep_timeline[i], ctx->ep_tl_events[LM_EP_TIMELINE_MAX],
                                                  ctx->ep_tl_events[i]));
            ctx->ep_timeline_chunks = C;
        }
        return LM_OK;
    }
    if (!piped) {
        // 3. Dispatch token rows.
        if ((st = exchange(0, false, s)) != LM_OK) return st;
        if ((st = sort(0, s, false)) != LM_OK) return st;
        prof_mark(ctx, 7, s);
        slots[n_slots++] = 7;
        if ((st = gemms(0, true)) != LM_OK) return st;
        // 5. Outputs back to the tokens' ranks, then the weighted combine.
        if ((st = exchange(0, true, s)) != LM_OK) return st;
    } else {
        cudaStream_t cs = ctx->ep_stream;
        // While profiling, timing events mark each step's end (lm_moe_profile_ep_timeline).
        const bool tl = ctx->profiling;
        if (tl && ctx->ep_tl_events[0] == nullptr)
            for (auto& e : ctx->ep_tl_events) LM_CUDA(ctx, cudaEventCreate(&e));
        auto stamp = [&](int i, cudaStream_t st) -> lm_status {
            if (tl) LM_CUDA(ctx, cudaEventRecord(ctx->ep_tl_events[i], st));
            return LM_OK;
        };
        if ((st = stamp(LM_EP_TIMELINE_MAX, s)) != LM_OK) return st;  // the origin
        LM_CUDA(ctx, cudaEventRecord(ctx->ep_ev_ready, s));
        LM_CUDA(ctx, cudaStreamWaitEvent(cs, ctx->ep_ev_ready, 0));
        for (int k = 0; k < C; ++k) {
            if ((st = exchange(k, false, cs)) != LM_OK) return st;
            LM_CUDA(ctx, cudaEventRecord(ctx->ep_ev_sent[k], cs));
            if ((st = stamp(k, cs)) != LM_OK) return st;
        }
        prof_mark(ctx, 7, s);
        slots[n_slots++] = 7;
        if ((st = gemms(C, false)) != LM_OK) return st;  // shared experts
        if ((st = stamp(C, s)) != LM_OK) return st;
        for (int k = 0; k < C; ++k) {
            LM_CUDA(ctx, cudaStreamWaitEvent(s, ctx->ep_ev_sent[k], 0));
            if ((st = stamp(C + 1 + k, s)) != LM_OK) return st;
            if ((st = sort(k, s, false)) != LM_OK) return st;
            if ((st = gemms(k, false)) != LM_OK) return st;
            LM_CUDA(ctx, cudaEventRecord(ctx->ep_ev_done[k], s));
            if ((st = stamp(2 * C + 1 + k, s)) != LM_OK) return st;
            LM_CUDA(ctx, cudaStreamWaitEvent(cs, ctx->ep_ev_done[k], 0));
            if ((st = exchange(k, true, cs)) != LM_OK) return st;
            if ((st = stamp(3 * C + 1 + k, cs)) != LM_OK) return st;
        }
        prof_mark(ctx, 5, s);
        slots[n_slots++] = 5;
        LM_CUDA(ctx, cudaEventRecord(ctx->ep_ev_back, cs));
        LM_CUDA(ctx, cudaStreamWaitEvent(s, ctx->ep_ev_back, 0));
        LM_CUDA(ctx, launch_ep_combine(y, ctx->y_back, ctx->slot_row, ctx->topk_w, T, K, H, s, false));
        if ((st = stamp(4 * C + 1, s)) != LM_OK) return st;
        prof_mark(ctx, 4, s);
        slots[n_slots++] = 4;
        if ((st = prof_end(ctx, slots, n_slots)) != LM_OK) return st;
        if (tl) {
            for (int i = 0; i <= 4 * C + 1; ++i)
                LM_CUDA(ctx, cudaEventElapsedTime(&ctx->ep_timeline[i], ctx->ep_tl_events[LM_EP_TIMELINE_MAX],
                                                  ctx->ep_tl_events[i]));
            ctx->ep_timeline_chunks = C;
        }
        return LM_OK;
    }
    LM_CUDA(ctx, launch_ep_combine(y, ctx->y_back, ctx->slot_row, ctx->topk_w, T, K, H, s, false));
    prof_mark(ctx, 4, s);
    slots[n_slots++] = 4;
    return prof_end(ctx, slots, n_slots);
}

lm_status lm_moe_forward(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, int32_t tokens, const float* logit_bias,
                         float* y, int32_t accumulate, void* stream) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    lm_status st;
    if ((st = check_layer(ctx, layer)) != LM_OK) return st;
    if (tokens < 0) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "negative token count");
    if (tokens > ctx->cfg.max_tokens) return fail(ctx, LM_ERR_TOO_MANY_TOKENS, "tokens exceed max_tokens");
    if (tokens == 0 && ctx->nranks == 1) return LM_OK;  // with experts on several ranks, this one still serves
    if (tokens > 0 && (x == nullptr || y == nullptr || !aligned16(x) || !aligned16(y)))
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "x and y must be 16-byte aligned device pointers");
    if ((st = set_device(ctx)) != LM_OK) return st;
    if (ctx->nranks > 1 || ctx->ep_single)
        return forward_ep(ctx, layer, x, nullptr, tokens, logit_bias, y, accumulate, static_cast<cudaStream_t>(stream));
    return forward_impl(ctx, layer, x, nullptr, tokens, logit_bias, y, accumulate, static_cast<cudaStream_t>(stream));
}

lm_status lm_moe_forward_host(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x_host, int32_t tokens,
                              const float* logit_bias_host, float* y_host) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    lm_status st;
    if ((st = check_layer(ctx, layer)) != LM_OK) return st;
    if (tokens < 0) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "negative token count");
    if (tokens > ctx->cfg.max_tokens) return fail(ctx, LM_ERR_TOO_MANY_TOKENS, "tokens exceed max_tokens");
    if (tokens == 0) return LM_OK;
    if (x_host == nullptr || y_host == nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "null host buffer");
    if ((st = set_device(ctx)) != LM_OK) return st;
    const lm_moe_config& c = ctx->cfg;
    const size_t T = c.max_tokens, H = c.hidden_size;
    if (ctx->x_stage == nullptr) {
        LM_CUDA(ctx, cudaMalloc(&ctx->x_stage, T * H * sizeof(uint16_t)));
        LM_CUDA(ctx, cudaMalloc(&ctx->y_stage, T * H * sizeof(float)));
        LM_CUDA(ctx, cudaMalloc(&ctx->bias_stage, static_cast<size_t>(c.n_routed_experts) * sizeof(float)));
        LM_CUDA(ctx, cudaMallocHost(&ctx->status_host, sizeof(int32_t)));
        LM_CUDA(ctx, cudaHostGetDevicePointer(reinterpret_cast<void**>(&ctx->status_host_dev), ctx->status_host, 0));
        LM_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking));
    }
    cudaStream_t s = ctx->own_stream;
    const size_t n = static_cast<size_t>(tokens) * H;
    const size_t x_bytes = n * sizeof(uint16_t), y_bytes = n * sizeof(float);
    const size_t bias_bytes = static_cast<size_t>(c.n_routed_experts) * sizeof(float);
    // Pinned buffers are mapped into the device's address space: SMs move them (no
    // copy-engine transfer and its fixed cost).  Pageable or unaligned ones are copied.
    const void* x_map = host_io_eligible(x_host, x_bytes) ? mapped_device_address(x_host) : nullptr;
    const void* bias_map = logit_bias_host != nullptr && host_io_eligible(logit_bias_host, bias_bytes)
                               ? mapped_device_address(logit_bias_host)
                               : nullptr;
    void* y_map = host_io_eligible(y_host, y_bytes) ? const_cast<void*>(mapped_device_address(y_host)) : nullptr;
    const bool bias_pulled = x_map != nullptr && bias_map != nullptr;
    if (x_map != nullptr)
        LM_CUDA(ctx, launch_host_pull(ctx->x_stage, x_map, x_bytes, ctx->bias_stage, bias_pulled ? bias_map : nullptr,
                                      bias_bytes, ctx->sms, s));
    else
        LM_CUDA(ctx, cudaMemcpyAsync(ctx->x_stage, x_host, x_bytes, cudaMemcpyHostToDevice, s));
    if (logit_bias_host != nullptr && !bias_pulled)
        LM_CUDA(ctx, cudaMemcpyAsync(ctx->bias_stage, logit_bias_host, bias_bytes, cudaMemcpyHostToDevice, s));
    const float* bias = logit_bias_host != nullptr ? ctx->bias_stage : nullptr;
    st = ctx->nranks > 1 || ctx->ep_single ? forward_ep(ctx, layer, ctx->x_stage, nullptr, tokens, bias, ctx->y_stage, 0, s)
                         : forward_impl(ctx, layer, ctx->x_stage, nullptr, tokens, bias, ctx->y_stage, 0, s);
    if (st != LM_OK) return st;
    // y and the status word come back in the same stream order: one synchronisation
    // covers both.
    if (y_map != nullptr) {
        LM_CUDA(ctx, launch_host_push(y_map, ctx->y_stage, y_bytes, ctx->status, ctx->status_host_dev, ctx->sms, s));
    } else {
        LM_CUDA(ctx, cudaMemcpyAsync(y_host, ctx->y_stage, y_bytes, cudaMemcpyDeviceToHost, s));
        LM_CUDA(ctx, cudaMemcpyAsync(ctx->status_host, ctx->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    }
    if ((st = ep_wait_stream(ctx, s, "lm_moe_forward_host")) != LM_OK) return st;
    return settle_status(ctx, *ctx->status_host);
}

lm_status lm_moe_block_forward(lm_moe_ctx* ctx, int32_t layer, float* hidden, int32_t tokens, void* stream) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    lm_status st;
    if ((st = check_layer(ctx, layer)) != LM_OK) return st;
    if (tokens < 0) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "negative token count");
    if (tokens > ctx->cfg.max_tokens) return fail(ctx, LM_ERR_TOO_MANY_TOKENS, "tokens exceed max_tokens");
    if (tokens == 0) return LM_OK;
    if (hidden == nullptr || !aligned16(hidden)) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "hidden must be aligned");
    if ((st = set_device(ctx)) != LM_OK) return st;
    const lm_moe_config& c = ctx->cfg;
    const size_t T = c.max_tokens, H = c.hidden_size;
    if (ctx->norm_f32 == nullptr) {
        LM_CUDA(ctx, cudaMalloc(&ctx->norm_f32, T * H * sizeof(float)));
        LM_CUDA(ctx, cudaMalloc(&ctx->norm_bf16, T * H * sizeof(uint16_t)));
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // src/DeepSeekRunner.cpp:265-267: rms_norm(post_attention_layernorm); the router
    // sees the f32 result (:273), the experts its bf16 rounding.
    LM_CUDA(ctx, launch_rms_norm_rows(hidden, ctx->norm_f32, ctx->norm_bf16, ctx->layers[layer].norm, tokens,
                                      c.hidden_size, c.rms_norm_eps, s));
    // The residual add (:290) is folded into the down-projection epilogue: it
    // accumulates straight into `hidden`.
    if (ctx->nranks > 1 || ctx->ep_single)
        return forward_ep(ctx, layer, ctx->norm_bf16, ctx->norm_f32, tokens, nullptr, hidden, 1, s);
    return forward_impl(ctx, layer, ctx->norm_bf16, ctx->norm_f32, tokens, nullptr, hidden, 1, s);
}

lm_status lm_moe_sync(lm_moe_ctx* ctx, void* stream) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    if ((st = ep_wait_stream(ctx, static_cast<cudaStream_t>(stream), "lm_moe_sync")) != LM_OK) return st;
    int32_t status = 0;
    LM_CUDA(ctx, cudaMemcpy(&status, ctx->status, sizeof(status), cudaMemcpyDeviceToHost));
    return settle_status(ctx, status);
}

lm_status lm_moe_debug_set(lm_moe_ctx* ctx, int32_t knob, int64_t value) {
    if (ctx == nullptr || value < 0) return LM_ERR_INVALID_ARGUMENT;
    switch (knob) {
        case LM_DEBUG_GRID_EXTRA:
            if (value > 1024) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "LM_DEBUG_GRID_EXTRA above 1024");
            ctx->debug_grid_extra = static_cast<uint32_t>(value);
            return LM_OK;
        case LM_DEBUG_WAIT_LIMIT_NS:
            if (value > static_cast<int64_t>(kWaitLimitNs))
                return fail(ctx, LM_ERR_INVALID_ARGUMENT, "LM_DEBUG_WAIT_LIMIT_NS above the 2 s default");
            ctx->debug_wait_limit_ns = static_cast<uint64_t>(value);
            return LM_OK;
        default:
            return fail(ctx, LM_ERR_INVALID_ARGUMENT, "unknown debug knob " + std::to_string(knob));
    }
}

lm_status lm_moe_expert_counts(lm_moe_ctx* ctx, int32_t* counts, int32_t capacity) {
    if (ctx == nullptr || counts == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (capacity < ctx->cfg.n_routed_experts)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT,
                    "counts holds " + std::to_string(capacity) + " slots; the context has " +
                        std::to_string(ctx->cfg.n_routed_experts) + " routed experts");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    LM_CUDA(ctx, cudaDeviceSynchronize());
    LM_CUDA(ctx, cudaMemcpy(counts, ctx->expert_totals, ctx->cfg.n_routed_experts * sizeof(int32_t),
                            cudaMemcpyDeviceToHost));
    return LM_OK;
}

lm_status lm_moe_memory(const lm_moe_ctx* ctx, uint64_t* resident_bytes, uint64_t* uploaded_bytes) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    if (resident_bytes) *resident_bytes = ctx->resident_bytes;
    if (uploaded_bytes) *uploaded_bytes = ctx->uploaded_bytes;
    return LM_OK;
}

lm_status lm_moe_profile_enable(lm_moe_ctx* ctx, int32_t enable) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    if (enable && ctx->prof_events[0] == nullptr) {
        for (auto& e : ctx->prof_events) LM_CUDA(ctx, cudaEventCreate(&e));
    }
    ctx->profiling = enable != 0;
    return LM_OK;
}

lm_status lm_moe_profile_read(lm_moe_ctx* ctx, double* total_ms, int64_t* launches, int32_t reset) {
    if (ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < LM_PROFILE_SLOTS; ++i) {
        if (total_ms) total_ms[i] = ctx->prof_ms[i];
        if (launches) launches[i] = ctx->prof_count[i];
        if (reset) {
            ctx->prof_ms[i] = 0.0;
            ctx->prof_count[i] = 0;
        }
    }
    return LM_OK;
}

lm_status lm_moe_profile_trace(lm_moe_ctx* ctx, uint64_t* stamps, int32_t ctas, int32_t* ctas_out) {
    if (ctx == nullptr || stamps == nullptr || ctas_out == nullptr || ctas < 0) return LM_ERR_INVALID_ARGUMENT;
    static_assert(LM_DECODE_TRACE_SLOTS == kDecodeTraceSlots, "trace layout");
    *ctas_out = 0;
    if (ctx->decode_trace == nullptr) return LM_OK;
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    const int n = std::min(ctas, ctx->sms);
    LM_CUDA(ctx, cudaDeviceSynchronize());
    LM_CUDA(ctx, cudaMemcpy(stamps, ctx->decode_trace, static_cast<size_t>(n) * kDecodeTraceSlots * 8,
                            cudaMemcpyDeviceToHost));
    *ctas_out = ctx->sms;
    return LM_OK;
}

static_assert(4 * kEpMaxChunks + 2 <= LM_EP_TIMELINE_MAX, "timeline layout");

lm_status lm_moe_profile_ep_timeline(lm_moe_ctx* ctx, float* ms, int32_t capacity, int32_t* chunks_out) {
    if (ctx == nullptr || ms == nullptr || chunks_out == nullptr || capacity < 0) return LM_ERR_INVALID_ARGUMENT;
    const int C = ctx->ep_timeline_chunks;
    *chunks_out = C;
    if (C > 0) std::memcpy(ms, ctx->ep_timeline, std::min(capacity, 4 * C + 2) * sizeof(float));
    return LM_OK;
}

lm_status lm_moe_ep_plan(int32_t nranks, int32_t experts, const int32_t* send_expert_counts,
                         const int32_t* recv_expert_counts, lm_ep_plan* plan) {
    return lm_moe_ep_chunk_plan(nranks, experts, 1, 0, send_expert_counts, recv_expert_counts, plan);
}

lm_status lm_moe_ep_chunk_plan(int32_t nranks, int32_t experts, int32_t chunks, int32_t chunk,
                               const int32_t* send_expert_counts, const int32_t* recv_expert_counts,
                               lm_ep_plan* plan) {
    if (plan == nullptr || send_expert_counts == nullptr || recv_expert_counts == nullptr || nranks < 1 ||
        nranks > LM_EP_MAX_RANKS || experts < 1 || experts % nranks != 0)
        return LM_ERR_INVALID_ARGUMENT;
    const int El = experts / nranks;
    if (chunks < 1 || chunks > El || chunk < 0 || chunk >= chunks) return LM_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < experts; ++i)
        if (send_expert_counts[i] < 0 || recv_expert_counts[i] < 0) return LM_ERR_INVALID_ARGUMENT;
    std::memset(plan, 0, sizeof(*plan));
    const int lo = chunk * El / chunks, hi = (chunk + 1) * El / chunks;
    // The send buffer is sorted by global expert: rank d's chunk is experts
    // d * El + [lo, hi).  The receive buffer holds whole chunks one after another.
    int64_t sent = 0, recv = 0;
    for (int d = 0; d < nranks; ++d)
        for (int e = 0; e < lo; ++e) recv += recv_expert_counts[d * El + e];
    for (int d = 0; d < nranks; ++d) {
        for (int e = 0; e < lo; ++e) sent += send_expert_counts[d * El + e];
        plan->send_offset[d] = static_cast<int32_t>(sent);
        plan->recv_offset[d] = static_cast<int32_t>(recv);
        for (int e = lo; e < hi; ++e) {
            plan->send_count[d] += send_expert_counts[d * El + e];
            plan->recv_count[d] += recv_expert_counts[d * El + e];
        }
        sent += plan->send_count[d];
        recv += plan->recv_count[d];
        for (int e = hi; e < El; ++e) sent += send_expert_counts[d * El + e];
        plan->n_send += plan->send_count[d];
        plan->n_recv += plan->recv_count[d];
    }
    if (sent > INT32_MAX || recv > INT32_MAX) return LM_ERR_INVALID_ARGUMENT;
    return LM_OK;
}

lm_status lm_moe_ep_unique_id(void* out) {
    if (out == nullptr) return LM_ERR_INVALID_ARGUMENT;
    std::string err;
    const NcclApi* nc = nccl_api(err);
    if (nc == nullptr) return LM_ERR_COMM;
    ncclUniqueId id;
    if (nc->GetUniqueId(&id) != ncclSuccess) return LM_ERR_COMM;
    std::memcpy(out, &id, sizeof(id));
    return LM_OK;
}

// Maps every peer's send rows (x_perm), returned outputs (y_ret) and flag slots into
// this process (IPC handles exchanged with one small NCCL all-gather) and creates one
// copy stream per peer.  Every rank calls it at lm_moe_ep_init; a peer is pulled from
// only after it has signalled, in a forward, so no rank maps a buffer before its owner
// finished this set-up.
static lm_status ep_copy_setup(lm_moe_ctx* ctx) {
    const int N = ctx->nranks, me = ctx->rank, E = ctx->cfg.n_routed_experts;
    const NcclApi& nc = *ctx->nccl;
    lm_status st;
    const size_t n_flags = ep_flag_slots(N);
    if ((st = alloc(ctx, &ctx->ep_flags, n_flags)) || (st = alloc(ctx, &ctx->counts_all, static_cast<size_t>(N) * E)))
        return st;
    LM_CUDA(ctx, cudaMemset(ctx->ep_flags, 0, n_flags * sizeof(uint32_t)));
    LM_CUDA(ctx, cudaMallocHost(&ctx->host_counts_all, static_cast<size_t>(N) * E * sizeof(int32_t)));
    cudaIpcMemHandle_t mine[3];
    LM_CUDA(ctx, cudaIpcGetMemHandle(&mine[0], ctx->x_perm));
    LM_CUDA(ctx, cudaIpcGetMemHandle(&mine[1], ctx->y_ret));
    LM_CUDA(ctx, cudaIpcGetMemHandle(&mine[2], ctx->ep_flags));
    constexpr size_t hb = sizeof(mine);
    uint8_t* dev = nullptr;
    if ((st = alloc(ctx, &dev, hb * static_cast<size_t>(N + 1))) != LM_OK) return st;
    std::vector<cudaIpcMemHandle_t> all(static_cast<size_t>(3) * N);
    cudaStream_t xs = nullptr;
    LM_CUDA(ctx, cudaStreamCreateWithFlags(&xs, cudaStreamNonBlocking));
    cudaError_t ce = cudaMemcpyAsync(dev, mine, hb, cudaMemcpyHostToDevice, xs);
    ncclResult_t nr = ncclSuccess;
    if (ce == cudaSuccess) {
        nr = nc.GroupStart();
        for (int d = 0; d < N && nr == ncclSuccess; ++d) {
            nr = nc.Send(dev, hb, ncclInt8, d, ctx->comm, xs);
            if (nr == ncclSuccess) nr = nc.Recv(dev + hb * (d + 1), hb, ncclInt8, d, ctx->comm, xs);
        }
        const ncclResult_t ne = nc.GroupEnd();
        if (nr == ncclSuccess) nr = ne;
    }
    if (ce == cudaSuccess && nr == ncclSuccess)
        ce = cudaMemcpyAsync(all.data(), dev + hb, hb * N, cudaMemcpyDeviceToHost, xs);
    const cudaError_t cs = cudaStreamSynchronize(xs);
    cudaStreamDestroy(xs);
    if (nr != ncclSuccess) return fail(ctx, LM_ERR_COMM, std::string("IPC handle exchange: ") + nc.GetErrorString(nr));
    if (ce != cudaSuccess) return cuda_fail(ctx, ce, "IPC handle exchange");
    if (cs != cudaSuccess) return cuda_fail(ctx, cs, "IPC handle exchange");
    ctx->ep_peer_flags.n = N;
    for (int r = 0; r < N; ++r) {
        if (r == me) {
            ctx->ep_peer_xperm[r] = ctx->x_perm;
            ctx->ep_peer_yret[r] = ctx->y_ret;
            ctx->ep_peer_flags.flags[r] = ctx->ep_flags;
            continue;
        }
        void* px = nullptr;
        void* py = nullptr;
        void* pf = nullptr;
        LM_CUDA(ctx, cudaIpcOpenMemHandle(&px, all[3 * r + 0], cudaIpcMemLazyEnablePeerAccess));
        LM_CUDA(ctx, cudaIpcOpenMemHandle(&py, all[3 * r + 1], cudaIpcMemLazyEnablePeerAccess));
        LM_CUDA(ctx, cudaIpcOpenMemHandle(&pf, all[3 * r + 2], cudaIpcMemLazyEnablePeerAccess));
        ctx->ep_peer_xperm[r] = static_cast<uint16_t*>(px);
        ctx->ep_peer_yret[r] = static_cast<uint16_t*>(py);
        ctx->ep_peer_flags.flags[r] = static_cast<uint32_t*>(pf);
        ctx->ep_peer_opened[r] = true;
        LM_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->ep_copy_stream[r], cudaStreamNonBlocking));
        LM_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ep_ev_returned[r], cudaEventDisableTiming));
        for (int k = 0; k < kEpMaxChunks; ++k)
            LM_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ep_ev_pulled[k][r], cudaEventDisableTiming));
    }
    // Every kernel the expert-parallel forward can launch is loaded now, before any
    // flag wait spins (a lazily loaded kernel's first launch could otherwise wait for
    // a spinning wait that waits for the peer's GEMMs, which wait likewise).
    for (cudaError_t (*preload)() : {preload_router_kernels, preload_grouped_gemm_kernels, preload_pair_gemm_kernels,
                                     preload_ops_kernels, preload_ep_peer_kernels, preload_host_io_kernels})
        LM_CUDA(ctx, preload());
    // Handshake (epoch 1): every rank stores into its slot of every peer's flags, waits
    // (bounded) for every peer's store into its own, then reads back through a copy
    // engine what it stored in each peer's buffer -- the three paths every forward uses.
    LM_CUDA(ctx, launch_ep_signal(ctx->ep_peer_flags, me, me, 1u, nullptr));
    for (int r = 0; r < N; ++r)
        if (r != me) LM_CUDA(ctx, launch_ep_wait(ctx->ep_flags, r, 1u, ctx->status, ctx->ep_flags + n_flags - kEpDiagSlots,
                                                 kWaitLimitNs, nullptr));
    LM_CUDA(ctx, cudaDeviceSynchronize());
    int32_t status = 0;
    LM_CUDA(ctx, cudaMemcpy(&status, ctx->status, sizeof(status), cudaMemcpyDeviceToHost));
    if (status != 0) {
        cudaMemset(ctx->status, 0, sizeof(int32_t));
        return fail(ctx, LM_ERR_COMM, "copy-engine exchange set-up: a peer's flag store never arrived (code " +
                                          std::to_string(status) + "); set LITEMIND_B200_EP_COPY=0 to use NCCL");
    }
    for (int r = 0; r < N; ++r) {
        if (r == me) continue;
        uint32_t v = 0;
        LM_CUDA(ctx, cudaMemcpy(&v, ctx->ep_peer_flags.flags[r] + me, sizeof(v), cudaMemcpyDeviceToHost));
        if (v != 1u)
            return fail(ctx, LM_ERR_COMM, "copy-engine exchange set-up: rank " + std::to_string(r) +
                                              "'s flag slot reads " + std::to_string(v) +
                                              " through a copy engine, 1 was stored");
    }
    ctx->ep_copy = true;
    ctx->ep_epoch = 1;
    return LM_OK;
}

lm_status lm_moe_ep_init(lm_moe_ctx* ctx, const void* nccl_unique_id, int32_t rank, int32_t nranks) {
    if (ctx == nullptr || nccl_unique_id == nullptr) return LM_ERR_INVALID_ARGUMENT;
    const lm_moe_config& c = ctx->cfg;
    if (nranks < 1 || rank < 0 || rank >= nranks || c.n_routed_experts % nranks != 0)
        return fail(ctx, LM_ERR_INVALID_ARGUMENT, "need 0 <= rank < nranks and nranks dividing n_routed_experts");
    if (ctx->comm != nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "expert parallelism is already initialised");
    for (const LayerWeights& L : ctx->layers)
        if (L.w13 != nullptr) return fail(ctx, LM_ERR_INVALID_ARGUMENT, "call lm_moe_ep_init before uploading weights");
    // NCCL's copy-engine mode for peer transfers makes NCCL's kernel on the caller's
    // stream wait for copies that NCCL's host proxy thread issues.  When the caller's
    // stream is the legacy default stream, a copy the driver orders behind that stream
    // waits for the very kernel that waits for it; an exchange in this mode once made
    // no progress until its process was killed.  Refused rather than risked.
    if (const char* v = std::getenv("NCCL_P2P_USE_CUDA_MEMCPY"); v != nullptr && std::atoi(v) != 0)
        return fail(ctx, LM_ERR_UNSUPPORTED,
                    "NCCL_P2P_USE_CUDA_MEMCPY is set: the expert-parallel exchange does not support NCCL's "
                    "copy-engine peer transfers (unset it, or set it to 0)");
    lm_status st;
    if ((st = set_device(ctx)) != LM_OK) return st;
    std::string err;
    ctx->nccl = nccl_api(err);
    if (ctx->nccl == nullptr) return fail(ctx, LM_ERR_COMM, err);
    const int El = c.n_routed_experts / nranks;
    const size_t T = c.max_tokens, K = c.num_experts_per_tok, H = c.hidden_size, I = c.moe_intermediate_size;
    // Small batches exchange fixed blocks of ep_cap rows per rank pair (no host round
    // trip): a token sends one rank at most min(k, local experts) rows.
    const size_t fixed_cap = T * std::min(K, static_cast<size_t>(El));
    ctx->ep_cap = static_cast<size_t>(nranks) * fixed_cap <= kEpFixedMaxRows ? static_cast<int>(fixed_cap) : 0;
    // Larger batches plan on the host and move the local experts in chunks, each
    // chunk's rows on an NCCL stream of its own while earlier chunks compute.
    if (const char* v = std::getenv("LITEMIND_B200_EP_CHUNKS")) ctx->ep_chunks = std::atoi(v);
    if (const char* v = std::getenv("LITEMIND_B200_EP_NCCL_CTAS")) ctx->ep_nccl_ctas = std::atoi(v);
    ctx->ep_chunks = ctx->ep_cap > 0 ? 1 : std::max(1, std::min({ctx->ep_chunks, kEpMaxChunks, El}));
    ctx->ep_nccl_ctas = std::max(1, std::min(ctx->ep_nccl_ctas, ctx->sms / 2 - 1));
    ncclUniqueId id;
    std::memcpy(&id, nccl_unique_id, sizeof(id));
    ncclResult_t r;
    if (ctx->ep_chunks > 1 && ctx->nccl->CommInitRankConfig != nullptr) {
        // NCCL's kernels run beside the GEMMs: cap their CTAs to the SMs left free.
        ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
        config.maxCTAs = ctx->ep_nccl_ctas;
        r = ctx->nccl->CommInitRankConfig(&ctx->comm, nranks, id, rank, &config);
    } else {
        r = ctx->nccl->CommInitRank(&ctx->comm, nranks, id, rank);
    }
    if (r != ncclSuccess) {
        ctx->comm = nullptr;
        return fail(ctx, LM_ERR_COMM, std::string("ncclCommInitRank: ") + ctx->nccl->GetErrorString(r));
    }
    ctx->rank = rank;
    ctx->nranks = nranks;
    if (const char* v = std::getenv("LITEMIND_B200_EP_SINGLE")) ctx->ep_single = nranks == 1 && std::atoi(v) != 0;
    ctx->first_expert = rank * El;
    ctx->local_experts = El;
    ctx->n_seg = El + c.n_shared_experts;
    // Receive capacity for the worst case (every rank's every slot on this rank),
    // so no rank can overflow mid-exchange and leave its peers waiting.
    const size_t cap = static_cast<size_t>(nranks) * T * K;
    ctx->routed_cap = static_cast<int>(cap);
    const size_t h_rows = cap + c.n_shared_experts * T;
    // Replace the single-GPU h with one sized for the received rows.
    for (auto it = ctx->allocations.begin(); it != ctx->allocations.end(); ++it)
        if (*it == ctx->h) {
            cudaFree(*it);
            ctx->allocations.erase(it);
            break;
        }
    const size_t back_rows = std::max(T * K, static_cast<size_t>(nranks) * ctx->ep_cap);
    if ((st = alloc(ctx, &ctx->h, h_rows * I)) || (st = alloc(ctx, &ctx->x_recv, cap * H)) ||
        (st = alloc(ctx, &ctx->y_ret, cap * H)) || (st = alloc(ctx, &ctx->y_back, back_rows * H)) ||
        (ctx->ep_cap > 0 && (st = alloc(ctx, &ctx->x_send, static_cast<size_t>(nranks) * ctx->ep_cap * H))) ||
        (st = alloc(ctx, &ctx->recv_counts, static_cast<size_t>(nranks) * El)) ||
        (st = alloc(ctx, &ctx->sched_ep, kEpMaxChunks + 1)) ||
        (st = alloc(ctx, &ctx->x_sorted, cap * H)) || (st = alloc(ctx, &ctx->ep_row_src, cap)))
        return st;
    LM_CUDA(ctx, cudaMallocHost(&ctx->host_sched, (kEpMaxChunks + 1) * sizeof(Schedule)));
    LM_CUDA(ctx, cudaMallocHost(&ctx->host_totals, c.n_routed_experts * sizeof(int32_t)));
    LM_CUDA(ctx, cudaMallocHost(&ctx->host_recv, static_cast<size_t>(nranks) * El * sizeof(int32_t)));
    std::memset(ctx->host_sched, 0, (kEpMaxChunks + 1) * sizeof(Schedule));
    if (ctx->ep_chunks > 1) {
        int lo = 0, hi = 0;
        LM_CUDA(ctx, cudaDeviceGetStreamPriorityRange(&lo, &hi));
        LM_CUDA(ctx, cudaStreamCreateWithPriority(&ctx->ep_stream, cudaStreamNonBlocking, hi));
        LM_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ep_ev_ready, cudaEventDisableTiming));
        LM_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ep_ev_back, cudaEventDisableTiming));
        for (int i = 0; i < ctx->ep_chunks; ++i) {
            LM_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ep_ev_sent[i], cudaEventDisableTiming));
            LM_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ep_ev_done[i], cudaEventDisableTiming));
        }
    }
    // The host-planned exchange moves rows with copy engines out of IPC-mapped peer buffers
    // by default on 2 ranks (where it is measured: 10% faster than NCCL send/recv, whose
    // kernels take SMs from the GEMMs), and with LITEMIND_B200_EP_COPY=1 on up to
    // kEpCopyMaxRanks; otherwise, or with LITEMIND_B200_EP_COPY=0, NCCL send/recv.
    bool want_copy = ctx->ep_cap == 0 && nranks == 2;
    if (const char* v = std::getenv("LITEMIND_B200_EP_COPY"))
        want_copy = ctx->ep_cap == 0 && nranks <= kEpCopyMaxRanks && std::atoi(v) != 0;
    // Every rank must take the same steps in every exchange, and a peer's rows must
    // fit this rank's buffers: compare the settings that decide both, once.
    {
        constexpr int kFields = 9;
        const int32_t mine[kFields] = {c.hidden_size, c.moe_intermediate_size, c.n_routed_experts,
                                       c.n_shared_experts, c.num_experts_per_tok, c.max_tokens,
                                       ctx->ep_cap, ctx->ep_chunks, want_copy ? 1 : 0};
        int32_t* dev = nullptr;
        if ((st = alloc(ctx, &dev, static_cast<size_t>(kFields) * (nranks + 1))) != LM_OK) return st;
        std::vector<int32_t> all(static_cast<size_t>(kFields) * nranks);
        cudaStream_t xs = nullptr;
        LM_CUDA(ctx, cudaStreamCreateWithFlags(&xs, cudaStreamNonBlocking));
        cudaError_t ce = cudaMemcpyAsync(dev, mine, sizeof(mine), cudaMemcpyHostToDevice, xs);
        ncclResult_t nr = ncclSuccess;
        if (ce == cudaSuccess) {
            nr = ctx->nccl->GroupStart();
            for (int d = 0; d < nranks && nr == ncclSuccess; ++d) {
                nr = ctx->nccl->Send(dev, kFields, ncclInt32, d, ctx->comm, xs);
                if (nr == ncclSuccess) nr = ctx->nccl->Recv(dev + kFields * (d + 1), kFields, ncclInt32, d, ctx->comm, xs);
            }
            const ncclResult_t ne = ctx->nccl->GroupEnd();
            if (nr == ncclSuccess) nr = ne;
        }
        if (ce == cudaSuccess && nr == ncclSuccess)
            ce = cudaMemcpyAsync(all.data(), dev + kFields, all.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, xs);
        const cudaError_t cs = cudaStreamSynchronize(xs);
        cudaStreamDestroy(xs);
        if (nr != ncclSuccess) return fail(ctx, LM_ERR_COMM, std::string("settings exchange: ") + ctx->nccl->GetErrorString(nr));
        if (ce != cudaSuccess) return cuda_fail(ctx, ce, "settings exchange");
        if (cs != cudaSuccess) return cuda_fail(ctx, cs, "settings exchange");
        for (int d = 0; d < nranks; ++d)
            if (std::memcmp(all.data() + static_cast<size_t>(kFields) * d, mine, sizeof(mine)) != 0)
                return fail(ctx, LM_ERR_INVALID_ARGUMENT,
                            "expert-parallel settings differ between ranks (shape, max_tokens, "
                            "LITEMIND_B200_EP_CHUNKS or LITEMIND_B200_EP_COPY): rank " + std::to_string(d));
    }
    if (want_copy && (st = ep_copy_setup(ctx)) != LM_OK) return st;
    for (int i = 0; i < 5; ++i) {
        if (!encode_tensor_map_bf16(&ctx->map_xrecv[i], ctx->x_recv, cap, H, kBnChoices[i], 64, err) ||
            !encode_tensor_map_bf16(&ctx->map_xsorted[i], ctx->x_sorted, cap, H, kBnChoices[i], 64, err) ||
            !encode_tensor_map_bf16(&ctx->map_h[i], ctx->h, h_rows, I, kBnChoices[i], 64, err))
            return fail(ctx, LM_ERR_CUDA, err);
    }
    return LM_OK;
}

}  // extern "C"
