/*
 * litemind_moe.h -- C ABI of the B200 MoE feed-forward path.
 *
 * Drop-in boundary for LiteMind's mixture-of-experts block (ragavanperarasu/LiteMind).
 * The reference runs that block on the CPU, one token at a time, inside
 * DeepSeekRunner::Impl::forward (src/DeepSeekRunner.cpp:264-290) over three
 * interfaces: MoeRouter (include/MoeRouter.hpp:27-55), the gemm:: kernels
 * (include/Gemm.hpp:23-72) and ExpertCache (include/ExpertCache.hpp:29-89).
 * This header exposes the same path for T tokens at once on one B200:
 *
 *   lm_moe_create / lm_moe_upload_layer   load: weights resident in HBM
 *                                         (replaces DeepSeekRunner::Impl::resolve_layer
 *                                          src/DeepSeekRunner.cpp:179-224 and the
 *                                          ExpertCache's SSD paging)
 *   lm_moe_route, lm_moe_select           MoeRouter::select (src/MoeRouter.cpp:54-107)
 *                                         after gemm::matvec_f32 (src/Gemm.cpp:132-137)
 *   lm_moe_forward                        the whole MoE block of src/DeepSeekRunner.cpp:268-288
 *   lm_gemm_*                             the gemm:: kernels of include/Gemm.hpp, on device
 *
 * Conventions
 *  - Plain C: pointers and sizes only.  bf16 tensors are passed as uint16_t bit
 *    patterns; a stream is a cudaStream_t passed as void* (NULL = legacy stream).
 *  - Every entry point returns an lm_status (0 = LM_OK).  No exception crosses the
 *    ABI.  The context keeps a message for the last failure (lm_moe_last_error).
 *  - "device" pointers are CUDA device memory on the context's device; "host"
 *    pointers are ordinary CPU memory.  Calls that take device pointers are
 *    asynchronous on the given stream; lm_moe_sync waits and reports device-side
 *    errors (a kernel that gave up waiting sets a status word instead of hanging).
 *  - One context per device per host thread; calls on one context are not
 *    thread-safe, as MoeRouter is not (include/MoeRouter.hpp:53-54).
 *  - There is no CPU fallback: a missing GPU is an error (LM_ERR_CUDA).
 */
#ifndef LITEMIND_MOE_H
#define LITEMIND_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t lm_status;

#define LM_OK 0
#define LM_ERR_INVALID_ARGUMENT 1 /* bad size, null pointer, unsupported shape */
#define LM_ERR_CUDA 2             /* a CUDA runtime call failed (message has details) */
#define LM_ERR_NOT_LOADED 3       /* layer weights were never uploaded */
#define LM_ERR_TOO_MANY_TOKENS 4  /* T exceeds the context's max_tokens */
#define LM_ERR_DEVICE_TIMEOUT 5   /* a kernel's bounded wait expired; results are invalid */
#define LM_ERR_COMM 6             /* NCCL failure in expert-parallel mode */
#define LM_ERR_UNSUPPORTED 7

#define LM_TOPK_GREEDY 0               /* Config::topk_method "greedy" */
#define LM_TOPK_GROUP_LIMITED_GREEDY 1 /* Config::topk_method "group_limited_greedy" */

/* The Config fields that drive the MoE path (include/Config.hpp:59-71), plus the
 * sizing of what the context keeps resident. */
typedef struct lm_moe_config {
    int32_t hidden_size;           /* 2048 on DeepSeek-V2-Lite */
    int32_t moe_intermediate_size; /* 1408 */
    int32_t n_routed_experts;      /* 64 */
    int32_t n_shared_experts;      /* 2: one shared FFN of width inter * n_shared */
    int32_t num_experts_per_tok;   /* 6 */
    int32_t norm_topk_prob;        /* 0: weights are raw softmax probabilities */
    float routed_scaling_factor;   /* 1.0; applied only when not normalising */
    int32_t topk_method;           /* LM_TOPK_* */
    int32_t n_group;               /* group-limited routing: groups of experts */
    int32_t topk_group;            /* group-limited routing: groups kept */
    float rms_norm_eps;            /* 1e-6, used by lm_moe_block_forward */
    int32_t num_layers;            /* MoE layers held resident */
    int32_t max_tokens;            /* largest T of one call (sizes the workspace) */
} lm_moe_config;

typedef struct lm_moe_ctx lm_moe_ctx;

/* DeepSeek-V2-Lite defaults (include/Config.hpp:43-71), one layer, 16384 tokens. */
void lm_moe_config_default(lm_moe_config* config);

/* Validates the configuration, selects the device and allocates the workspace.
 * Replaces DeepSeekRunner::load's router/expert-cache set-up (src/DeepSeekRunner.cpp:358-362). */
lm_status lm_moe_create(const lm_moe_config* config, int device, lm_moe_ctx** out);
lm_status lm_moe_destroy(lm_moe_ctx* ctx);

/* Message for the last failing call on this context ("" when none). */
const char* lm_moe_last_error(const lm_moe_ctx* ctx);
const char* lm_status_string(lm_status status);

/*
 * Uploads one MoE layer from host memory, in the reference's safetensors layouts
 * (src/DeepSeekRunner.cpp:157-222):
 *   router      [E, hidden] f32   (mlp.gate.weight, widened as read_float32 does)
 *   gate, up    [E, inter, hidden] bf16     down [E, hidden, inter] bf16
 *   shared_gate, shared_up [S, hidden] bf16 shared_down [hidden, S] bf16,  S = inter * n_shared
 *   norm_weight [hidden] f32 or NULL (post_attention_layernorm, for lm_moe_block_forward)
 * The host arrays are read once; the context owns the device copies.
 */
lm_status lm_moe_upload_layer(lm_moe_ctx* ctx, int32_t layer, const float* router,
                              const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                              const uint16_t* shared_gate, const uint16_t* shared_up,
                              const uint16_t* shared_down, const float* norm_weight);

/*
 * The HBM expert loader: uploads one mixture-of-experts layer straight from
 * SafeTensors checkpoint shards (the format the reference reads with
 * SafeTensor::open, src/SafeTensor.cpp:87-152), with the tensor names of
 * DeepSeekRunner::Impl::resolve_layer (src/DeepSeekRunner.cpp:157-224):
 *   model.layers.{L}.mlp.gate.weight                     [E, H]  BF16, F16 or F32
 *   model.layers.{L}.post_attention_layernorm.weight     [H]     BF16, F16 or F32
 *   model.layers.{L}.mlp.experts.{e}.{gate,up}_proj.weight [I, H] BF16
 *   model.layers.{L}.mlp.experts.{e}.down_proj.weight    [H, I]  BF16
 *   model.layers.{L}.mlp.shared_experts.{gate,up}_proj.weight [n_shared * I, H] BF16
 *   model.layers.{L}.mlp.shared_experts.down_proj.weight [H, n_shared * I] BF16
 * `layer` is this context's layer slot, `checkpoint_layer` the L in the names.
 * Tensors may be spread over the shards in any way; each shard is memory-mapped and
 * only the tensors this device holds are read (under expert parallelism, its own
 * experts).  Shape and dtype mismatches fail with the reference's messages
 * (WeightStore::require, src/WeightStore.cpp:119-140) in lm_moe_last_error.
 */
lm_status lm_moe_load_safetensors(lm_moe_ctx* ctx, int32_t layer, int32_t checkpoint_layer,
                                  const char* const* shard_paths, int32_t n_shards);

/*
 * Header lookup of one tensor in one SafeTensors shard, without a GPU: dtype
 * (LM_DTYPE_*), rank, up to LM_SAFETENSORS_MAX_DIMS dimensions, file-absolute
 * payload offset and size.  Returns LM_ERR_INVALID_ARGUMENT for a malformed shard
 * and LM_ERR_NOT_LOADED when the name is absent, with the reason in `error`
 * (truncated to error_len bytes; may be null).  No reference counterpart as a C
 * entry: it exposes SafeTensor::find (src/SafeTensor.cpp:154-157) to tests and tools.
 */
#define LM_DTYPE_UNKNOWN 0
#define LM_DTYPE_BF16 1
#define LM_DTYPE_F16 2
#define LM_DTYPE_F32 3
#define LM_DTYPE_OTHER 4
#define LM_SAFETENSORS_MAX_DIMS 8
lm_status lm_safetensors_info(const char* path, const char* name, int32_t* dtype, int32_t* ndim, int64_t* shape,
                              uint64_t* offset, uint64_t* nbytes, char* error, int32_t error_len);

/*
 * Dense feed-forward layers (DeepSeek-V2-Lite's first layer, intermediate 10944:
 * src/DeepSeekRunner.cpp:270-271, include/Config.hpp:59) on the same grouped GEMM
 * kernels, as one segment of every token with weight 1.  Dense layers have their
 * own index space, 0.. per context.  gate/up [inter, hidden], down [hidden, inter]
 * bf16; inter a multiple of 64; norm_weight [hidden] f32 or NULL (ones).
 * lm_ffn_forward: y (f32 [T, hidden]) = FFN(x) (or += with accumulate != 0);
 * lm_ffn_block_forward: hidden += FFN(rms_norm(hidden)).  lm_ffn_load_safetensors
 * reads model.layers.{L}.mlp.{gate,up,down}_proj.weight and
 * post_attention_layernorm.weight from SafeTensors shards.
 */
lm_status lm_ffn_upload(lm_moe_ctx* ctx, int32_t layer, int32_t intermediate, const uint16_t* gate, const uint16_t* up,
                        const uint16_t* down, const float* norm_weight);
lm_status lm_ffn_load_safetensors(lm_moe_ctx* ctx, int32_t layer, int32_t checkpoint_layer, int32_t intermediate,
                                  const char* const* shard_paths, int32_t n_shards);
lm_status lm_ffn_forward(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, int32_t tokens, float* y,
                         int32_t accumulate, void* stream);
lm_status lm_ffn_block_forward(lm_moe_ctx* ctx, int32_t layer, float* hidden, int32_t tokens, void* stream);

/* Uploads one routed expert (the unit ExpertCache::touch streams,
 * src/ExpertCache.cpp:9-47): gate, up [inter, hidden], down [hidden, inter]. */
lm_status lm_moe_upload_expert(lm_moe_ctx* ctx, int32_t layer, int32_t expert,
                               const uint16_t* gate, const uint16_t* up, const uint16_t* down);

/*
 * Router only: logits = router . x (+ bias) and MoeRouter::select per token.
 *   x           device bf16 [T, hidden]
 *   logit_bias  device f32 [E] or NULL (added to every token's logits before the softmax)
 *   topk_idx    device int32 [T, k]   topk_w device f32 [T, k]  (descending weight)
 *   logits      device f32 [T, E] or NULL (after the bias)
 */
lm_status lm_moe_route(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, int32_t tokens,
                       const float* logit_bias, int32_t* topk_idx, float* topk_w, float* logits,
                       void* stream);

/* MoeRouter::select on caller-provided logits (device f32 [T, E]). */
lm_status lm_moe_select(lm_moe_ctx* ctx, const float* logits, int32_t tokens, int32_t* topk_idx,
                        float* topk_w, void* stream);

/*
 * The MoE block for T tokens: route, dispatch, grouped SwiGLU experts, weighted
 * combine with the shared experts (weight 1.0).
 *   x       device bf16 [T, hidden]
 *   y       device f32 [T, hidden]; overwritten, or added to when accumulate != 0
 *           (the reference accumulates into a zeroed buffer, src/DeepSeekRunner.cpp:268)
 */
lm_status lm_moe_forward(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x, int32_t tokens,
                         const float* logit_bias, float* y, int32_t accumulate, void* stream);

/* lm_moe_forward from host memory: copies x (and the bias) in, runs, copies y out,
 * and waits.  The end-to-end form of the call the reference makes per token.
 * Page-locked buffers (cudaHostAlloc, cudaMallocHost, cudaHostRegister) that start on a
 * 16-byte boundary, with sizes a multiple of 16 bytes, move by kernel loads and stores over
 * mapped memory, which saves each copy-engine transfer's fixed cost; others are copied with
 * cudaMemcpyAsync.  The result is the same either way. */
lm_status lm_moe_forward_host(lm_moe_ctx* ctx, int32_t layer, const uint16_t* x_host,
                              int32_t tokens, const float* logit_bias_host, float* y_host);

/*
 * One decoder feed-forward sub-layer, as src/DeepSeekRunner.cpp:264-290 runs it:
 * normalised = rms_norm(hidden, post_attention_layernorm); hidden += moe(normalised).
 *   hidden  device f32 [T, hidden], updated in place.
 * The router sees the f32 normalised activations; the experts see them rounded to bf16.
 */
lm_status lm_moe_block_forward(lm_moe_ctx* ctx, int32_t layer, float* hidden, int32_t tokens,
                               void* stream);

/* Waits for the stream and reports a device-side timeout recorded since the last
 * call (then clears it and re-arms the kernels' counters, so the context stays usable). */
lm_status lm_moe_sync(lm_moe_ctx* ctx, void* stream);

/*
 * Testing hooks for the failure-detection path; production code leaves them at 0.
 *   LM_DEBUG_GRID_EXTRA     arrivals the fused decode kernel's grid-wide waits expect
 *                           beyond its own grid (at most 1024).  Nothing provides them,
 *                           so the waits run out: the kernel records a status code and
 *                           returns, and lm_moe_sync / lm_moe_forward_host report
 *                           LM_ERR_DEVICE_TIMEOUT.  0 = off.
 *   LM_DEBUG_WAIT_LIMIT_NS  bound of those grid-wide waits in ns (0 = the 2 s default,
 *                           which is also the maximum).
 * No GPU fault is involved: the kernel only stops waiting.
 */
enum { LM_DEBUG_GRID_EXTRA = 1, LM_DEBUG_WAIT_LIMIT_NS = 2 };
lm_status lm_moe_debug_set(lm_moe_ctx* ctx, int32_t knob, int64_t value);

/* Tokens routed to each expert by the last route/forward: the per-expert token
 * histogram, written to host int32 counts[0 .. E-1].  `capacity` is the number of
 * int32 slots at `counts`; a capacity below the context's n_routed_experts is
 * refused with LM_ERR_INVALID_ARGUMENT and nothing is written.  Waits for the device. */
lm_status lm_moe_expert_counts(lm_moe_ctx* ctx, int32_t* counts, int32_t capacity);

/* Bytes of weights resident on the device, and bytes uploaded so far. */
lm_status lm_moe_memory(const lm_moe_ctx* ctx, uint64_t* resident_bytes, uint64_t* uploaded_bytes);

/*
 * Profiling hook.  While enabled, each forward records a CUDA event after every
 * launch of its sequence, waits for the last one and adds each launch's device
 * time to a per-slot total: slot 1 routing (the fused kernel for T <= 32, else the
 * router logits), 2 router top-k, 3 dispatch scan, 4 placement, 0 the copy of
 * token rows into expert order, 5 gate/up GEMM, 6 down GEMM, 7 expert-parallel
 * exchange, 8 the fused single-launch decode layer (T <= 32 on one GPU).  A dense
 * feed-forward (lm_ffn_forward) records its schedule in slot 3 and its GEMMs in 5 / 6.
 * lm_moe_profile_read copies LM_PROFILE_SLOTS totals (ms) and launch
 * counts to host memory and, when reset != 0, clears them.  No counterpart in the
 * reference, which has no device launches to time.
 */
#define LM_PROFILE_SLOTS 9
lm_status lm_moe_profile_enable(lm_moe_ctx* ctx, int32_t enable);
lm_status lm_moe_profile_read(lm_moe_ctx* ctx, double* total_ms, int64_t* launches, int32_t reset);
/* While profiling, the fused decode kernel (T <= 32 on one GPU) stamps each of its
 * CTAs' phases with the device's global timer (ns): LM_DECODE_TRACE_SLOTS values
 * per CTA (0 start, 1 logits written, 2 every CTA's logits seen, 10 logits in
 * shared memory, 11 every token routed, 12 active experts compacted, 3 schedule
 * built, 4 gate/up epilogues done, 5 producer saw every h row, 6 producer done,
 * 7 down epilogues done, 8 MMA done; 9 and 13-15 unused; 0 = not reached).  Copies the last
 * launch's stamps for up to `ctas` CTAs and sets *ctas_out to the number of CTAs it
 * ran with (0 if none was traced). */
#define LM_DECODE_TRACE_SLOTS 16
lm_status lm_moe_profile_trace(lm_moe_ctx* ctx, uint64_t* stamps, int32_t ctas, int32_t* ctas_out);
/* While profiling, the chunked expert-parallel exchange (C chunks, see
 * lm_moe_ep_chunk_plan) times each of its steps on the device from the moment its
 * rows start to leave.  Copies the last such forward's 4 C + 2 times (ms) -- C ends
 * of the chunks' dispatches (exchange stream), the end of the shared experts' GEMMs,
 * C starts of the chunks' GEMMs (their rows in), C ends of the chunks' GEMMs, C ends
 * of the chunks' returns (exchange stream), the end of the combine -- up to
 * `capacity` values, and sets *chunks_out to C (0 when no chunked forward was
 * profiled). */
#define LM_EP_TIMELINE_MAX 40
lm_status lm_moe_profile_ep_timeline(lm_moe_ctx* ctx, float* ms, int32_t capacity, int32_t* chunks_out);

/*
 * Expert parallelism over NCCL (NVLink within a node).  Every rank creates its
 * context with the same config, then calls this with the same 128-byte
 * ncclUniqueId, before uploading any weights.  Rank r then keeps routed experts
 * [r*E/N, (r+1)*E/N) (upload_layer still takes the full arrays and uploads the
 * rank's shard plus the shared experts), and lm_moe_forward -- called by every rank
 * with its own T tokens, T <= max_tokens, possibly 0 -- routes them over all
 * experts, exchanges per-expert row counts, sends the rows to the experts' ranks,
 * runs the local experts, returns their outputs and combines them with the
 * routing weights and the shared experts.  Contexts whose nranks x max_tokens x
 * min(k, E/N) stays within 8192 rows exchange fixed blocks of rows and plan on the
 * device (no host wait); larger ones wait once on the host for the counts and move
 * the rows in chunks of local experts overlapped with the GEMMs
 * (lm_moe_ep_chunk_plan).  The ranks compare their configs here (one small NCCL
 * exchange) and all fail with LM_ERR_INVALID_ARGUMENT when any differs.  NCCL is
 * loaded at run time (libnccl.so.2).  NCCL's copy-engine peer transfers
 * (NCCL_P2P_USE_CUDA_MEMCPY set to non-zero) are refused with LM_ERR_UNSUPPORTED
 * before NCCL is touched.  A peer that stops taking part (a rank that failed between
 * forwards) never leaves the others waiting for ever: lm_moe_forward's wait for the row
 * counts, lm_moe_sync and lm_moe_forward_host give up after 30 s (the
 * LM_DEBUG_WAIT_LIMIT_NS knob shortens it), abort the communicator and return
 * LM_ERR_COMM; every later forward on that context returns LM_ERR_COMM at once, and
 * the context can only be destroyed.
 */
lm_status lm_moe_ep_init(lm_moe_ctx* ctx, const void* nccl_unique_id, int32_t rank,
                         int32_t nranks);

/*
 * The exchange plan of one expert-parallel forward, computed on the host from
 * row counts: this rank sends send_count[d] rows to rank d starting at row
 * send_offset[d] of its expert-sorted send buffer, and receives recv_count[s] rows
 * from rank s at row recv_offset[s] of its receive buffer.
 *   send_expert_counts  [E]: this rank's rows per expert (all experts)
 *   recv_expert_counts  [nranks, E/nranks]: rows each rank sends to this rank's experts
 * lm_moe_forward's host-planned exchange moves exactly these rows (in chunks, see
 * below); the plan is exported so callers can size buffers and so it can be checked
 * across ranks without a GPU.
 */
#define LM_EP_MAX_RANKS 64
typedef struct lm_ep_plan {
    int32_t send_count[LM_EP_MAX_RANKS];
    int32_t send_offset[LM_EP_MAX_RANKS];
    int32_t recv_count[LM_EP_MAX_RANKS];
    int32_t recv_offset[LM_EP_MAX_RANKS];
    int32_t n_send;
    int32_t n_recv;
} lm_ep_plan;
lm_status lm_moe_ep_plan(int32_t nranks, int32_t experts, const int32_t* send_expert_counts,
                         const int32_t* recv_expert_counts, lm_ep_plan* plan);

/*
 * The same exchange in `chunks` pieces: chunk c carries the rows of this rank's
 * local experts [c El / chunks, (c+1) El / chunks) (El = experts / nranks), so one
 * chunk's rows can travel while an earlier chunk's experts compute.  Chunk c's plan:
 * send_count[d] rows to rank d from send_offset[d] of the expert-sorted send buffer
 * (rank d's chunk-c experts are contiguous there); recv_count[s] rows from rank s at
 * recv_offset[s] of the receive buffer, which holds all of chunk 0 (by source rank),
 * then all of chunk 1, and so on.  n_send / n_recv are the chunk's totals.  The
 * outputs go back with the offsets reversed.  chunks = 1 is lm_moe_ep_plan.
 * lm_moe_forward uses LITEMIND_B200_EP_CHUNKS chunks (default 2, at most 8 and at
 * most El) when the context exchanges by host plan, with NCCL capped to
 * LITEMIND_B200_EP_NCCL_CTAS CTAs (default 32) and the GEMMs leaving it that many
 * SMs; every rank must use the same (lm_moe_ep_init checks).  Testing and profiling
 * only: with LITEMIND_B200_EP_SINGLE=1 at lm_moe_ep_init, a one-rank context runs this
 * exchange path (NCCL sending to itself) instead of the local path.
 */
lm_status lm_moe_ep_chunk_plan(int32_t nranks, int32_t experts, int32_t chunks, int32_t chunk,
                               const int32_t* send_expert_counts, const int32_t* recv_expert_counts,
                               lm_ep_plan* plan);

/* A fresh 128-byte ncclUniqueId for lm_moe_ep_init (rank 0 makes it; the caller
 * shares it with the other ranks by any host channel). */
lm_status lm_moe_ep_unique_id(void* nccl_unique_id_out);

/*
 * Routing that allocates nothing, for callers that cannot allocate device memory:
 * code inside a CUDA graph capture (cudaMalloc cannot be captured), plugins whose
 * host application owns all device memory through its own pool, and paths that
 * must never trigger an allocation's implicit synchronisation.  It has no
 * counterpart in the reference, which routes on the CPU.
 *
 * Same results as lm_moe_route with greedy top-k (normalise or scale as given),
 * but without a context: the caller passes the router weights (device f32 [E, H],
 * the layout of lm_moe_upload_layer's `router`), x (device bf16 [T, H]), the
 * optional bias (device f32 [E]) and the outputs (device int32 / f32 [T, k]).
 * Its only scratch is a fixed 1 MiB device array inside the library (held by every
 * GPU that loads it until the process exits), so: T <= 2047 and T * E <= 262144,
 * else LM_ERR_TOO_MANY_TOKENS.  The first call on a device looks up that array's
 * address (cudaGetSymbolAddress); make that first call before any stream capture.
 * After a reset of the device (cudaDeviceReset) the next call looks it up again,
 * so that call too should come before any capture.
 * All calls share the array: calls whose kernels overlap on the GPU (different
 * streams without ordering) race on it and give wrong results.  Errors are
 * status codes only; lm_moe_last_error does not describe them.
 */
lm_status lm_moe_route_static(const float* router, const uint16_t* x, int32_t tokens, int32_t hidden,
                              int32_t experts, int32_t top_k, int32_t norm_topk_prob, float routed_scaling_factor,
                              const float* logit_bias, int32_t* topk_idx, float* topk_w, void* stream);

/* ── gemm:: kernels on device memory (include/Gemm.hpp:23-72) ──────────────── */

/* gemm::kernel_description (src/Gemm.cpp:108-123): which kernels this build runs, for
 * logs.  A static string; needs no GPU. */
const char* lm_kernel_description(void);

/* gemm::matvec_bf16 (src/Gemm.cpp:139-154): out = W x, W [rows, cols] bf16. */
lm_status lm_gemm_matvec_bf16(const uint16_t* weights, const float* input, float* out,
                              int64_t rows, int64_t cols, void* stream);
/* gemm::matvec_bf16_accumulate (src/Gemm.cpp:156-175): out += scale * W x. */
lm_status lm_gemm_matvec_bf16_accumulate(const uint16_t* weights, const float* input, float* out,
                                         int64_t rows, int64_t cols, float scale, void* stream);
/* gemm::matvec_f32 (src/Gemm.cpp:132-137). */
lm_status lm_gemm_matvec_f32(const float* weights, const float* input, float* out, int64_t rows,
                             int64_t cols, void* stream);
/* gemm::softmax (src/Gemm.cpp:209-223), in place, over `count` values of each of `rows` rows. */
lm_status lm_gemm_softmax(float* values, int64_t rows, int64_t count, void* stream);
/* gemm::silu_multiply (src/Gemm.cpp:225-231). */
lm_status lm_gemm_silu_multiply(const float* gate, const float* up, float* destination,
                                int64_t count, void* stream);
/* gemm::rms_norm (src/Gemm.cpp:197-207), in place over each of `rows` rows. */
lm_status lm_gemm_rms_norm(float* values, const float* weight, int64_t rows, int64_t count,
                           float epsilon, void* stream);
/* gemm::axpy (src/Gemm.cpp:191-195): destination += scale * source. */
lm_status lm_gemm_axpy(float scale, const float* source, float* destination, int64_t count,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LITEMIND_MOE_H */
