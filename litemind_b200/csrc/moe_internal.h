// moe_internal.h -- shared declarations of the MoE path's kernels and context.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>
#include <vector>

#include "litemind_moe.h"

namespace lm {

constexpr int kMaxExperts = 256;          // routed experts supported by the router kernels
constexpr int kMaxShared = 8;             // shared-expert splits (n_shared_experts)
constexpr int kMaxSegments = kMaxExperts + kMaxShared;
constexpr int kMaxTopK = 16;
constexpr int kRouteTile = 32;            // tokens per routing tile (one warp per token)
constexpr int kRouteMidTokens = 256;      // largest batch routed by the single-launch mid-size kernel
constexpr int kRouteTickets = 16;         // [0] route_small's ticket, [1, ...] route_mid's block + final tickets

// Per-call schedule read by the grouped GEMMs: written on the device by the
// routing kernels (one GPU: segment s is local expert s, then the shared splits),
// or on the host from the exchanged counts (expert parallelism: one segment per
// (source rank, local expert), then the shared splits).
struct Schedule {
    int32_t seg_off[kMaxSegments];     // first row of the segment in h (expert-sorted rows)
    int32_t seg_cnt[kMaxSegments];     // rows in the segment
    int32_t tiles1[kMaxSegments + 1];  // exclusive prefix of gate/up tiles
    int32_t tiles2[kMaxSegments + 1];  // exclusive prefix of down tiles
    int32_t seg_weight[kMaxSegments];  // weight slot (local expert, then shared split) of each segment
    int32_t n_seg;                     // segments in this schedule
    int32_t first_expert;              // expert-parallel shard start (0 on one GPU)
};

struct RouterParams {
    int32_t experts;
    int32_t top_k;
    int32_t n_group;
    int32_t topk_group;
    int32_t group_limited;
    int32_t normalize;
    float scale;
};

// When router logits come from the tensor cores, the top-k kernel recomputes a
// token's logits in plain f32 wherever two of its first k+1 ranked probabilities
// are closer than `margin` (x null: logits are already plain f32).
struct RouterFix {
    const uint16_t* x = nullptr;   // [T, hidden] bf16 tokens
    const float* w = nullptr;      // [E, hidden] f32 router
    const float* bias = nullptr;   // [E] or null
    int32_t hidden = 0;
    float margin = 0.0f;
};

// Kernel launchers (router.cu).  All return cudaGetLastError() after launching.
cudaError_t launch_router_logits(const uint16_t* x, const float* x_f32, const float* w, const float* w_t,
                                 const float* bias, float* logits, int tokens, int hidden, int experts,
                                 float* split_ws, size_t split_ws_bytes, cudaStream_t stream, bool pdl);
cudaError_t launch_router_topk(float* logits, int tokens, RouterParams rp, int32_t* topk_idx, float* topk_w,
                               int32_t* tile_counts, cudaStream_t stream, bool pdl, RouterFix fix = RouterFix{});
cudaError_t launch_dispatch_scan(const int32_t* tile_counts, int32_t* tile_base, int32_t* expert_totals,
                                 Schedule* sched, int tokens, int top_k, int experts, int n_shared,
                                 int first_expert, int local_experts, int shared_base, int bn, int mb1,
                                 int mb2, cudaStream_t stream, bool pdl);
// x_perm non-null: also copy each token's row of x to its expert-sorted rows.
cudaError_t launch_place(const int32_t* topk_idx, const float* topk_w, const int32_t* tile_base, int tokens,
                         int hidden, int top_k, int experts, int first_expert, int local_experts, int32_t* row_token,
                         float* row_weight, int32_t* slot_row, float* y_zero, const uint16_t* x, uint16_t* x_perm,
                         cudaStream_t stream, bool pdl);
cudaError_t launch_ep_combine(float* y, const uint16_t* back, const int32_t* slot_row, const float* topk_w, int tokens,
                              int top_k, int hidden, cudaStream_t stream, bool pdl);
// The dense feed-forward's one-segment schedule; also zeroes y_count floats of y_zero
// (16-byte aligned, a multiple of 4) unless it is null.
cudaError_t launch_dense_schedule(Schedule* sched, int tokens, int bn, int mb1, int mb2, float* y_zero,
                                  int64_t y_count, int sms, cudaStream_t stream);
// Expert parallelism: received rows -> expert-major, with row_src[row] = the row's
// index in the receive buffer.  The receive buffer holds local-expert chunks one after
// another, each source-major; a launch sorts chunk [e_lo, e_hi) (the whole [0, El) when
// the exchange is not chunked).  max_group_rows: the largest (source, expert) group in
// the chunk.  src_stride > 0: source r's rows start at r * src_stride (fixed-capacity
// exchange, whole range only).
cudaError_t launch_ep_sort_rows(const uint16_t* x_recv, uint16_t* x_sorted, int32_t* row_src,
                               const int32_t* recv_counts, int nranks, int local_experts, int max_group_rows,
                               int hidden, int src_stride, int e_lo, int e_hi, cudaStream_t stream, bool pdl);
// Fixed-capacity expert parallelism: pack this rank's rows into per-destination
// blocks of `cap` rows (and point slot_row at them), and build the receiver's
// schedule on the device from the received counts.
cudaError_t launch_ep_pack(const uint16_t* x, const int32_t* row_token, const int32_t* expert_totals,
                           int32_t* slot_row, uint16_t* x_send, int tokens, int top_k, int experts,
                           int local_experts, int cap, int hidden, cudaStream_t stream, bool pdl);
cudaError_t launch_ep_schedule(const int32_t* recv_counts, Schedule* sched, int nranks, int local_experts,
                               int n_shared, int tokens, int shared_base, int bn, int mb1, int mb2,
                               cudaStream_t stream, bool pdl);
cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* row_token, int rows, int hidden, uint16_t* x_perm,
                               cudaStream_t stream, bool pdl);
cudaError_t launch_route_small(const uint16_t* x, const float* x_f32, const float* w, const float* bias,
                               float* logits, int tokens, int hidden, RouterParams rp, int32_t* topk_idx,
                               float* topk_w, int32_t* expert_totals, Schedule* sched, int32_t* row_token,
                               float* row_weight, int32_t* slot_row, float* y_zero, unsigned int* ticket,
                               int n_shared, int first_expert, int local_experts, int shared_base, int bn, int mb1,
                               int mb2, cudaStream_t stream, bool pdl);

// kRouteTile < T <= kRouteMidTokens: the same single-launch routing stage (logits,
// top-k, counts, schedule, placement; E <= kMaxExperts), routed per 32-token block.
// tickets: kRouteMidTokens / 32 + 1 zeroed counters (re-armed by the kernel);
// blk_mask: [blocks, E] scratch.
cudaError_t launch_route_mid(const uint16_t* x, const float* x_f32, const float* w, const float* bias,
                             float* logits, int tokens, int hidden, RouterParams rp, int32_t* topk_idx,
                             float* topk_w, int32_t* expert_totals, Schedule* sched, int32_t* row_token,
                             float* row_weight, int32_t* slot_row, float* y_zero, unsigned int* tickets,
                             uint32_t* blk_mask, int n_shared, int first_expert, int local_experts, int shared_base,
                             int bn, int mb1, int mb2, cudaStream_t stream, bool pdl);

// Grouped SwiGLU GEMMs (grouped_gemm.cu).
struct GemmArgs {
    const Schedule* sched;
    const uint16_t* x;         // [T, hidden] bf16 tokens (the shared experts' operand)
    uint16_t* h;               // [rows, inter] bf16 (gate/up output, down input)
    float* y;                  // [T, hidden] f32 (down output, accumulated)
    const int32_t* row_token;  // routed row -> token
    const float* row_weight;   // routed row -> routing weight
    int32_t* status;           // device status word
    int32_t tokens;
    int32_t hidden;
    int32_t inter;
    uint16_t* y_rows;          // when set, routed rows' down outputs are stored here by row, unweighted, bf16
    const int32_t* y_rows_map; // with y_rows: routed row r is stored at row y_rows_map[r] (null: at r)
    int32_t y_rows_cap;        // with y_rows: rows of y_rows and entries of y_rows_map; a row outside is
                               // skipped and reported (kDevBadRow)
    float* logits;             // router kind: [T, experts] f32 output
    const float* bias;         // router kind: per-expert logit bias or null
    int32_t experts;           // router kind: experts (<= 128)
    int32_t n_routed_local;    // segments [0, n_routed_local) are routed experts
    // Split-K ("stream-K") for launches of few tiles: a CTA whose k-block range
    // cuts a gate/up tile stores its partial sums in split_ws slot 2 * cta (its
    // first unit) or 2 * cta + 1 (its last), [BN][128] f32 each, and counts
    // k-blocks in split_ticket[tile] (zero between uses); the CTA that completes
    // the tile sums the slots in CTA order and applies SiLU.  Null split_ws: no
    // split for gate/up.
    float* split_ws;
    int32_t* split_ticket;
    int32_t split_ws_floats;   // capacity of split_ws in floats
    int32_t split_max_waves;   // split when the tiles fill fewer waves of the grid than this (0: never)
};
// The fused decode kernel (decode_fused.cu): the whole layer for T <= 256 tokens in
// one cooperative launch -- routing, dispatch, gate/up, down and the combine.
constexpr int kDecodeMaxTokens = 256;
constexpr int kDecodeMaxRows = 1536;        // tokens x top-k
constexpr int kDecodeDirectTokens = 32;     // direct mode takes at most this many tokens (x itself is every
                                            // expert's token operand); gather mode takes any batch
constexpr int kDecodeColTile = 32;          // token rows per column tile above that (gather mode)
struct DecodeArgs {
    const uint16_t* x;         // [T, hidden] bf16 tokens (GEMM operand; logits too unless x_f32)
    const float* x_f32;        // optional [T, hidden] f32 tokens for the router logits
    const float* router;       // [E, hidden] f32
    const float* bias;         // [E] per-expert logit bias or null
    float* y;                  // [T, hidden] f32
    int32_t zero_y;            // 1: y = MoE(x), 0: y += MoE(x)
    int32_t tokens;
    int32_t hidden;
    int32_t inter;
    int32_t n_shared;
    RouterParams rp;
    int32_t gather;            // 1: routed token rows are gathered into x_perm and tiled 32 at a time
    int32_t weight_evict_first;  // 1: weight tiles load with an L2 evict-first hint (read once)
    float* logits;             // [T, E] (output, also the exchange between CTAs)
    int32_t* topk_idx;         // [T, k] outputs (gather mode: also the exchange between CTAs)
    float* topk_w;
    int32_t* expert_totals;    // [E]
    int32_t* row_token;        // [T * k] expert-sorted row -> token
    float* row_weight;         // [T * k] expert-sorted row -> routing weight
    uint16_t* x_perm;          // gather mode: [T * k, hidden] expert-sorted token rows
    uint16_t* h;               // SwiGLU outputs: routed rows, then n_shared blocks of T rows
    int32_t h_shared_base;     // first h row of the shared experts
    float* split_ws;           // gate/up split-K partials: 2 slots of [BN][128] per CTA
    int32_t* split_ticket;     // per gate/up tile, zero between uses
    unsigned long long* grid_bar;  // [kDecodeCounters] arrival counters: logits, h, x_perm, top-k, and
                                   // CTAs finished (the last CTA to finish zeroes all of them)
    uint32_t grid_extra;           // testing only: arrivals each grid wait expects beyond gridDim.x
    uint64_t wait_limit_ns;        // bound of the grid waits
    int32_t* status;
    unsigned long long* trace;     // optional: kDecodeTraceSlots global-timer stamps per CTA
    // Weights to bring into L2 while the routing runs with HBM otherwise idle: once the
    // router logits are written, each CTA prefetches its share of these two byte ranges
    // (lengths multiples of 4096, 0 = none).
    const uint8_t* prefetch_base[2];
    uint64_t prefetch_len[2];
};
constexpr int kDecodeCounters = 5;
// Phase stamps of the fused decode kernel (profiling only), per CTA:
//  0 start  1 logits written  2 every CTA's logits seen  3 schedule built
//  4 gate/up epilogues done  5 producer saw every h row  6 producer issued
//  everything  7 down epilogues done  8 MMA done  9 top-k written (gather mode)
//  10 logits loaded (direct mode)  11 routed  12 experts scanned
//  13 every CTA's top-k seen  14 rows gathered  15 producer saw every gathered row
constexpr int kDecodeTraceSlots = 16;
// Router logits the fused decode kernel keeps in shared memory in direct mode
// (tokens x experts).
constexpr int kDecodeMaxLogits = 4096;
cudaError_t launch_moe_decode(int bn, const CUtensorMap& w13, const CUtensorMap& w2, const CUtensorMap& x,
                              const CUtensorMap& xperm, const CUtensorMap& h, const DecodeArgs& args, int sms,
                              cudaStream_t stream);

// Expert parallelism exchanges fixed blocks (no host round trip) while
// nranks x rows-per-block stays within this many rows.
constexpr size_t kEpFixedMaxRows = 8192;
// The host-planned exchange moves the local experts in at most this many chunks, so
// that one chunk's rows travel while another chunk's GEMMs run.
constexpr int kEpMaxChunks = 8;

// The copy-engine exchange (ep_peer.cu): ranks of one node pull rows out of IPC-mapped
// peer buffers; readiness is an epoch stored into flag slots of each rank's flag buffer.
constexpr int kEpCopyMaxRanks = 8;
struct EpPeerFlags {
    uint32_t* flags[kEpCopyMaxRanks];  // every rank's flag buffer (this rank's own at [self])
    int32_t n;
};
cudaError_t launch_ep_signal(const EpPeerFlags& peers, int self, int slot, uint32_t epoch, cudaStream_t stream);
cudaError_t launch_ep_wait(const uint32_t* flags, int slot, uint32_t epoch, int32_t* status, uint32_t* diag,
                           uint64_t limit_ns, cudaStream_t stream);
// Kernels load lazily by default (CUDA_MODULE_LOADING=LAZY): a kernel's first launch may
// wait for the kernels already running on the device.  A flag wait that spins until a
// peer's GEMMs finish must therefore never run while a kernel is still to be loaded on
// either side: the copy-engine exchange loads every kernel the expert-parallel forward
// can launch before its first wait (one function per source file).
cudaError_t preload_router_kernels();
cudaError_t preload_grouped_gemm_kernels();
cudaError_t preload_pair_gemm_kernels();
cudaError_t preload_ops_kernels();
cudaError_t preload_ep_peer_kernels();
cudaError_t preload_host_io_kernels();

// lm_moe_forward_host's transfers by SMs over mapped pinned host memory (host_io.cu).
// A buffer qualifies when it is 16-byte aligned and its size a multiple of 16 bytes.
bool host_io_eligible(const void* p, size_t bytes);
// dst0 <- src0 (bytes0) and, when src1 is not null, dst1 <- src1 (bytes1); sources are
// device addresses of mapped host memory.  The next kernel may launch meanwhile.
cudaError_t launch_host_pull(void* dst0, const void* src0_mapped, size_t bytes0, void* dst1,
                             const void* src1_mapped, size_t bytes1, int sms, cudaStream_t stream);
// dst (mapped host memory) <- src (bytes) and *status_host <- *status, after the previous
// kernel in the stream has finished (programmatic dependent launch).
cudaError_t launch_host_push(void* dst_mapped, const void* src, size_t bytes, const int32_t* status,
                             int32_t* status_host_mapped, int sms, cudaStream_t stream);
// A flag buffer: N (rows ready) + kEpMaxChunks * N (outputs ready) slots, then the
// expired wait's record (slot, value seen, epoch wanted).
constexpr int kEpDiagSlots = 4;
inline size_t ep_flag_slots(int nranks) { return static_cast<size_t>(nranks) * (1 + kEpMaxChunks) + kEpDiagSlots; }

// Split-K workspace for gate/up partial tiles (bytes) and its ticket count.
constexpr size_t kSplitWsBytes = size_t(32) << 20;
constexpr int kSplitTickets = 4096;
cudaError_t launch_gemm_gate_up(int bn, const CUtensorMap& w13, const CUtensorMap& xperm, const CUtensorMap& x,
                                const GemmArgs& args, int sms, cudaStream_t stream, bool pdl);
// Router logits on tensor cores: wcat is [128, 3*hidden] bf16 (the f32 router
// split exactly into three bf16 parts, concatenated along K; rows >= experts zero).
cudaError_t launch_gemm_router(int bn, const CUtensorMap& wcat, const CUtensorMap& x, const GemmArgs& args, int sms,
                               cudaStream_t stream, bool pdl);
cudaError_t launch_gemm_down(int bn, const CUtensorMap& w2, const CUtensorMap& hmap, const GemmArgs& args,
                             int sms, cudaStream_t stream, bool pdl);

// The same two GEMMs on CTA pairs (tcgen05 cta_group::2, 256-row weight tiles) for
// prefill-sized token tiles (grouped_gemm_pair.cu).  Token maps have boxes of bn/2 rows.
cudaError_t launch_gemm_gate_up_pair(int bn, const CUtensorMap& w13, const CUtensorMap& xperm_half,
                                     const CUtensorMap& x_half, const GemmArgs& args, int sms, cudaStream_t stream,
                                     bool pdl);
cudaError_t launch_gemm_down_pair(int bn, const CUtensorMap& w2, const CUtensorMap& h_half, const GemmArgs& args,
                                  int sms, cudaStream_t stream, bool pdl);

// gemm:: mirror kernels and row kernels (gemm_ops.cu).
cudaError_t launch_rms_norm_rows(const float* in, float* out_f32, uint16_t* out_bf16, const float* weight,
                                 int rows, int count, float eps, cudaStream_t stream);
cudaError_t launch_add_rows(float* dst, const float* src, int64_t count, cudaStream_t stream);
// Row-major gate/up [inter, hidden] and down [hidden, inter] (device) into the
// tile-major w13 (gate and up rows interleaved) and w2 the grouped GEMMs read.
// inter must be a multiple of 64, hidden of 128.
cudaError_t launch_pack_swiglu(const uint16_t* gate, const uint16_t* up, const uint16_t* down, int inter, int hidden,
                               uint16_t* w13, uint16_t* w2, int sms, cudaStream_t stream);
const std::string& context_free_error();

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device.
// The attribute belongs to the device's context, so it is set once per device
// (`done` is the caller's per-kernel bit set of devices; ordinals >= 64 set it on
// every launch).  Setting it twice from racing threads is harmless.
template <typename Kernel>
cudaError_t set_smem_limit_once(Kernel kernel, int bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t{1} << dev) : 0;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// Host-side TMA descriptor encoding (tensor_map.cpp).
bool encode_tensor_map_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                            uint32_t box_rows, uint32_t box_cols, std::string& error);

}  // namespace lm
