// decode_fused.cu -- the whole MoE layer for decode-sized batches (T <= 256 tokens)
// in one persistent, cooperative launch.
//
// At these sizes the layer is a stream of expert weights (about 139 MB at T=1,
// 1.1 GB from T=32 on) and every separate launch costs a ramp-up and a tail in
// which HBM idles.  Here one CTA per SM runs the layer's steps back to back, each
// step split evenly over all CTAs ("stream-K": a list's k-block iterations cut into
// gridDim.x equal ranges), with grid-wide arrival counters between them.
//
// Routing (src/Gemm.cpp:132-137, MoeRouter::select src/MoeRouter.cpp:54-107) comes
// first, before any weight is streamed through the MMA: under a saturated weight
// stream every global access of the routing waits microseconds in the memory queues.
// (In direct mode the producer only brings the shared experts' gate/up weights into
// L2 once the router logits are read.)  Two modes:
//
//   direct  (small T)  router dot products spread over every warp of the grid;
//           after counter 0 every CTA reads all T x E logits into shared memory and
//           recomputes the whole routing identically (top-k, histogram, row order).
//           Every expert's token operand is x itself (all T tokens as the MMA's N):
//           the tensor cores are idle at these sizes anyway, and it spares a gather
//           and a grid-wide wait; the epilogue keeps the expert's own tokens.
//   gather  (larger T) router logits as (expert, 8 tokens) warp tasks; after counter
//           0 each token's top-k is computed once in the grid (one warp per token)
//           and published; after counter 3 every CTA reads all T x k selections and
//           builds the histogram and row order; each CTA then copies its share of
//           token rows into expert order (x_perm) and arrives on counter 2.  Every
//           expert's rows are tiled 32 at a time (column tiles); the shared
//           experts' tiles read x directly, so they stream while the rows gather.
//
// Then two lists of tiles, each spread over all CTAs:
//   gate/up   shared experts' tiles, then the routed experts'
//   down      routed experts' tiles, then the shared experts'.  Their h tiles wait for
//             counter 1 (every CTA finished gate/up); their weight tiles are loaded
//             before that, so the switch costs no HBM time.
//
// Epilogues are the grouped GEMMs' (grouped_gemm.cu): h = silu(gate) * up in bf16
// for gate/up (src/DeepSeekRunner.cpp:228-240), and the routing-weighted atomic add
// into y for down (the weighted combine and un-permute of :273-288).  A gate/up tile
// whose k-blocks several CTAs share is completed by the one holding its first
// k-blocks, which adds the others' partial sums (split workspace, fixed CTA order) to
// its own; a shared down tile simply adds every part into y.
//
// Warp roles as in the grouped GEMMs: warp 0 TMA producer, warp 1 tcgen05.mma
// issuer, warps 2-9 routing and then the epilogue.  The routing's scratch lives in
// the pipeline ring, which no TMA load touches before the schedule exists.  Every
// wait -- mbarriers and the grid counters -- is bounded; an expired wait records a
// status code and the CTA winds down, and CTAs that see a recorded status stop
// waiting too.
#include "moe_internal.h"
#include "ptx.cuh"
#include "route_device.cuh"

#include <cuda_bf16.h>

namespace lm {
namespace {

constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kBlockM = 128;
constexpr int kBlockK = 64;
constexpr int kATile = kBlockM * kBlockK * 2;
constexpr int kMaskWords = kDecodeMaxTokens / 32;  // token bit set per expert
constexpr int kMaxGroups = kMaxExperts + kMaxShared;
constexpr int kDynBudget = 206 * 1024;  // leaves room for the static shared arrays below (227 KB in all)
constexpr int kMaxPending = 16;
constexpr int kLogitTokens = 8;  // gather mode: tokens per router-logit warp task

// Grid counters (DecodeArgs::grid_bar).
constexpr int kCtrLogits = 0;
constexpr int kCtrH = 1;
constexpr int kCtrXperm = 2;
constexpr int kCtrTopk = 3;
constexpr int kCtrExit = 4;
static_assert(kCtrExit + 1 == kDecodeCounters, "counter count");

template <int BN>
struct DCfg {
    static constexpr int kBTile = BN * kBlockK * 2;
    static constexpr int kStage = kATile + kBTile;
    static constexpr int kStaging = BN * 64 * 2;
    static constexpr int kBar = 1024;
    static constexpr int kStagesFit = (kDynBudget - 1024 - kStaging - kBar) / kStage;
    static constexpr int kStages = kStagesFit > 12 ? 12 : kStagesFit;
    static constexpr int kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;
    static constexpr int kSmem = 1024 + kStages * kStage + kStaging + kBar;
    static_assert(BN == 16 || BN == 32, "decode token tiles are 16 or 32 wide");
    static_assert(kStages >= 4 && kStages <= kMaxPending, "pipeline depth");
    static_assert(kSmem <= kDynBudget, "shared memory");
};

// Routing scratch, placed at the start of the pipeline ring (unused until the
// schedule is built).
struct RouteScratch {
    float logits[kDecodeMaxLogits];           // direct mode: [t * E + e]
    int idx[kDecodeMaxRows];                  // top-k experts, [t * K + k]
    float w[kDecodeMaxRows];                  // top-k weights
    uint32_t emask[kMaxExperts][kMaskWords];  // tokens of each expert (bit t)
    float probs[kEpiWarps][kMaxExperts];      // group-limited routing scratch
};
static_assert(sizeof(RouteScratch) <= 4 * kATile, "routing scratch fits in the first pipeline stages");

__device__ __forceinline__ float silu_times(float g, float u) {
    // src/Gemm.cpp:225-231, with fast exp and divide: the result is rounded to bf16.
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// One list's stream-K walk: this CTA's equal share of the list's k-block iterations.
struct ListWalk {
    int64_t it, end;
    int num_kb;
    __device__ void init(int tiles, int num_kb_) {
        num_kb = num_kb_;
        const int64_t iters = static_cast<int64_t>(tiles) * num_kb_;
        it = iters * blockIdx.x / gridDim.x;
        end = iters * (blockIdx.x + 1) / gridDim.x;
    }
    __device__ bool next(int& t, int& kb0, int& kb1) {
        if (it >= end) return false;
        t = static_cast<int>(it / num_kb);
        kb0 = static_cast<int>(it - static_cast<int64_t>(t) * num_kb);
        const int64_t left = end - it;
        kb1 = left < num_kb - kb0 ? kb0 + static_cast<int>(left) : num_kb;
        it += kb1 - kb0;
        return true;
    }
};

// Token operand of a unit.
constexpr int kBx = 0;      // x (direct mode: all T tokens; gather mode: a shared expert's column tile)
constexpr int kBxperm = 1;  // x_perm rows (gather mode, routed gate/up)
constexpr int kBh = 2;      // h rows (down)

// The decoded work unit: which weights, which token rows, where its outputs go.
struct UnitInfo {
    int a_row;      // tile-major weight row of k-block 0 (the A coordinate is a_row + kb * 128)
    int bmap;       // kBx, kBxperm or kBh
    int b_row;      // first row of the token tile in its B tensor
    int hrow0;      // h row of output column 0 (gate/up: row written; down: row read)
    int nout;       // valid output columns
    int tok0;       // shared experts: token of column 0
    int mb;         // 128-row weight block within the expert
    bool routed;    // routed expert (rows map to tokens through the row maps) or shared
    bool by_token;  // direct-mode routed gate/up: column c is token c, output row j takes column row_token[j]
};

template <int BN, int EPL>
__global__ void __launch_bounds__(kThreads, 1)
    moe_decode_kernel(const __grid_constant__ CUtensorMap map_w13, const __grid_constant__ CUtensorMap map_w2,
                      const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_xperm,
                      const __grid_constant__ CUtensorMap map_h, const __grid_constant__ DecodeArgs args) {
    using C = DCfg<BN>;
    constexpr int S = C::kStages;
    constexpr uint32_t kIdesc = umma_idesc_bf16(kBlockM, BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ int s_row_token[kDecodeMaxRows];   // expert-sorted row -> token
    __shared__ float s_row_w[kDecodeMaxRows];     // expert-sorted row -> routing weight
    __shared__ int s_cnt[kMaxExperts];            // rows per expert
    __shared__ int s_eoff[kMaxExperts];           // first expert-sorted row of each expert
    __shared__ int s_seg_e[kMaxExperts];          // active (non-empty) experts, in expert order
    __shared__ int s_tp[2][kMaxGroups + 1];       // per list: first tile of each group (prefix)
    __shared__ RouterParams s_rp;  // read once at entry: a late read of a kernel parameter can miss
                                   // the constant cache and wait behind the weight stream
    __shared__ int s_n_act;
    __shared__ int s_go[2];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + S * kATile;
    uint8_t* staging = smem_b + S * C::kBTile;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C::kStaging);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tmem_full = bars + 2 * S;
    uint64_t* tmem_empty = bars + 2 * S + 2;
    uint64_t* sched_ready = bars + 2 * S + 4;
    uint64_t* drain_bar = bars + 2 * S + 5;
    uint64_t* logit_bar = bars + 2 * S + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 7);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    RouteScratch& rs = *reinterpret_cast<RouteScratch*>(smem_a);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int T = args.tokens;
    const int H = args.hidden;
    const int I = args.inter;
    const int E = args.rp.experts;
    const int K = args.rp.top_k;
    const int G = gridDim.x;
    const bool gather = args.gather != 0;
    const unsigned long long target = static_cast<unsigned long long>(G) + args.grid_extra;
    const int mb1 = 2 * I / kBlockM;  // 128-row blocks of interleaved gate/up rows
    const int nkb1 = H / kBlockK;
    const int mb2 = H / kBlockM;
    const int nkb2 = I / kBlockK;
    const int nsh = args.n_shared;
    // Gather mode with bf16 activations: a CTA's router-logit tasks are kEpiWarps
    // consecutive experts (its expert block, one per warp) against one group of
    // kLogitTokens tokens per round -- groups q, q + cta_per_eb, ... -- so their inputs
    // are contiguous ranges: the block's router rows once and each round's token rows.
    // The producer brings them all into the ring from stage 4 on (free until the schedule
    // exists; the routing scratch holds stages 0-3; the token stages follow the weight
    // stages) with bulk copies: one round trip, where loads from global memory would
    // take one per step of the dot products.
    const int ntg = (T + kLogitTokens - 1) / kLogitTokens;
    const int n_eb = E / kEpiWarps;                        // expert blocks
    const int cta_per_eb = n_eb > 0 ? G / n_eb : 0;        // CTAs sharing an expert block
    const int rounds = cta_per_eb > 0 ? (ntg + cta_per_eb - 1) / cta_per_eb : 0;
    const bool staged = gather && args.x_f32 == nullptr && E % kEpiWarps == 0 && cta_per_eb > 0 && rounds <= 2 &&
                        static_cast<int64_t>(kEpiWarps) * H * 4 + static_cast<int64_t>(rounds) * kLogitTokens * H * 2 <=
                            static_cast<int64_t>(S - 4) * kATile + static_cast<int64_t>(S) * C::kBTile;
    const int my_eb = n_eb > 0 ? static_cast<int>(blockIdx.x) % n_eb : 0;  // this CTA's expert block
    const int my_q = n_eb > 0 ? static_cast<int>(blockIdx.x) / n_eb : 0;   // and its first token group
    const bool has_tasks = staged && my_q < cta_per_eb && my_q < ntg;
    float* st_router = reinterpret_cast<float*>(smem_a + 4 * kATile);
    // Round r's token rows: st_x + r * kLogitTokens * H.
    uint16_t* st_x = reinterpret_cast<uint16_t*>(smem_a + 4 * kATile + static_cast<size_t>(kEpiWarps) * H * 4);

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], kEpiWarps);
        }
        mbar_init(sched_ready, 1);
        mbar_init(drain_bar, 1);
        mbar_init(logit_bar, 1);
        s_rp = args.rp;
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&map_w13);
        tma_prefetch_desc(&map_w2);
        tma_prefetch_desc(&map_x);
        tma_prefetch_desc(&map_xperm);
        tma_prefetch_desc(&map_h);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    // Everything above overlaps the previous kernel's tail (programmatic launch);
    // x, y and the workspaces are touched only after it has finished.
    pdl_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    auto stamp = [&](int k) {
        if (args.trace != nullptr) args.trace[blockIdx.x * kDecodeTraceSlots + k] = global_timer_ns();
    };
    if (threadIdx.x == 0) stamp(0);

    // Both lists need the schedule, which exists once `sched_ready` has completed.
    // Groups: list 0 = shared experts, then active routed experts; list 1 = active
    // routed experts, then shared experts.  Each group has one or more column tiles
    // (32 token rows each in gather mode, one in direct mode) of mb weight blocks,
    // ordered (group, weight block, column tile).
    auto n_groups = [&]() { return nsh + s_n_act; };
    auto list_tiles = [&](int list) { return s_tp[list][n_groups()]; };
    auto unit_info = [&](int list, int tile) {
        const int* tp = s_tp[list];
        int lo = 0, hi = n_groups() - 1;  // the group g with tp[g] <= tile < tp[g + 1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (tp[mid] <= tile) lo = mid;
            else hi = mid - 1;
        }
        const int g = lo;
        const bool shared = list == 0 ? g < nsh : g >= s_n_act;
        const int s = list == 0 ? g : g - s_n_act;
        const int e = shared ? 0 : s_seg_e[list == 0 ? g - nsh : g];
        const int rows = shared ? T : s_cnt[e];
        const int nct = gather ? (rows + kDecodeColTile - 1) / kDecodeColTile : 1;
        const int local = tile - tp[g];
        UnitInfo u;
        u.mb = local / nct;
        const int ct = local - u.mb * nct;
        const int slot = shared ? E + s : e;
        u.a_row = list == 0 ? ((slot * mb1 + u.mb) * nkb1) * kBlockM : ((slot * mb2 + u.mb) * nkb2) * kBlockM;
        u.routed = !shared;
        const int base = shared ? args.h_shared_base + s * T : s_eoff[e];
        u.hrow0 = base + ct * kDecodeColTile;
        u.nout = gather ? min(kDecodeColTile, rows - ct * kDecodeColTile) : rows;
        u.tok0 = shared ? ct * kDecodeColTile : 0;
        u.by_token = !gather && !shared && list == 0;
        if (list == 1) {
            u.bmap = kBh;
            u.b_row = u.hrow0;
        } else if (shared || !gather) {
            u.bmap = kBx;
            u.b_row = gather ? ct * kDecodeColTile : 0;
        } else {
            u.bmap = kBxperm;
            u.b_row = u.hrow0;
        }
        return u;
    };

    if (warp == 0) {
        if (lane == 0) {
            // ── TMA producer ──
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0;
            uint32_t issued_phase = 0;
            bool ok = true;
            if (has_tasks) {
                // The CTA's router rows and each round's token rows (see `staged`).
                const uint32_t rbytes = static_cast<uint32_t>(kEpiWarps) * H * 4;
                uint32_t xbytes[2] = {0, 0};
                for (int r = 0; r < rounds; ++r) {
                    const int tg = my_q + r * cta_per_eb;
                    if (tg < ntg) xbytes[r] = static_cast<uint32_t>(min(kLogitTokens, T - tg * kLogitTokens)) * H * 2;
                }
                mbar_arrive_expect_tx(logit_bar, rbytes + xbytes[0] + xbytes[1]);
                const uint8_t* rsrc =
                    reinterpret_cast<const uint8_t*>(args.router + static_cast<size_t>(my_eb) * kEpiWarps * H);
                for (uint32_t off = 0; off < rbytes; off += 16384)
                    bulk_load(reinterpret_cast<uint8_t*>(st_router) + off, rsrc + off,
                              rbytes - off < 16384 ? rbytes - off : 16384, logit_bar);
                for (int r = 0; r < rounds; ++r) {
                    const int t0 = (my_q + r * cta_per_eb) * kLogitTokens;
                    const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(args.x + static_cast<size_t>(t0) * H);
                    uint8_t* dst = reinterpret_cast<uint8_t*>(st_x + static_cast<size_t>(r) * kLogitTokens * H);
                    for (uint32_t off = 0; off < xbytes[r]; off += 16384)
                        bulk_load(dst + off, xsrc + off, xbytes[r] - off < 16384 ? xbytes[r] - off : 16384, logit_bar);
                }
            }
            // Token tiles whose rows are not written yet (x_perm before counter 2, h
            // before counter 1), oldest first: every x_perm entry precedes every h one.
            int pend_stage[kMaxPending], pend_map[kMaxPending], pend_y[kMaxPending], pend_x[kMaxPending];
            int pend_head = 0, pend_n = 0;
            bool ready[2] = {!gather, false};  // [0] x_perm, [1] h
            auto flush = [&](bool block) {
                while (pend_n > 0) {
                    const int m = pend_map[pend_head];
                    if (!ready[m]) {
                        unsigned long long* ctr = args.grid_bar + (m == 0 ? kCtrXperm : kCtrH);
                        if (block) {
                            if (!grid_wait(ctr, target, abort_flag, args.status, kDevTimeoutGrid,
                                           args.wait_limit_ns)) {
                                ok = false;
                                return;
                            }
                        } else if (ld_acquire_u64(ctr) < target) {
                            return;
                        }
                        fence_proxy_async_global();
                        ready[m] = true;
                        stamp(m == 0 ? 15 : 5);
                    }
                    const int st = pend_stage[pend_head];
                    tma_load_2d(smem_b + st * C::kBTile, m == 0 ? &map_xperm : &map_h, &full[st], pend_x[pend_head],
                                pend_y[pend_head]);
                    pend_head = (pend_head + 1) % kMaxPending;
                    --pend_n;
                }
            };
            // Stay off HBM until the routing is done: under a saturated weight stream
            // every global access of the routing -- the logits, and the instruction
            // fetches of code run for the first time -- waits microseconds in the
            // memory queues, which costs more than streaming early gains.
            const uint64_t pf_total = args.prefetch_len[0] + args.prefetch_len[1];
            if (pf_total > 0) {
                // The router logits are read once every CTA has written its share: from then
                // on the routing touches only L2 and shared memory, and HBM would idle until
                // the schedule exists.  Bring this CTA's share of the weights into L2 meanwhile.
                ok = grid_wait(args.grid_bar + kCtrLogits, target, abort_flag, args.status, kDevTimeoutGrid,
                               args.wait_limit_ns);
                const uint64_t per = ((pf_total + G - 1) / G + 4095) & ~uint64_t(4095);
                uint64_t off = per * blockIdx.x;
                const uint64_t hi = off + per < pf_total ? off + per : pf_total;
                while (ok && off < hi) {
                    const int r = off < args.prefetch_len[0] ? 0 : 1;
                    const uint64_t r0 = r == 0 ? 0 : args.prefetch_len[0];
                    const uint64_t r_end = r == 0 && hi > args.prefetch_len[0] ? args.prefetch_len[0] : hi;
                    const uint64_t n = r_end - off < 32768 ? r_end - off : 32768;
                    bulk_prefetch_l2(args.prefetch_base[r] + (off - r0), static_cast<uint32_t>(n));
                    off += n;
                }
            }
            if (ok) ok = mbar_wait(sched_ready, 0, abort_flag, args.status, kDevTimeoutProducer);
            const uint64_t weight_policy = policy_evict_first();
            for (int list = 0; list <= 1 && ok; ++list) {
                const int nkb = list == 1 ? nkb2 : nkb1;
                const CUtensorMap* amap = list == 1 ? &map_w2 : &map_w13;
                ListWalk walk;
                walk.init(list_tiles(list), nkb);
                int tile, kb0, kb1;
                while (ok && walk.next(tile, kb0, kb1)) {
                    const UnitInfo u = unit_info(list, tile);
                    for (int kb = kb0; kb < kb1 && ok; ++kb) {
                        // A ring of stages all waiting for token rows drains only once
                        // every CTA has written them.
                        flush(pend_n == S);
                        if (!ok) break;
                        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, kDevTimeoutProducer)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[stage], kATile + C::kBTile);
                        if (args.weight_evict_first)
                            tma_load_2d_hint(smem_a + stage * kATile, amap, &full[stage], 0, u.a_row + kb * kBlockM,
                                             weight_policy);
                        else
                            tma_load_2d(smem_a + stage * kATile, amap, &full[stage], 0, u.a_row + kb * kBlockM);
                        if (u.bmap == kBx) {
                            tma_load_2d(smem_b + stage * C::kBTile, &map_x, &full[stage], kb * kBlockK, u.b_row);
                        } else {
                            const int m = u.bmap == kBxperm ? 0 : 1;
                            if (ready[m] && pend_n == 0) {
                                tma_load_2d(smem_b + stage * C::kBTile, m == 0 ? &map_xperm : &map_h, &full[stage],
                                            kb * kBlockK, u.b_row);
                            } else {
                                const int slot = (pend_head + pend_n) % kMaxPending;
                                pend_stage[slot] = stage;
                                pend_map[slot] = m;
                                pend_x[slot] = kb * kBlockK;
                                pend_y[slot] = u.b_row;
                                ++pend_n;
                                flush(false);
                            }
                        }
                        issued_mask |= 1u << stage;
                        issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (ok) flush(true);
            stamp(6);
            if (!ok) {
                // Loads already issued still land in this CTA's shared memory: wait for
                // them (bounded) before the CTA can exit.
                for (int st = 0; st < S; ++st)
                    if (issued_mask & (1u << st)) mbar_wait_drain(&full[st], (issued_phase >> st) & 1u, 100000000ull);
            }
            // The logit inputs' copies (long landed on every path that got this far).
            if (has_tasks) mbar_wait_drain(logit_bar, 0, 100000000ull);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ── MMA issuer ──
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            bool issued_any = false;
            if (!mbar_wait(sched_ready, 0, abort_flag, args.status, kDevTimeoutMma)) ok = false;
            for (int list = 0; list <= 1 && ok; ++list) {
                ListWalk walk;
                walk.init(list_tiles(list), list == 1 ? nkb2 : nkb1);
                int tile, kb0, kb1;
                while (ok && walk.next(tile, kb0, kb1)) {
                    if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, args.status, kDevTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                    for (int kb = kb0; kb < kb1; ++kb) {
                        if (!mbar_wait(&full[stage], phase, abort_flag, args.status, kDevTimeoutMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t a_desc = umma_desc_sw128(smem_u32(smem_a + stage * kATile));
                        const uint64_t b_desc = umma_desc_sw128(smem_u32(smem_b + stage * C::kBTile));
#pragma unroll
                        for (int kk = 0; kk < kBlockK / 16; ++kk)
                            umma_bf16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, kIdesc, (kb != kb0) || (kk != 0));
                        issued_any = true;
                        umma_commit(&empty[stage]);
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    umma_commit(&tmem_full[acc]);
                    if (++acc == 2) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                }
            }
            if (!ok && issued_any) {
                umma_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0, 100000000ull);
            }
            stamp(8);
        }
    } else {
        // ── Routing, then the epilogue: warps 2..9 ──
        const int epi_tid = threadIdx.x - 64;
        const int ew = epi_tid >> 5;
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        bool ok = true;
        // One thread waits; the named barrier hands the outcome to all eight warps
        // (the slot alternates so a slow warp never reads the next outcome).
        int go_slot = 0;
        auto broadcast = [&](bool v) {
            if (epi_tid == 0) s_go[go_slot] = v ? 1 : 0;
            named_bar_sync(2, kEpiThreads);
            const bool r = s_go[go_slot] != 0;
            go_slot ^= 1;
            return r;
        };
        auto arrive_grid = [&](int g) {
            __threadfence();
            named_bar_sync(2, kEpiThreads);
            if (epi_tid == 0) red_release_add_u64(args.grid_bar + g, 1ull);
        };
        auto wait_grid = [&](int g) {
            return broadcast(epi_tid == 0 ? grid_wait(args.grid_bar + g, target, abort_flag, args.status,
                                                      kDevTimeoutGrid, args.wait_limit_ns)
                                          : true);
        };

        // (1) y = 0 when not accumulating; the down epilogues add into it after counter 1.
        if (args.zero_y) {
            const int n4 = T * H / 4;
            const int per = (n4 + G - 1) / G;
            float4* yz = reinterpret_cast<float4*>(args.y);
            for (int i = blockIdx.x * per + epi_tid; i < min(n4, (blockIdx.x + 1) * per); i += kEpiThreads)
                yz[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int e = epi_tid; e < E; e += kEpiThreads) {
            s_cnt[e] = 0;
#pragma unroll
            for (int w = 0; w < kMaskWords; ++w) rs.emask[e][w] = 0u;
        }

        if (!gather) {
            // (2) Router logits: (token, expert) dot products spread over every warp of
            // the grid; each lane's loads of a row are all issued before any is used.
            for (int p = blockIdx.x * kEpiWarps + ew; p < T * E; p += G * kEpiWarps) {
                const int t = p / E;
                const int e = p - t * E;
                const float* wr = args.router + static_cast<size_t>(e) * H;
                float acc = 0.0f;
                if (args.x_f32 != nullptr) {
                    const float* xt = args.x_f32 + static_cast<size_t>(t) * H;
#pragma unroll 8
                    for (int hh = lane * 8; hh < H; hh += 256) {
                        float xv[8], wv[8];
                        load8(xt + hh, xv);
                        load8(wr + hh, wv);
#pragma unroll
                        for (int i = 0; i < 8; ++i) acc = fmaf(xv[i], wv[i], acc);
                    }
                } else {
                    const uint16_t* xt = args.x + static_cast<size_t>(t) * H;
#pragma unroll 8
                    for (int hh = lane * 8; hh < H; hh += 256) {
                        float xv[8], wv[8];
                        load8(xt + hh, xv);
                        load8(wr + hh, wv);
#pragma unroll
                        for (int i = 0; i < 8; ++i) acc = fmaf(xv[i], wv[i], acc);
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(kFull, acc, off);
                if (lane == 0) args.logits[p] = args.bias != nullptr ? acc + args.bias[e] : acc;
            }
            arrive_grid(kCtrLogits);
            if (epi_tid == 0) stamp(1);
            ok = wait_grid(kCtrLogits);
            if (epi_tid == 0) stamp(2);
            if (ok) {
                // (3) All logits into shared memory in one round trip, then every token's
                // routing from there (every CTA the same).
                for (int i = epi_tid; i < T * E; i += kEpiThreads) rs.logits[i] = __ldcg(args.logits + i);
                named_bar_sync(1, kEpiThreads);
                if (epi_tid == 0) stamp(10);
                for (int t = ew; t < T; t += kEpiWarps) {
                    const Selection sel = route_one_token<EPL, true>(rs.logits + t * E, s_rp, rs.probs[ew], lane);
                    if (lane < K) {
                        rs.idx[t * K + lane] = sel.idx;
                        rs.w[t * K + lane] = sel.w;
                        atomicAdd(&s_cnt[sel.idx], 1);
                        atomicOr(&rs.emask[sel.idx][t >> 5], 1u << (t & 31));
                        if (blockIdx.x == 0) {
                            args.topk_idx[t * K + lane] = sel.idx;
                            args.topk_w[t * K + lane] = sel.w;
                        }
                    }
                }
                named_bar_sync(1, kEpiThreads);
                if (epi_tid == 0) stamp(11);
            }
        } else {
            // (2g) Router logits as warp tasks of (expert e, 8 tokens): the warp streams
            // the router row once for its 8 tokens.  Consecutive warps take consecutive
            // experts of the same tokens, so a CTA's token rows stay in L1.
            if (staged) {
                // Inputs in shared memory: warp ew takes expert my_eb * kEpiWarps + ew of
                // each round's token group (every thread waits for the copies itself; an
                // expired wait has recorded its status, which the grid wait below sees).
                const bool got = has_tasks && mbar_wait(logit_bar, 0, abort_flag, args.status, kDevTimeoutEpilogue);
                for (int r = 0; got && r < rounds; ++r) {
                    const int tg = my_q + r * cta_per_eb;
                    if (tg >= ntg) break;
                    const int e = my_eb * kEpiWarps + ew;
                    const int t0 = tg * kLogitTokens;
                    const int nt = min(kLogitTokens, T - t0);
                    const float* wr = st_router + static_cast<size_t>(ew) * H;
                    const uint16_t* xr = st_x + static_cast<size_t>(r) * kLogitTokens * H;
                    float acc[kLogitTokens];
#pragma unroll
                    for (int j = 0; j < kLogitTokens; ++j) acc[j] = 0.0f;
                    for (int hh = lane * 8; hh < H; hh += 256) {
                        const float4 w0 = *reinterpret_cast<const float4*>(wr + hh);
                        const float4 w1 = *reinterpret_cast<const float4*>(wr + hh + 4);
                        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                        for (int j = 0; j < kLogitTokens; ++j) {
                            const uint4 raw = *reinterpret_cast<const uint4*>(xr + static_cast<size_t>(min(j, nt - 1)) * H + hh);
                            const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                acc[j] = fmaf(__uint_as_float(words[i] << 16), wv[2 * i], acc[j]);
                                acc[j] = fmaf(__uint_as_float(words[i] & 0xFFFF0000u), wv[2 * i + 1], acc[j]);
                            }
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kLogitTokens; ++j) {
#pragma unroll
                        for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(kFull, acc[j], off);
                    }
                    float v = acc[0];
#pragma unroll
                    for (int j = 1; j < kLogitTokens; ++j)
                        if (lane == j) v = acc[j];
                    if (lane < nt) args.logits[(t0 + lane) * E + e] = args.bias != nullptr ? v + args.bias[e] : v;
                }
            }
            for (int p = blockIdx.x * kEpiWarps + ew; !staged && p < E * ntg; p += G * kEpiWarps) {
                const int tg = p / E;
                const int e = p - tg * E;
                const int t0 = tg * kLogitTokens;
                const int nt = min(kLogitTokens, T - t0);
                const float* wr = args.router + static_cast<size_t>(e) * H;
                float acc[kLogitTokens];
#pragma unroll
                for (int j = 0; j < kLogitTokens; ++j) acc[j] = 0.0f;
                // Every load of a step is issued before any is used (a load under a
                // token-count branch would wait out its own round trip): tokens past the
                // batch re-read its last row and are never stored.
                if (args.x_f32 != nullptr) {
                    for (int hh = lane * 8; hh < H; hh += 256) {
                        float wv[8];
                        load8(wr + hh, wv);
#pragma unroll
                        for (int j = 0; j < kLogitTokens; ++j) {
                            float xv[8];
                            load8(args.x_f32 + static_cast<size_t>(min(t0 + j, T - 1)) * H + hh, xv);
#pragma unroll
                            for (int i = 0; i < 8; ++i) acc[j] = fmaf(xv[i], wv[i], acc[j]);
                        }
                    }
                } else {
#pragma unroll 2
                    for (int hh = lane * 8; hh < H; hh += 256) {
                        float wv[8];
                        load8(wr + hh, wv);
                        uint4 raw[kLogitTokens];
#pragma unroll
                        for (int j = 0; j < kLogitTokens; ++j)
                            raw[j] = *reinterpret_cast<const uint4*>(args.x + static_cast<size_t>(min(t0 + j, T - 1)) * H + hh);
#pragma unroll
                        for (int j = 0; j < kLogitTokens; ++j) {
                            const uint32_t words[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                acc[j] = fmaf(__uint_as_float(words[i] << 16), wv[2 * i], acc[j]);
                                acc[j] = fmaf(__uint_as_float(words[i] & 0xFFFF0000u), wv[2 * i + 1], acc[j]);
                            }
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < kLogitTokens; ++j) {
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(kFull, acc[j], off);
                }
                float v = acc[0];
#pragma unroll
                for (int j = 1; j < kLogitTokens; ++j)
                    if (lane == j) v = acc[j];
                if (lane < nt) args.logits[(t0 + lane) * E + e] = args.bias != nullptr ? v + args.bias[e] : v;
            }
            arrive_grid(kCtrLogits);
            if (epi_tid == 0) stamp(1);
            ok = wait_grid(kCtrLogits);
            if (epi_tid == 0) stamp(2);
            if (ok) {
                // (3g) Each token's top-k once in the grid: token t on warp t / G of CTA t % G.
                for (int t = blockIdx.x + G * ew; t < T; t += G * kEpiWarps) {
                    const Selection sel = route_one_token<EPL, false>(args.logits + t * E, s_rp, rs.probs[ew], lane);
                    if (lane < K) {
                        args.topk_idx[t * K + lane] = sel.idx;
                        args.topk_w[t * K + lane] = sel.w;
                    }
                }
                arrive_grid(kCtrTopk);
                if (epi_tid == 0) stamp(9);
                ok = wait_grid(kCtrTopk);
                if (epi_tid == 0) stamp(13);
            }
            if (ok) {
                // (4g) Every CTA reads all selections (16 bytes per load, every load of a
                // thread issued before any is used) and builds the same histogram.
                const int n_pairs = T * K;
                const int n_vec = n_pairs / 4;
                constexpr int kVecPerThread = (kDecodeMaxRows / 4 + kEpiThreads - 1) / kEpiThreads;
                int4 vi[kVecPerThread];
                float4 vw[kVecPerThread];
#pragma unroll
                for (int j = 0; j < kVecPerThread; ++j) {
                    const int v = epi_tid + j * kEpiThreads;
                    if (v < n_vec) {
                        vi[j] = __ldcg(reinterpret_cast<const int4*>(args.topk_idx) + v);
                        vw[j] = __ldcg(reinterpret_cast<const float4*>(args.topk_w) + v);
                    }
                }
                auto take = [&](int q, int e, float w) {
                    const int t = q / K;
                    rs.idx[q] = e;
                    rs.w[q] = w;
                    atomicAdd(&s_cnt[e], 1);
                    atomicOr(&rs.emask[e][t >> 5], 1u << (t & 31));
                };
#pragma unroll
                for (int j = 0; j < kVecPerThread; ++j) {
                    const int v = epi_tid + j * kEpiThreads;
                    if (v < n_vec) {
                        take(4 * v, vi[j].x, vw[j].x);
                        take(4 * v + 1, vi[j].y, vw[j].y);
                        take(4 * v + 2, vi[j].z, vw[j].z);
                        take(4 * v + 3, vi[j].w, vw[j].w);
                    }
                }
                for (int q = 4 * n_vec + epi_tid; q < n_pairs; q += kEpiThreads)
                    take(q, __ldcg(args.topk_idx + q), __ldcg(args.topk_w + q));
                named_bar_sync(1, kEpiThreads);
                if (epi_tid == 0) stamp(11);
            }
        }

        if (ok) {
            // (4) Active experts and their first rows: a warp-wide compaction and scan.
            if (ew == 0) {
                int n = 0, off = 0;
                for (int base = 0; base < E; base += 32) {
                    const int e = base + lane;
                    const int c = e < E ? s_cnt[e] : 0;
                    int incl = c;
#pragma unroll
                    for (int d = 1; d < 32; d <<= 1) {
                        const int v = __shfl_up_sync(kFull, incl, d);
                        if (lane >= d) incl += v;
                    }
                    const uint32_t act = __ballot_sync(kFull, c > 0);
                    if (c > 0) {
                        s_seg_e[n + __popc(act & ((1u << lane) - 1u))] = e;
                        s_eoff[e] = off + incl - c;
                    }
                    n += __popc(act);
                    off += __shfl_sync(kFull, incl, 31);
                }
                if (lane == 0) s_n_act = n;
            }
            named_bar_sync(1, kEpiThreads);
            if (epi_tid == 0) stamp(12);
            // (5) Expert-sorted rows, tokens in order within an expert: a token picks an
            // expert at most once, so its rank there counts the expert's earlier tokens.
            const int n_pairs = T * K;
            for (int q = epi_tid; q < n_pairs; q += kEpiThreads) {
                const int e = rs.idx[q];
                const int t = q / K;
                int r = 0;
                for (int w = 0; w < (t >> 5); ++w) r += __popc(rs.emask[e][w]);
                r += __popc(rs.emask[e][t >> 5] & ((1u << (t & 31)) - 1u));
                const int row = s_eoff[e] + r;
                s_row_token[row] = t;
                s_row_w[row] = rs.w[q];
            }
            // (6) The two lists' tile prefixes (warps 1 and 2 of the epilogue).
            if (ew == 1 || ew == 2) {
                const int list = ew - 1;
                const int ng = nsh + s_n_act;
                const int mbn = list == 0 ? mb1 : mb2;
                int run = 0;
                if (lane == 0) s_tp[list][0] = 0;
                for (int base = 0; base < ng; base += 32) {
                    const int g = base + lane;
                    int v = 0;
                    if (g < ng) {
                        const bool shared = list == 0 ? g < nsh : g >= s_n_act;
                        const int rows = shared ? T : s_cnt[s_seg_e[list == 0 ? g - nsh : g]];
                        v = (gather ? (rows + kDecodeColTile - 1) / kDecodeColTile : 1) * mbn;
                    }
                    int incl = v;
#pragma unroll
                    for (int d = 1; d < 32; d <<= 1) {
                        const int o = __shfl_up_sync(kFull, incl, d);
                        if (lane >= d) incl += o;
                    }
                    if (g < ng) s_tp[list][g + 1] = run + incl;
                    run += __shfl_sync(kFull, incl, 31);
                }
            }
            // The ring's stages held the routing's scratch and the logit inputs: order
            // those shared-memory accesses before the pipeline's TMA writes.
            fence_proxy_async_shared();
            named_bar_sync(1, kEpiThreads);
            if (epi_tid == 0) {
                mbar_arrive(sched_ready);  // producer and MMA may decode the lists
                stamp(3);
            }
            if (blockIdx.x == 0) {
                for (int r = epi_tid; r < n_pairs; r += kEpiThreads) {
                    args.row_token[r] = s_row_token[r];
                    args.row_weight[r] = s_row_w[r];
                }
                for (int e = epi_tid; e < E; e += kEpiThreads) args.expert_totals[e] = s_cnt[e];
            }
            if (gather) {
                // (7g) This CTA's share of the token rows into expert order.
                const int q0 = static_cast<int>(static_cast<int64_t>(n_pairs) * blockIdx.x / G);
                const int q1 = static_cast<int>(static_cast<int64_t>(n_pairs) * (blockIdx.x + 1) / G);
                const int vec = H / 8;
                constexpr int kGatherBatch = 8;  // rows whose loads are in flight together
                for (int qb = q0; qb < q1; qb += kGatherBatch) {
                    for (int i = epi_tid; i < vec; i += kEpiThreads) {
                        uint4 v[kGatherBatch];
#pragma unroll
                        for (int j = 0; j < kGatherBatch; ++j)
                            if (qb + j < q1)
                                v[j] = reinterpret_cast<const uint4*>(
                                    args.x + static_cast<size_t>(s_row_token[qb + j]) * H)[i];
#pragma unroll
                        for (int j = 0; j < kGatherBatch; ++j)
                            if (qb + j < q1)
                                reinterpret_cast<uint4*>(args.x_perm + static_cast<size_t>(qb + j) * H)[i] = v[j];
                    }
                }
                fence_proxy_async_global();
                arrive_grid(kCtrXperm);
                if (epi_tid == 0) stamp(14);
            }
        }

        // (8) Epilogues of both lists, in the order the MMA issuer produced them.
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int list = 0; list <= 1 && ok; ++list) {
            if (list == 1) {
                // Every h row this CTA writes is written: publish them for the TMA reads.
                fence_proxy_async_global();
                arrive_grid(kCtrH);
                if (epi_tid == 0) stamp(4);
            }
            const int tiles = list_tiles(list);
            const int nkb = list == 1 ? nkb2 : nkb1;
            ListWalk walk;
            walk.init(tiles, nkb);
            int tile, kb0, kb1;
            while (walk.next(tile, kb0, kb1)) {
                const UnitInfo u = unit_info(list, tile);
                // TMEM columns holding results: direct-mode routed gate/up has every token
                // as a column; otherwise the unit's own rows.
                const int ncols = u.by_token ? T : u.nout;
                const bool whole = kb0 == 0 && kb1 == nkb;
                // A gate/up tile split over CTAs is completed by the CTA holding its first
                // k-blocks: they end that CTA's range, so the other CTAs' shares (the
                // starts of theirs) are written long before.  It fetches those partial
                // sums while its own accumulator fills; its own sums never leave TMEM.
                const bool completes = list == 0 && kb0 == 0 && !whole;
                const int row = quad * 32 + lane;  // this thread's TMEM lane (weight row)
                const int c0 = 16 * half;          // and its 16 columns (BN <= 32)
                float pre[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) pre[j] = 0.0f;
                if (completes) {
                    const int64_t iters = static_cast<int64_t>(tiles) * nkb;
                    const int64_t j0 = static_cast<int64_t>(tile) * nkb;
                    // CTA owning iteration j: the largest c with iters * c / G <= j.
                    const int c_hi = static_cast<int>(((j0 + nkb) * G + iters - 1) / iters) - 1;
                    ok = broadcast(epi_tid == 0 ? count_wait_s32(args.split_ticket + tile, nkb - kb1, abort_flag,
                                                                 args.status, kDevTimeoutEpilogue,
                                                                 args.wait_limit_ns)
                                                : true);
                    if (!ok) break;
                    __threadfence();
                    if (c0 < ncols) {
                        // The tile's other k-blocks start the ranges of CTAs blockIdx.x + 1 ..
                        // c_hi, each the first unit there: slot 2 * cta.  Summed in CTA order.
                        for (int cta = static_cast<int>(blockIdx.x) + 1; cta <= c_hi; ++cta) {
                            if (iters * (cta + 1) / G == iters * cta / G) continue;  // empty range
                            const float* part = args.split_ws + static_cast<size_t>(2 * cta) * (kBlockM * BN);
                            float v[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                v[j] = c0 + j < ncols ? __ldcg(part + (c0 + j) * kBlockM + row) : 0.0f;
#pragma unroll
                            for (int j = 0; j < 16; ++j) pre[j] += v[j];
                        }
                    }
                }
                ok = broadcast(epi_tid == 0 ? mbar_wait(&tmem_full[acc], acc_phase, abort_flag, args.status,
                                                        kDevTimeoutEpilogue)
                                            : true);
                if (!ok) break;
                tc_fence_after();
                const uint32_t t_row =
                    tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
                if (list == 0 && !whole && !completes) {
                    // This CTA's share of a tile another CTA completes (the first unit of
                    // its range): the partial sums to its slot, then the k-block count.
                    float* wt = args.split_ws + static_cast<size_t>(2 * blockIdx.x) * (kBlockM * BN);
                    if (c0 < ncols) {
                        uint32_t r[16];
                        tmem_ld16(t_row + c0, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (c0 + j < ncols) __stcg(wt + (c0 + j) * kBlockM + row, __uint_as_float(r[j]));
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                    __threadfence();
                    named_bar_sync(1, kEpiThreads);
                    if (epi_tid == 0) red_release_add_s32(args.split_ticket + tile, kb1 - kb0);
                } else if (list == 0) {
                    // A whole gate/up tile, or a split one this CTA completes:
                    // h = silu(gate) * up through a staging tile.
                    __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(staging);
                    const int i_local = row >> 1;
                    if (c0 < ncols) {
                        uint32_t r[16];
                        tmem_ld16(t_row + c0, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float mine = __uint_as_float(r[j]) + pre[j];
                            const float other = __shfl_xor_sync(kFull, mine, 1);
                            if ((lane & 1) == 0)
                                st[(c0 + j) * 64 + i_local] = __float2bfloat16_rn(silu_times(mine, other));
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                    named_bar_sync(1, kEpiThreads);
                    const uint4* src = reinterpret_cast<const uint4*>(staging);
                    for (int q = epi_tid; q < u.nout * 8; q += kEpiThreads) {
                        const int j = q >> 3;
                        const int part = q & 7;
                        const int col = u.by_token ? s_row_token[u.hrow0 + j] : j;
                        uint4* dst =
                            reinterpret_cast<uint4*>(args.h + static_cast<size_t>(u.hrow0 + j) * I + u.mb * 64) + part;
                        *dst = src[col * 8 + part];
                    }
                    if (completes && epi_tid == 0) args.split_ticket[tile] = 0;  // every share is consumed
                    named_bar_sync(1, kEpiThreads);
                } else {
                    // Down: routing weight x output, added into y[token] (128-byte runs).
                    const int d = u.mb * kBlockM + row;
                    if (c0 < ncols) {
                        uint32_t r[16];
                        tmem_ld16(t_row + c0, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int c = c0 + j;
                            if (c < ncols) {
                                const int tok = u.routed ? s_row_token[u.hrow0 + c] : u.tok0 + c;
                                const float w = u.routed ? s_row_w[u.hrow0 + c] : 1.0f;
                                atomicAdd(args.y + static_cast<size_t>(tok) * H + d, w * __uint_as_float(r[j]));
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                }
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
        if (epi_tid == 0) stamp(7);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
    // Every wait of this CTA is over.  The last CTA to get here has seen every CTA
    // finish waiting, so it re-arms the counters for the next launch.
    if (threadIdx.x == 0 &&
        atom_acq_rel_add_u64(args.grid_bar + kCtrExit, 1ull) == static_cast<unsigned long long>(G) - 1ull) {
        for (int i = 0; i < kDecodeCounters; ++i) args.grid_bar[i] = 0ull;
        __threadfence();
    }
}

template <int BN, int EPL>
cudaError_t launch_t(const CUtensorMap& w13, const CUtensorMap& w2, const CUtensorMap& x, const CUtensorMap& xperm,
                     const CUtensorMap& h, const DecodeArgs& args, int sms, cudaStream_t stream) {
    using C = DCfg<BN>;
    auto kernel = moe_decode_kernel<BN, EPL>;
    static std::atomic<uint64_t> configured{0};  // devices whose limit is raised
    if (const cudaError_t e = set_smem_limit_once(kernel, C::kSmem, configured); e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    // Co-residency of every CTA is what makes the grid counters safe to wait on.
    // Programmatic serialization lets the launch and the prologue overlap the
    // previous kernel; the kernel waits for it before touching memory.
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, w13, w2, x, xperm, h, args);
}

}  // namespace

cudaError_t launch_moe_decode(int bn, const CUtensorMap& w13, const CUtensorMap& w2, const CUtensorMap& x,
                              const CUtensorMap& xperm, const CUtensorMap& h, const DecodeArgs& args, int sms,
                              cudaStream_t stream) {
    if (args.tokens <= 0) return cudaSuccess;
    const bool gather = args.gather != 0;
    if (args.tokens > kDecodeMaxTokens || args.rp.experts > kMaxExperts || args.rp.top_k > kMaxTopK ||
        args.tokens * args.rp.top_k > kDecodeMaxRows || args.n_shared > kMaxShared ||
        (gather ? bn != kDecodeColTile : (args.tokens > bn || args.tokens * args.rp.experts > kDecodeMaxLogits)))
        return cudaErrorInvalidValue;
    const int need = (args.rp.experts + 31) / 32;
    const int epl = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : 8;
#define LM_DECODE(BN_)                                                                \
    switch (epl) {                                                                    \
        case 1: return launch_t<BN_, 1>(w13, w2, x, xperm, h, args, sms, stream);     \
        case 2: return launch_t<BN_, 2>(w13, w2, x, xperm, h, args, sms, stream);     \
        case 4: return launch_t<BN_, 4>(w13, w2, x, xperm, h, args, sms, stream);     \
        default: return launch_t<BN_, 8>(w13, w2, x, xperm, h, args, sms, stream);    \
    }
    if (bn == 16) LM_DECODE(16)
    if (bn == 32) LM_DECODE(32)
#undef LM_DECODE
    return cudaErrorInvalidValue;
}

}  // namespace lm
