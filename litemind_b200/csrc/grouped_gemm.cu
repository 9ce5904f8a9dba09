// grouped_gemm.cu -- the expert products of the MoE path on tcgen05 tensor cores.
//
// The reference computes each selected expert per token as three BF16 matvecs
// (Impl::feed_forward, src/DeepSeekRunner.cpp:228-240: gemm::matvec_bf16 for gate
// and up, gemm::silu_multiply, gemm::matvec_bf16_accumulate for down with the
// routing weight).  Here all tokens of all experts run as two grouped GEMMs over
// ragged expert segments, weights on the MMA's M side ("swap-AB"), tokens on N:
//
//   gate/up:  D[128 weight rows, BN tokens] = W13_e[rows] . X_e^T     (K = hidden)
//             W13 interleaves gate and up rows in pairs, so the epilogue pairs
//             lanes 2i/2i+1 and writes h = silu(gate) * up (bf16) for 64 columns
//             of the intermediate axis.
//   down:     D[128 hidden rows, BN tokens] = W2_e[rows] . H_e^T       (K = inter)
//             The epilogue multiplies by each token's routing weight (1.0 for the
//             shared experts) and adds into y[token] -- the weighted combine and
//             the un-permute in one step.  Lanes of a warp hold 32 consecutive
//             hidden rows, so every atomic add is a coalesced 128-byte run.
//
// One persistent CTA per SM walks the tile list in the device-built Schedule --
// whole tiles, or for launches of few tiles an equal share of all tiles' k-blocks
// ("stream-K").  Warp 0 fills a ring of smem stages by TMA tile loads (128-byte
// swizzle, each CTA loading its own tiles): weight tiles, and token tiles from the
// expert-sorted copy x_perm (routed experts) or from x itself (shared experts).
// Contiguous rows keep every token tile one TMA request; gathering rows
// individually (TMA gather4 or cp.async) measured 1.3x (decode) to 2.6x (prefill)
// slower on B200.  Warp 1 allocates TMEM and issues tcgen05.mma from one thread;
// warps 2-9 drain the double-buffered TMEM accumulators, two warps per TMEM lane
// quadrant.  Every mbarrier wait is bounded (ptx.cuh): a stalled pipeline records a
// status code and the kernel returns.
#include "moe_internal.h"
#include "ptx.cuh"
#include "gemm_rows.cuh"

#include <cuda_bf16.h>

namespace lm {
namespace {

constexpr int kBlockM = 128;
constexpr int kBlockK = 64;
constexpr int kEpiThreads = 256;  // 8 epilogue warps: two per TMEM lane quadrant
constexpr int kThreads = 64 + kEpiThreads;  // + TMA producer warp, MMA warp
constexpr int kATileBytes = kBlockM * kBlockK * 2;
constexpr int kSmemBudget = 225 * 1024;

enum class Kind { GateUp, Down, Router };

template <int BN, Kind KIND>
struct Cfg {
    static constexpr int kBTileBytes = BN * kBlockK * 2;
    static constexpr int kStageBytes = kATileBytes + kBTileBytes;
    static constexpr int kStagingBytes = (KIND == Kind::GateUp) ? BN * 64 * 2 : 0;
    static constexpr int kBarrierBytes = 1024;
    static constexpr int kStagesFit = (kSmemBudget - kStagingBytes - kBarrierBytes - 1024) / kStageBytes;
    static constexpr int kStages = kStagesFit > 12 ? 12 : kStagesFit;
    static constexpr int kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;
    static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kStagingBytes + kBarrierBytes;
    static_assert(kStages >= 2, "pipeline needs at least two stages");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ int find_segment(const int* tiles, int n_seg, int tile) {
    int lo = 0, hi = n_seg;  // tiles[lo] <= tile < tiles[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (tiles[mid] <= tile) lo = mid; else hi = mid;
    }
    return lo;
}

// Every role of a CTA walks the same list of work units (tile, k-blocks [kb0, kb1)).
// Unsplit: whole tiles, blockIdx.x + i * gridDim.x.  Split ("stream-K"): the
// tiles' k-block iterations laid end to end and cut into gridDim.x equal
// contiguous ranges, so a launch of few tiles keeps every SM streaming weights
// instead of leaving a part-empty last wave.
struct UnitWalk {
    int64_t it, end;  // split: this CTA's iteration range
    int tile;         // unsplit: next tile
    int total, num_kb;
    bool split;
    __device__ UnitWalk(bool split_, int total_tiles, int num_kb_)
        : tile(blockIdx.x), total(total_tiles), num_kb(num_kb_), split(split_) {
        const int64_t iters = static_cast<int64_t>(total_tiles) * num_kb_;
        it = iters * blockIdx.x / gridDim.x;
        end = iters * (blockIdx.x + 1) / gridDim.x;
    }
    __device__ bool next(int& t, int& kb0, int& kb1) {
        if (!split) {
            if (tile >= total) return false;
            t = tile;
            kb0 = 0;
            kb1 = num_kb;
            tile += gridDim.x;
            return true;
        }
        if (it >= end) return false;
        t = static_cast<int>(it / num_kb);
        kb0 = static_cast<int>(it - static_cast<int64_t>(t) * num_kb);
        const int64_t left = end - it;
        kb1 = left < num_kb - kb0 ? kb0 + static_cast<int>(left) : num_kb;
        it += kb1 - kb0;
        return true;
    }
};

__device__ __forceinline__ float silu_times(float g, float u) {
    // src/Gemm.cpp:225-231: value / (1 + exp(-value)) * up, with fast exp and
    // divide: the result is rounded to bf16 (8 significant bits) right after.
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}

template <int BN, Kind KIND>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_x, const GemmArgs args) {
    using C = Cfg<BN, KIND>;
    constexpr int S = C::kStages;
    constexpr uint32_t kIdesc = umma_idesc_bf16(kBlockM, BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ int s_tiles[kMaxSegments + 1];
    __shared__ int s_off[kMaxSegments];
    __shared__ int s_cnt[kMaxSegments];
    __shared__ int s_wslot[kMaxSegments];
    __shared__ int s_n_seg;
    __shared__ int s_epi_go[2];
    __shared__ int s_split_last;
    constexpr int kMapCols = (KIND == Kind::Down) ? BN : 1;
    __shared__ __align__(16) int s_ep_tok[2][kMapCols];  // down epilogue: this tile's token and routing weight per column
    __shared__ __align__(16) float s_ep_w[2][kMapCols];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + S * kATileBytes;
    uint8_t* staging = smem_b + S * C::kBTileBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C::kStagingBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tmem_full = bars + 2 * S;
    uint64_t* tmem_empty = bars + 2 * S + 2;
    uint64_t* drain_bar = bars + 2 * S + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], kEpiThreads / 32);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
        if (KIND != Kind::Down) tma_prefetch_desc(&map_x);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    // Everything above overlaps the previous kernel; the schedule is its output.
    pdl_wait();
    if constexpr (KIND == Kind::Router) {
        // One segment: every token, one 128-row block of router weights.
        if (threadIdx.x == 0) {
            s_n_seg = 1;
            s_off[0] = 0;
            s_cnt[0] = args.tokens;
            s_wslot[0] = 0;
            s_tiles[0] = 0;
            s_tiles[1] = (args.tokens + BN - 1) / BN;
        }
    } else {
        const Schedule* sched = args.sched;
        if (threadIdx.x == 0) s_n_seg = sched->n_seg;
        for (int i = threadIdx.x; i <= kMaxSegments; i += kThreads) {
            if (i < kMaxSegments) {
                s_off[i] = sched->seg_off[i];
                s_cnt[i] = sched->seg_cnt[i];
                s_wslot[i] = sched->seg_weight[i];
            }
            s_tiles[i] = (KIND == Kind::GateUp) ? sched->tiles1[i] : sched->tiles2[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch_dependents();

    const int n_seg = s_n_seg;
    const int total_tiles = s_tiles[n_seg];
    const uint32_t tmem_base = *tmem_slot;
    // Router: K runs over [x | x | x] against the router split into three bf16
    // parts; A is one 128-row block (experts, zero-padded).
    const int K = (KIND == Kind::GateUp) ? args.hidden : (KIND == Kind::Down) ? args.inter : 3 * args.hidden;
    const int num_kb = K / kBlockK;
    const int x_kb = args.hidden / kBlockK;
    const int rows_a = (KIND == Kind::GateUp) ? 2 * args.inter : (KIND == Kind::Down) ? args.hidden : kBlockM;
    const int mb_per = rows_a / kBlockM;
    // Down partial sums add into y like whole tiles (the combine is linear), unless
    // rows are stored unweighted for expert parallelism; gate/up partial sums need
    // the workspace.
    const bool split = total_tiles > 0 && total_tiles < args.split_max_waves * static_cast<int>(gridDim.x) &&
                       ((KIND == Kind::Down && args.y_rows == nullptr) ||
                        (KIND == Kind::GateUp && args.split_ws != nullptr && total_tiles <= kSplitTickets &&
                         static_cast<int64_t>(2 * gridDim.x) * kBlockM * BN <= args.split_ws_floats));

    if (warp == 0) {
        if (lane == 0) {
            // ── TMA producer ──
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0;
            uint32_t issued_phase = 0;
            bool ok = true;
            UnitWalk walk(split, total_tiles, num_kb);
            int tile, kb0, kb1;
            while (ok && walk.next(tile, kb0, kb1)) {
                const int s = find_segment(s_tiles, n_seg, tile);
                const int local = tile - s_tiles[s];
                const int nb = local / mb_per;
                const int mb = local - nb * mb_per;
                // Weights are tile-major: tile (segment slot, row block, k block) is 128
                // consecutive rows of a [*, 64] matrix.
                const int a_tile0 = (s_wslot[s] * mb_per + mb) * num_kb;
                // Routed experts read their expert-sorted rows of x_perm (gate/up) or h
                // (down); the shared experts read x itself, token by token.
                const bool from_x =
                    (KIND == Kind::Router) || ((KIND == Kind::GateUp) && s >= args.n_routed_local);
                const int b_row = from_x ? nb * BN : s_off[s] + nb * BN;
                const CUtensorMap* bmap = from_x ? &map_x : &map_b;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, kDevTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], kATileBytes + C::kBTileBytes);
                    if constexpr (KIND == Kind::Router) {
                        tma_load_2d(smem_a + stage * kATileBytes, &map_a, &full[stage], kb * kBlockK, 0);
                        tma_load_2d(smem_b + stage * C::kBTileBytes, bmap, &full[stage], (kb % x_kb) * kBlockK, b_row);
                    } else {
                        tma_load_2d(smem_a + stage * kATileBytes, &map_a, &full[stage], 0, (a_tile0 + kb) * kBlockM);
                        tma_load_2d(smem_b + stage * C::kBTileBytes, bmap, &full[stage], kb * kBlockK, b_row);
                    }
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                for (int st = 0; st < S; ++st)
                    if (issued_mask & (1u << st)) mbar_wait_drain(&full[st], (issued_phase >> st) & 1u, 100000000ull);
            }
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
            UnitWalk walk(split, total_tiles, num_kb);
            int tile, kb0, kb1;
            while (ok && walk.next(tile, kb0, kb1)) {
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, args.status, kDevTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, args.status, kDevTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = umma_desc_sw128(smem_u32(smem_a + stage * kATileBytes));
                    const uint64_t b_desc = umma_desc_sw128(smem_u32(smem_b + stage * C::kBTileBytes));
#pragma unroll
                    for (int kk = 0; kk < kBlockK / 16; ++kk) {
                        // +32 bytes per 16-element K step inside the swizzle atom (>> 4 in the descriptor).
                        umma_bf16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, kIdesc, (kb != kb0) || (kk != 0));
                    }
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
            if (!ok && issued_any) {
                // Wait for the MMAs already issued before TMEM is released.
                umma_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0, 100000000ull);
            }
        }
    } else {
        // ── Epilogue: warps 2..9; warp % 4 is the TMEM lane quadrant, two warps per
        // quadrant split the accumulator's 16-column chunks between them ──
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;  // which 16-column chunks: c0 = 16 * half + 32 k
        const int epi_tid = threadIdx.x - 64;  // 0..255
        int acc = 0;
        uint32_t acc_phase = 0;
        int iter = 0;
        UnitWalk walk(split, total_tiles, num_kb);
        int tile, kb0, kb1;
        for (; walk.next(tile, kb0, kb1); ++iter) {
            const int s = find_segment(s_tiles, n_seg, tile);
            const int local = tile - s_tiles[s];
            const int nb = local / mb_per;
            const int mb = local - nb * mb_per;
            const int valid = min(BN, s_cnt[s] - nb * BN);
            const int row0 = s_off[s] + nb * BN;  // first h row / routed row of this tile
            if constexpr (KIND == Kind::Down) {
                // This tile's token and routing weight per column, read once into
                // shared memory (published by the named barrier below).
                if (args.y_rows == nullptr || s >= args.n_routed_local) {
                    const bool routed = s < args.n_routed_local;
                    for (int c = epi_tid; c < valid; c += kEpiThreads) {
                        s_ep_tok[iter & 1][c] = routed ? args.row_token[row0 + c] : nb * BN + c;
                        s_ep_w[iter & 1][c] = routed ? args.row_weight[row0 + c] : 1.0f;
                    }
                }
            }
            // One thread waits; the named barrier hands its outcome to all eight
            // warps, so they leave together and never strand each other at a barrier.
            // The outcome slot alternates per tile so a slow warp never reads the next one.
            if (epi_tid == 0)
                s_epi_go[iter & 1] =
                    mbar_wait(&tmem_full[acc], acc_phase, abort_flag, args.status, kDevTimeoutEpilogue) ? 1 : 0;
            named_bar_sync(2, kEpiThreads);
            if (!s_epi_go[iter & 1]) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
            if constexpr (KIND == Kind::Router) {
                // Lane = expert, column = token: logits[token][expert] (+ bias), 32
                // consecutive experts per warp per token.
                const int e = quad * 32 + lane;
                const bool live = e < args.experts;
                const float b = (live && args.bias != nullptr) ? args.bias[e] : 0.0f;
#pragma unroll 1
                for (int c0 = 16 * half; c0 < BN; c0 += 32) {
                    if (c0 >= valid) break;
                    uint32_t r[16];
                    tmem_ld16(t_row + c0, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (live && c0 + j < valid)
                            args.logits[static_cast<size_t>(nb * BN + c0 + j) * args.experts + e] =
                                args.bias != nullptr ? __uint_as_float(r[j]) + b : __uint_as_float(r[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tmem_empty[acc]);
            } else if constexpr (KIND == Kind::GateUp) {
                if (kb0 != 0 || kb1 != num_kb) {
                    // Part of the tile's k-blocks.  Each CTA owns two workspace slots
                    // (its range's first and last unit -- the only ones that can be
                    // partial); it stores the partial gate/up sums there and counts
                    // the k-blocks.  The CTA that completes the tile sums the parts in
                    // CTA order -- the same order whichever CTA finishes last, so the
                    // result is deterministic -- and applies SiLU.
                    const int slot = 2 * static_cast<int>(blockIdx.x) + (iter == 0 ? 0 : 1);
                    float* wt = args.split_ws + static_cast<size_t>(slot) * (kBlockM * BN);
                    const int row = quad * 32 + lane;
#pragma unroll 1
                    for (int c0 = 16 * half; c0 < BN; c0 += 32) {
                        if (c0 >= valid) break;
                        uint32_t r[16];
                        tmem_ld16(t_row + c0, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (c0 + j < valid) __stcg(wt + (c0 + j) * kBlockM + row, __uint_as_float(r[j]));
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                    __threadfence();
                    named_bar_sync(1, kEpiThreads);
                    if (epi_tid == 0)
                        s_split_last = atomicAdd(args.split_ticket + tile, kb1 - kb0) + (kb1 - kb0) == num_kb;
                    named_bar_sync(1, kEpiThreads);
                    if (s_split_last) {
                        __threadfence();
                        const int64_t iters = static_cast<int64_t>(total_tiles) * num_kb;
                        const int G = gridDim.x;
                        const int64_t j0 = static_cast<int64_t>(tile) * num_kb;
                        // CTA owning iteration j: the largest c with iters * c / G <= j.
                        const int c_lo = static_cast<int>(((j0 + 1) * G + iters - 1) / iters) - 1;
                        const int c_hi = static_cast<int>(((j0 + num_kb) * G + iters - 1) / iters) - 1;
                        for (int q = epi_tid; q < valid * 64; q += kEpiThreads) {
                            const int c = q >> 6;
                            const int i = q & 63;
                            float g = 0.0f, u = 0.0f;
                            for (int cta = c_lo; cta <= c_hi; ++cta) {
                                const int64_t b = iters * cta / G;
                                if (iters * (cta + 1) / G == b) continue;  // empty range
                                const int sl = 2 * cta + (b >= j0 ? 0 : 1);
                                const float2 v = __ldcg(reinterpret_cast<const float2*>(
                                    args.split_ws + static_cast<size_t>(sl) * (kBlockM * BN) + c * kBlockM + 2 * i));
                                g += v.x;
                                u += v.y;
                            }
                            reinterpret_cast<__nv_bfloat16*>(args.h)[static_cast<size_t>(row0 + c) * args.inter +
                                                                     mb * 64 + i] = __float2bfloat16_rn(silu_times(g, u));
                        }
                        if (epi_tid == 0) args.split_ticket[tile] = 0;
                    }
                    if (++acc == 2) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                    continue;
                }
                __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(staging);
                const int i_local = (quad * 32 + lane) >> 1;  // h column within the tile's 64
#pragma unroll 1
                for (int c0 = 16 * half; c0 < BN; c0 += 32) {
                    if (c0 >= valid) break;  // warp-uniform
                    uint32_t r[16];
                    tmem_ld16(t_row + c0, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float mine = __uint_as_float(r[j]);
                        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
                        if ((lane & 1) == 0) st[(c0 + j) * 64 + i_local] = __float2bfloat16_rn(silu_times(mine, other));
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                named_bar_sync(1, kEpiThreads);
                // Staging [valid tokens][64] -> h rows, 128 contiguous bytes per row.
                const uint4* src = reinterpret_cast<const uint4*>(staging);
                for (int q = epi_tid; q < valid * 8; q += kEpiThreads) {
                    const int c = q >> 3;
                    const int part = q & 7;
                    uint4* dst = reinterpret_cast<uint4*>(args.h + static_cast<size_t>(row0 + c) * args.inter +
                                                          mb * 64) + part;
                    *dst = src[c * 8 + part];
                }
                named_bar_sync(1, kEpiThreads);
            } else {
                const int d = mb * kBlockM + quad * 32 + lane;  // hidden row
                const bool routed = s < args.n_routed_local;
                if (routed && args.y_rows != nullptr) {
                    // Expert parallelism: each routed row's output goes back to its
                    // token's rank, which applies the weight; one writer per element.
#pragma unroll 1
                    for (int c0 = 16 * half; c0 < BN; c0 += 32) {
                        if (c0 >= valid) break;
                        uint32_t r[16];
                        tmem_ld16(t_row + c0, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (c0 + j < valid) {
                                const int row = row0 + c0 + j;
                                const int dst = y_row_dst(args, row);
                                if (dst >= 0)
                                    reinterpret_cast<__nv_bfloat16*>(args.y_rows)[static_cast<size_t>(dst) * args.hidden +
                                                                                  d] =
                                        __float2bfloat16_rn(__uint_as_float(r[j]));
                            }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                    if (++acc == 2) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                    continue;
                }
#pragma unroll 1
                for (int c0 = 16 * half; c0 < BN; c0 += 32) {
                    if (c0 >= valid) break;
                    uint32_t r[16];
                    tmem_ld16(t_row + c0, r);
                    // The columns' tokens and weights, read while the TMEM load is in flight.
                    int tok[16];
                    float w[16];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int4 t4 = reinterpret_cast<const int4*>(&s_ep_tok[iter & 1][c0])[q];
                        const float4 w4 = reinterpret_cast<const float4*>(&s_ep_w[iter & 1][c0])[q];
                        tok[4 * q] = t4.x;
                        tok[4 * q + 1] = t4.y;
                        tok[4 * q + 2] = t4.z;
                        tok[4 * q + 3] = t4.w;
                        w[4 * q] = w4.x;
                        w[4 * q + 1] = w4.y;
                        w[4 * q + 2] = w4.z;
                        w[4 * q + 3] = w4.w;
                    }
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (c0 + j < valid)
                            atomicAdd(args.y + static_cast<size_t>(tok[j]) * args.hidden + d, w[j] * __uint_as_float(r[j]));
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

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int BN, Kind KIND>
cudaError_t launch_one(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& x, const GemmArgs& args,
                       int sms, cudaStream_t stream, bool pdl) {
    using C = Cfg<BN, KIND>;
    auto kernel = moe_gemm_kernel<BN, KIND>;
    static std::atomic<uint64_t> configured{0};  // devices whose limit is raised
    if (const cudaError_t e = set_smem_limit_once(kernel, C::kSmemBytes, configured); e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, a, b, x, args);
}

}  // namespace

// Loads every instantiation launch_gemm_* can launch (see preload_kernels in moe_internal.h).
cudaError_t preload_grouped_gemm_kernels() {
    cudaFuncAttributes a{};
    const void* kernels[] = {
        reinterpret_cast<const void*>(moe_gemm_kernel<16, Kind::GateUp>),
        reinterpret_cast<const void*>(moe_gemm_kernel<32, Kind::GateUp>),
        reinterpret_cast<const void*>(moe_gemm_kernel<64, Kind::GateUp>),
        reinterpret_cast<const void*>(moe_gemm_kernel<128, Kind::GateUp>),
        reinterpret_cast<const void*>(moe_gemm_kernel<256, Kind::GateUp>),
        reinterpret_cast<const void*>(moe_gemm_kernel<16, Kind::Down>),
        reinterpret_cast<const void*>(moe_gemm_kernel<32, Kind::Down>),
        reinterpret_cast<const void*>(moe_gemm_kernel<64, Kind::Down>),
        reinterpret_cast<const void*>(moe_gemm_kernel<128, Kind::Down>),
        reinterpret_cast<const void*>(moe_gemm_kernel<256, Kind::Down>),
        reinterpret_cast<const void*>(moe_gemm_kernel<16, Kind::Router>),
        reinterpret_cast<const void*>(moe_gemm_kernel<32, Kind::Router>),
        reinterpret_cast<const void*>(moe_gemm_kernel<64, Kind::Router>),
        reinterpret_cast<const void*>(moe_gemm_kernel<128, Kind::Router>),
    };
    for (const void* k : kernels)
        if (const cudaError_t e = cudaFuncGetAttributes(&a, k); e != cudaSuccess) return e;
    return cudaSuccess;
}

cudaError_t launch_gemm_gate_up(int bn, const CUtensorMap& w13, const CUtensorMap& xperm, const CUtensorMap& x,
                                const GemmArgs& args, int sms, cudaStream_t stream, bool pdl) {
    switch (bn) {
        case 16: return launch_one<16, Kind::GateUp>(w13, xperm, x, args, sms, stream, pdl);
        case 32: return launch_one<32, Kind::GateUp>(w13, xperm, x, args, sms, stream, pdl);
        case 64: return launch_one<64, Kind::GateUp>(w13, xperm, x, args, sms, stream, pdl);
        case 128: return launch_one<128, Kind::GateUp>(w13, xperm, x, args, sms, stream, pdl);
        case 256: return launch_one<256, Kind::GateUp>(w13, xperm, x, args, sms, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm_router(int bn, const CUtensorMap& wcat, const CUtensorMap& x, const GemmArgs& args, int sms,
                               cudaStream_t stream, bool pdl) {
    const int tiles = (args.tokens + bn - 1) / bn;
    const int grid = tiles < sms ? tiles : sms;
    switch (bn) {
        case 16: return launch_one<16, Kind::Router>(wcat, x, x, args, grid, stream, pdl);
        case 32: return launch_one<32, Kind::Router>(wcat, x, x, args, grid, stream, pdl);
        case 64: return launch_one<64, Kind::Router>(wcat, x, x, args, grid, stream, pdl);
        case 128: return launch_one<128, Kind::Router>(wcat, x, x, args, grid, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm_down(int bn, const CUtensorMap& w2, const CUtensorMap& hmap, const GemmArgs& args, int sms,
                             cudaStream_t stream, bool pdl) {
    switch (bn) {
        case 16: return launch_one<16, Kind::Down>(w2, hmap, hmap, args, sms, stream, pdl);
        case 32: return launch_one<32, Kind::Down>(w2, hmap, hmap, args, sms, stream, pdl);
        case 64: return launch_one<64, Kind::Down>(w2, hmap, hmap, args, sms, stream, pdl);
        case 128: return launch_one<128, Kind::Down>(w2, hmap, hmap, args, sms, stream, pdl);
        case 256: return launch_one<256, Kind::Down>(w2, hmap, hmap, args, sms, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace lm
