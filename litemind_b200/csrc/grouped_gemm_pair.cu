// grouped_gemm_pair.cu -- the prefill form of the grouped SwiGLU GEMMs on CTA pairs.
//
// Same products as grouped_gemm.cu (gate/up with the SiLU epilogue, down with the
// weighted combine; weights on the MMA's M side, tokens on N), but each tile is
// 256 weight rows x 256 tokens computed by a cluster of two CTAs with
// tcgen05.mma.cta_group::2: each CTA loads its own 128 weight rows and half of the
// token rows, the pair's leader issues one M=256 MMA that reads both CTAs' shared
// memory, and each CTA's TMEM holds its 128 rows of the accumulator.  Per SM that is
// a third fewer operand bytes per FLOP than a 128 x 256 tile, which buys the deeper
// pipeline (5-6 stages) a compute-bound prefill needs.
//
// Synchronisation: every TMA load of either CTA completes on the leader's `full`
// barrier; the leader's MMA completion arrives on the `empty` / `tmem_full` barriers
// of both CTAs (one commit per CTA); each CTA's epilogue warps arrive on the
// leader's `tmem_empty`.  All waits are bounded (ptx.cuh); a cluster barrier keeps
// both CTAs alive until neither touches the other's shared memory or TMEM.
#include "moe_internal.h"
#include "ptx.cuh"
#include "gemm_rows.cuh"

#include <cuda_bf16.h>

namespace lm {
namespace {

constexpr int kRows = 128;  // weight rows per CTA (256 per pair)
constexpr int kBK = 64;
constexpr int kEpiThreads = 256;  // 8 epilogue warps: two per TMEM lane quadrant
constexpr int kThreads = 64 + kEpiThreads;  // + TMA producer warp, MMA warp
constexpr int kATile = kRows * kBK * 2;
constexpr int kBudget = 225 * 1024;

enum class PKind { GateUp, Down };

template <int BN, PKind KIND>
struct PCfg {
    static constexpr int kBHalf = BN / 2;  // token rows each CTA loads
    static constexpr int kBTile = kBHalf * kBK * 2;
    static constexpr int kStage = kATile + kBTile;
    static constexpr int kStaging = (KIND == PKind::GateUp) ? BN * 64 * 2 : 0;
    static constexpr int kBar = 1024;
    static constexpr int kStagesFit = (kBudget - kStaging - kBar - 1024) / kStage;
    static constexpr int kStages = kStagesFit > 10 ? 10 : kStagesFit;
    static constexpr int kTmemCols = 2 * BN;
    static constexpr int kSmem = 1024 + kStages * kStage + kStaging + kBar;
    static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
    static_assert((BN / 2) % 32 == 0, "epilogue warps drain 32 columns per TMEM wait");
    static_assert(kBTile % 1024 == 0, "token half-tiles must keep 1024-byte alignment");
    static_assert(kStages >= 3, "pipeline depth");
    static_assert(kSmem <= 220 * 1024, "shared memory");
};

__device__ __forceinline__ int find_segment(const int* tiles, int n_seg, int tile) {
    int lo = 0, hi = n_seg;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (tiles[mid] <= tile) lo = mid; else hi = mid;
    }
    return lo;
}

// silu(g) * u with fast exp and divide: the result is rounded to bf16 (8 bits).
__device__ __forceinline__ float silu_times(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

template <int BN, PKind KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ CUtensorMap map_x, const GemmArgs args) {
    using C = PCfg<BN, KIND>;
    constexpr int S = C::kStages;
    constexpr uint32_t kIdesc = umma_idesc_bf16(2 * kRows, BN);
    // A segment's last token block with at most BN/2 rows left runs at N = BN/2: the
    // tensor cores skip the padding (384 rows per expert are 256 + 128, not 2 x 256).
    constexpr uint32_t kIdescNarrow = umma_idesc_bf16(2 * kRows, BN / 2);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ int s_tiles[kMaxSegments + 1];
    __shared__ int s_off[kMaxSegments];
    __shared__ int s_cnt[kMaxSegments];
    __shared__ int s_wslot[kMaxSegments];
    __shared__ int s_n_seg;
    __shared__ int s_epi_go[2];
    constexpr int kMapCols = (KIND == PKind::Down) ? BN : 1;
    __shared__ __align__(16) int s_ep_tok[2][kMapCols];  // down epilogue: this tile's token and routing weight per column
    __shared__ __align__(16) float s_ep_w[2][kMapCols];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + S * kATile;
    uint8_t* staging = smem_b + S * C::kBTile;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C::kStaging);
    uint64_t* full = bars;                   // used in the leader
    uint64_t* empty = bars + S;              // both CTAs
    uint64_t* tmem_full = bars + 2 * S;      // both CTAs
    uint64_t* tmem_empty = bars + 2 * S + 2; // used in the leader: 8 epilogue warps x 2 CTAs
    uint64_t* drain_bar = bars + 2 * S + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int n_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], 16);  // 8 epilogue warps x 2 CTAs
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
        if (KIND == PKind::GateUp) tma_prefetch_desc(&map_x);
    }
    cluster_sync();  // both CTAs' barriers exist before either can signal the other's
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, C::kTmemCols);
        tmem_relinquish_pair();
    }
    pdl_wait();
    const Schedule* sched = args.sched;
    if (threadIdx.x == 0) s_n_seg = sched->n_seg;
    for (int i = threadIdx.x; i < kMaxSegments; i += kThreads) {
        s_off[i] = sched->seg_off[i];
        s_cnt[i] = sched->seg_cnt[i];
        s_wslot[i] = sched->seg_weight[i];
    }
    __syncthreads();
    const int rows_total = (KIND == PKind::GateUp) ? 2 * args.inter : args.hidden;
    const int mb_per = rows_total / (2 * kRows);     // 256-row blocks per segment
    const int tiles128_per = rows_total / kRows;     // 128-row tiles of the tile-major weights
    if (threadIdx.x == 0) {
        // Pair tiles per segment: ceil(rows / BN) token blocks x 256-row weight blocks.
        int p = 0;
        for (int s = 0; s < s_n_seg; ++s) {
            s_tiles[s] = p;
            p += ((s_cnt[s] + BN - 1) / BN) * mb_per;
        }
        s_tiles[s_n_seg] = p;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch_dependents();

    const int n_seg = s_n_seg;
    const int total_tiles = s_tiles[n_seg];
    const uint32_t tmem_base = *tmem_slot;
    const int K = (KIND == PKind::GateUp) ? args.hidden : args.inter;
    const int num_kb = K / kBK;

    if (warp == 0) {
        if (lane == 0) {
            // ── TMA producer (both CTAs): own A rows and own half of the token rows ──
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0;
            uint32_t issued_phase = 0;
            bool ok = true;
            for (int tile = pair; tile < total_tiles && ok; tile += n_pairs) {
                const int s = find_segment(s_tiles, n_seg, tile);
                const int local = tile - s_tiles[s];
                const int nb = local / mb_per;
                const int mb = local - nb * mb_per;
                const int a_tile0 = (s_wslot[s] * tiles128_per + 2 * mb + static_cast<int>(rank)) * num_kb;
                const bool from_x = (KIND == PKind::GateUp) && s >= args.n_routed_local;
                // Each CTA holds its half of the block's N token rows: BN/2 of them, or
                // BN/4 for a narrow last block (the box still loads BN/2; the MMA reads
                // the first BN/4 of them).
                const bool narrow = s_cnt[s] - nb * BN <= BN / 2;
                const int b_row = (from_x ? nb * BN : s_off[s] + nb * BN) +
                                  static_cast<int>(rank) * (narrow ? C::kBHalf / 2 : C::kBHalf);
                const CUtensorMap* bmap = from_x ? &map_x : &map_b;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, kDevTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (kATile + C::kBTile));
                    tma_load_2d_pair(smem_a + stage * kATile, &map_a, leader_full, 0, (a_tile0 + kb) * kRows);
                    tma_load_2d_pair(smem_b + stage * C::kBTile, bmap, leader_full, kb * kBK, b_row);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok && leader) {
                for (int st = 0; st < S; ++st)
                    if (issued_mask & (1u << st)) mbar_wait_drain(&full[st], (issued_phase >> st) & 1u, 100000000ull);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ── MMA issuer (leader only): M=256 across the pair ──
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            bool issued_any = false;
            for (int tile = pair; tile < total_tiles && ok; tile += n_pairs) {
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, args.status, kDevTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                const int seg = find_segment(s_tiles, n_seg, tile);
                const int nb = (tile - s_tiles[seg]) / mb_per;
                const uint32_t idesc = s_cnt[seg] - nb * BN <= BN / 2 ? kIdescNarrow : kIdesc;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, args.status, kDevTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = umma_desc_sw128(smem_u32(smem_a + stage * kATile));
                    const uint64_t b_desc = umma_desc_sw128(smem_u32(smem_b + stage * C::kBTile));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_bf16_pair(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0);
                    issued_any = true;
                    umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 0));
                    umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair(mapa_shared(smem_u32(&tmem_full[acc]), 0));
                umma_commit_pair(mapa_shared(smem_u32(&tmem_full[acc]), 1));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok && issued_any) {
                umma_commit_pair(mapa_shared(smem_u32(drain_bar), 0));
                mbar_wait_drain(drain_bar, 0, 100000000ull);
            }
        }
    } else {
        // ── Epilogue (both CTAs): this CTA's 128 accumulator rows ──
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;  // which half of the tile's columns this warp drains
        const int c_beg = half * (BN / 2);
        const int c_end = c_beg + BN / 2;
        const int epi_tid = threadIdx.x - 64;  // 0..255
        const uint32_t leader_tmem_empty0 = mapa_shared(smem_u32(&tmem_empty[0]), 0);
        const uint32_t leader_tmem_empty1 = mapa_shared(smem_u32(&tmem_empty[1]), 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        int iter = 0;
        for (int tile = pair; tile < total_tiles; tile += n_pairs, ++iter) {
            const int s = find_segment(s_tiles, n_seg, tile);
            const int local = tile - s_tiles[s];
            const int nb = local / mb_per;
            const int mb = local - nb * mb_per;
            const int valid = min(BN, s_cnt[s] - nb * BN);
            const int row0 = s_off[s] + nb * BN;
            if constexpr (KIND == PKind::Down) {
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
            if (epi_tid == 0)
                s_epi_go[iter & 1] =
                    mbar_wait(&tmem_full[acc], acc_phase, abort_flag, args.status, kDevTimeoutEpilogue) ? 1 : 0;
            named_bar_sync(2, kEpiThreads);
            if (!s_epi_go[iter & 1]) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
            const int block128 = 2 * mb + static_cast<int>(rank);  // this CTA's 128-row weight block
            const uint32_t release = acc == 0 ? leader_tmem_empty0 : leader_tmem_empty1;
            if constexpr (KIND == PKind::GateUp) {
                __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(staging);
                const int i_local = (quad * 32 + lane) >> 1;
                // 32 columns per TMEM wait: two loads in flight together.
#pragma unroll 1
                for (int c0 = c_beg; c0 < c_end; c0 += 32) {
                    if (c0 >= valid) break;
                    uint32_t r[32];
                    tmem_ld16(t_row + c0, *reinterpret_cast<uint32_t(*)[16]>(r));
                    tmem_ld16(t_row + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float mine = __uint_as_float(r[j]);
                        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
                        if ((lane & 1) == 0) st[(c0 + j) * 64 + i_local] = __float2bfloat16_rn(silu_times(mine, other));
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(release);
                named_bar_sync(1, kEpiThreads);
                const uint4* src = reinterpret_cast<const uint4*>(staging);
                for (int q = epi_tid; q < valid * 8; q += kEpiThreads) {
                    const int c = q >> 3;
                    const int part = q & 7;
                    uint4* dst = reinterpret_cast<uint4*>(args.h + static_cast<size_t>(row0 + c) * args.inter +
                                                          block128 * 64) + part;
                    *dst = src[c * 8 + part];
                }
                named_bar_sync(1, kEpiThreads);
            } else {
                const int d = block128 * kRows + quad * 32 + lane;
                const bool to_rows = s < args.n_routed_local && args.y_rows != nullptr;
                // 32 columns per TMEM wait; the columns' tokens and weights are read
                // from shared memory while the TMEM loads are in flight.
#pragma unroll 1
                for (int c0 = c_beg; c0 < c_end; c0 += 32) {
                    if (c0 >= valid) break;
                    uint32_t r[32];
                    tmem_ld16(t_row + c0, *reinterpret_cast<uint32_t(*)[16]>(r));
                    tmem_ld16(t_row + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
                    if (to_rows) {
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int c = c0 + j;
                            const int dst = c < valid ? y_row_dst(args, row0 + c) : -1;
                            if (dst >= 0)
                                reinterpret_cast<__nv_bfloat16*>(args.y_rows)[static_cast<size_t>(dst) * args.hidden +
                                                                              d] =
                                    __float2bfloat16_rn(__uint_as_float(r[j]));
                        }
                    } else {
                        int tok[32];
                        float w[32];
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
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
                        for (int j = 0; j < 32; ++j)
                            if (c0 + j < valid)
                                atomicAdd(args.y + static_cast<size_t>(tok[j]) * args.hidden + d,
                                          w[j] * __uint_as_float(r[j]));
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(release);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the other may still signal it or read its TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

template <int BN, PKind KIND>
cudaError_t launch_pair(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& x, const GemmArgs& args,
                        int sms, cudaStream_t stream, bool pdl) {
    using C = PCfg<BN, KIND>;
    auto kernel = moe_gemm_pair_kernel<BN, KIND>;
    static std::atomic<uint64_t> configured{0};  // devices whose limit is raised
    if (const cudaError_t e = set_smem_limit_once(kernel, C::kSmem, configured); e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms & ~1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, a, b, x, args);
}

}  // namespace

// Loads every instantiation launch_gemm_*_pair can launch (see preload_kernels in moe_internal.h).
cudaError_t preload_pair_gemm_kernels() {
    cudaFuncAttributes a{};
    const void* kernels[] = {
        reinterpret_cast<const void*>(moe_gemm_pair_kernel<128, PKind::GateUp>),
        reinterpret_cast<const void*>(moe_gemm_pair_kernel<256, PKind::GateUp>),
        reinterpret_cast<const void*>(moe_gemm_pair_kernel<128, PKind::Down>),
        reinterpret_cast<const void*>(moe_gemm_pair_kernel<256, PKind::Down>),
    };
    for (const void* k : kernels)
        if (const cudaError_t e = cudaFuncGetAttributes(&a, k); e != cudaSuccess) return e;
    return cudaSuccess;
}

cudaError_t launch_gemm_gate_up_pair(int bn, const CUtensorMap& w13, const CUtensorMap& xperm_half,
                                     const CUtensorMap& x_half, const GemmArgs& args, int sms, cudaStream_t stream,
                                     bool pdl) {
    switch (bn) {
        case 128: return launch_pair<128, PKind::GateUp>(w13, xperm_half, x_half, args, sms, stream, pdl);
        case 256: return launch_pair<256, PKind::GateUp>(w13, xperm_half, x_half, args, sms, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm_down_pair(int bn, const CUtensorMap& w2, const CUtensorMap& h_half, const GemmArgs& args,
                                  int sms, cudaStream_t stream, bool pdl) {
    switch (bn) {
        case 128: return launch_pair<128, PKind::Down>(w2, h_half, h_half, args, sms, stream, pdl);
        case 256: return launch_pair<256, PKind::Down>(w2, h_half, h_half, args, sms, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace lm
