// router.cu -- routing and dispatch kernels of the MoE path.
//
// The reference routes one token at a time: gemm::matvec_f32 for the router
// logits (src/Gemm.cpp:132-137), then MoeRouter::select (src/MoeRouter.cpp:54-107):
// softmax over every expert, optional group-limited masking, greedy top-k by
// (allowed, probability descending, index ascending), then normalise or scale.
// Here that is four kernels over all T tokens:
//   router_logits_*   logits[T, E] in f32 (+ optional per-expert bias)
//   router_topk       warp per token: softmax, group mask, top-k, weights, and the
//                     per-routing-tile expert histogram
//   dispatch_scan     one CTA: per-expert totals, segment offsets, each tile's
//                     first row per expert, and the grouped GEMMs' tile tables
//   permute           token rows copied into expert-sorted order (x_perm) with the
//                     row -> (token, weight) maps; stable in token order, so the
//                     permutation is deterministic.
#include "moe_internal.h"
#include "ptx.cuh"

#include <cfloat>

namespace lm {
namespace {

__device__ __forceinline__ void load8(const uint16_t* p, float (&v)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(words[i] << 16);
        v[2 * i + 1] = __uint_as_float(words[i] & 0xFFFF0000u);
    }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Small T: one warp per (token, group of 8 experts); lanes split the hidden axis.
template <typename XT>
__global__ void __launch_bounds__(256) router_logits_warp_kernel(const XT* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ bias,
                                                                 float* __restrict__ logits, int T, int H,
                                                                 int E) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int groups = (E + 7) >> 3;
    const int t = warp / groups;
    const int g = warp - t * groups;
    if (t >= T) return;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    const XT* xt = x + static_cast<size_t>(t) * H;
    for (int h = lane * 8; h < H; h += 256) {
        float xv[8];
        load8(xt + h, xv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = g * 8 + j;
            if (e < E) {
                float wv[8];
                load8(w + static_cast<size_t>(e) * H + h, wv);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[j] = fmaf(xv[i], wv[i], acc[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
    }
    if (lane < 8) {
        const int e = g * 8 + lane;
        float v = acc[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) v = (lane == j) ? acc[j] : v;
        if (e < E) logits[static_cast<size_t>(t) * E + e] = bias != nullptr ? v + bias[e] : v;
    }
}

// Large T: 64 tokens x 64 experts per CTA from smem tiles; w_t is the router
// transposed to [H, E] so expert vectors are contiguous.
template <typename XT>
__global__ void __launch_bounds__(256) router_logits_tiled_kernel(const XT* __restrict__ x,
                                                                  const float* __restrict__ w_t,
                                                                  const float* __restrict__ bias,
                                                                  float* __restrict__ logits, int T, int H,
                                                                  int E) {
    __shared__ __align__(16) float xs[32][68];  // [k][token]
    __shared__ __align__(16) float ws[32][68];  // [k][expert]
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * 64;
    const int e0 = blockIdx.y * 64;
    const int tx = tid & 15;  // expert quad
    const int ty = tid >> 4;  // token quad
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int k0 = 0; k0 < H; k0 += 32) {
        {   // x: 64 tokens x 32 k; each thread one 8-wide run of one token
            const int tl = tid >> 2;
            const int kp = (tid & 3) * 8;
            float v[8];
            if (t0 + tl < T) {
                load8(x + static_cast<size_t>(t0 + tl) * H + k0 + kp, v);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) xs[kp + i][tl] = v[i];
        }
        {   // w: 32 k x 64 experts; each thread 8 experts of one k
            const int kk = tid >> 3;
            const int ep = (tid & 7) * 8;
            const float* src = w_t + static_cast<size_t>(k0 + kk) * E + e0 + ep;
#pragma unroll
            for (int i = 0; i < 8; ++i) ws[kk][ep + i] = (e0 + ep + i < E) ? src[i] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < 32; ++kk) {
            const float4 xv = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
            const float4 wv = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
            const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + tx * 4 + j;
            if (e < E) logits[static_cast<size_t>(t) * E + e] = bias != nullptr ? acc[i][j] + bias[e] : acc[i][j];
        }
    }
}

// (allowed, probability, index) ordering of top_k_indices (src/MoeRouter.cpp:21-32).
__device__ __forceinline__ bool ranks_ahead(bool a_ok, float a_p, int a_i, bool b_ok, float b_p, int b_i) {
    if (b_i < 0) return a_i >= 0;
    if (a_i < 0) return false;
    if (a_ok != b_ok) return a_ok;
    if (a_p != b_p) return a_p > b_p;
    return a_i < b_i;
}

constexpr int kTopkWarps = 8;

__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int T, RouterParams rp,
                                                          int32_t* __restrict__ topk_idx,
                                                          float* __restrict__ topk_w,
                                                          int32_t* __restrict__ tile_counts) {
    __shared__ int counts[kMaxExperts];
    __shared__ float probs[kTopkWarps][kMaxExperts];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int E = rp.experts;
    const int K = rp.top_k;
    for (int e = tid; e < E; e += blockDim.x) counts[e] = 0;
    __syncthreads();
    pdl_wait();
    pdl_launch_dependents();

    const int t_begin = blockIdx.x * kRouteTile;
    const int t_end = min(T, t_begin + kRouteTile);
    for (int t = t_begin + warp; t < t_end; t += kTopkWarps) {
        float p[kMaxExperts / 32];
        uint32_t taken = 0u;  // bit j: expert lane + 32 j already selected
        float m = -FLT_MAX;
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; ++j) {
            const int e = lane + 32 * j;
            p[j] = (e < E) ? logits[static_cast<size_t>(t) * E + e] : -FLT_MAX;
            m = fmaxf(m, p[j]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        // Softmax over every expert before the cut (src/MoeRouter.cpp:61-64, src/Gemm.cpp:209-223).
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; ++j) {
            const int e = lane + 32 * j;
            p[j] = (e < E) ? expf(p[j] - m) : 0.0f;
            sum += p[j];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; ++j) p[j] *= inv;

        // Group-limited masking (src/MoeRouter.cpp:66-84): keep the topk_group groups
        // whose best probability ranks highest.
        uint32_t group_mask = 0xffffffffu;
        int per_group = E;
        if (rp.group_limited && rp.n_group > 1) {
            per_group = E / rp.n_group;
#pragma unroll
            for (int j = 0; j < kMaxExperts / 32; ++j) {
                const int e = lane + 32 * j;
                if (e < E) probs[warp][e] = p[j];
            }
            __syncwarp();
            float gbest = -FLT_MAX;
            int gi = -1;
            if (lane < rp.n_group) {
                gi = lane;
                gbest = probs[warp][lane * per_group];
                for (int o = 1; o < per_group; ++o) gbest = fmaxf(gbest, probs[warp][lane * per_group + o]);
            }
            __syncwarp();
            group_mask = 0u;
            const int keep = min(rp.topk_group, rp.n_group);
            bool g_taken = false;
            for (int r = 0; r < keep; ++r) {
                float bp = (!g_taken && gi >= 0) ? gbest : -FLT_MAX;
                int bi = (!g_taken && gi >= 0) ? gi : -1;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const float op = __shfl_xor_sync(0xffffffffu, bp, off);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                    if (ranks_ahead(true, op, oi, true, bp, bi)) {
                        bp = op;
                        bi = oi;
                    }
                }
                if (bi >= 0) {
                    group_mask |= 1u << bi;
                    if (bi == gi) g_taken = true;
                }
            }
        }

        // Greedy top-k, lower index first on equal probability.
        int my_idx = -1;
        float my_p = 0.0f;
        for (int s = 0; s < K; ++s) {
            bool b_ok = false;
            float b_p = -FLT_MAX;
            int b_i = -1;
#pragma unroll
            for (int j = 0; j < kMaxExperts / 32; ++j) {
                const int e = lane + 32 * j;
                if (e < E && !((taken >> j) & 1u)) {
                    const bool ok = (group_mask >> (e / per_group)) & 1u;
                    if (ranks_ahead(ok, p[j], e, b_ok, b_p, b_i)) {
                        b_ok = ok;
                        b_p = p[j];
                        b_i = e;
                    }
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const bool o_ok = __shfl_xor_sync(0xffffffffu, static_cast<int>(b_ok), off) != 0;
                const float o_p = __shfl_xor_sync(0xffffffffu, b_p, off);
                const int o_i = __shfl_xor_sync(0xffffffffu, b_i, off);
                if (ranks_ahead(o_ok, o_p, o_i, b_ok, b_p, b_i)) {
                    b_ok = o_ok;
                    b_p = o_p;
                    b_i = o_i;
                }
            }
            if (b_i >= 0 && (b_i & 31) == lane) taken |= 1u << (b_i >> 5);
            if (lane == s) {
                my_idx = b_i;
                my_p = b_p;
            }
        }
        // Normalise or scale, never both (src/MoeRouter.cpp:96-106).  The sum runs
        // in selection order, as the reference's does.
        float w = my_p;
        if (K > 1 && rp.normalize) {
            float selected = 0.0f;
            for (int s = 0; s < K; ++s) selected += __shfl_sync(0xffffffffu, my_p, s);
            w = my_p / (selected + 1e-20f);
        } else if (rp.scale != 1.0f) {
            w = my_p * rp.scale;
        }
        if (lane < K) {
            topk_idx[static_cast<size_t>(t) * K + lane] = my_idx;
            topk_w[static_cast<size_t>(t) * K + lane] = w;
            if (tile_counts != nullptr && my_idx >= 0) atomicAdd(&counts[my_idx], 1);
        }
    }
    if (tile_counts != nullptr) {
        __syncthreads();
        for (int e = tid; e < E; e += blockDim.x) tile_counts[static_cast<size_t>(blockIdx.x) * E + e] = counts[e];
    }
}

constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kScanThreads) dispatch_scan_kernel(const int32_t* __restrict__ tile_counts,
                                                                     int32_t* __restrict__ tile_base,
                                                                     int32_t* __restrict__ expert_totals,
                                                                     Schedule* __restrict__ sched, int T, int K,
                                                                     int E, int n_shared, int first_expert,
                                                                     int local_E, int shared_base, int bn,
                                                                     int mb1, int mb2) {
    __shared__ int part_sum[kScanThreads];
    __shared__ int seg_off_s[kMaxExperts];
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x;
    const int nt = (T + kRouteTile - 1) / kRouteTile;
    const int parts = max(1, kScanThreads / E);
    const int chunk = (nt + parts - 1) / parts;
    const int e = tid % E;
    const int part = tid / E;
    const bool active = part < parts;
    int lo = 0, hi = 0;
    if (active) {
        lo = min(nt, part * chunk);
        hi = min(nt, lo + chunk);
        int s = 0;
        for (int t = lo; t < hi; ++t) s += tile_counts[static_cast<size_t>(t) * E + e];
        part_sum[part * E + e] = s;
    }
    __syncthreads();
    if (tid < E) {  // exclusive scan over parts, per expert
        int run = 0;
        for (int q = 0; q < parts; ++q) {
            const int v = part_sum[q * E + tid];
            part_sum[q * E + tid] = run;
            run += v;
        }
        expert_totals[tid] = run;
        seg_off_s[tid] = run;  // total for now
    }
    __syncthreads();
    if (tid == 0) {
        int off = 0;
        for (int s = 0; s < local_E; ++s) {
            const int total = seg_off_s[first_expert + s];
            sched->seg_off[s] = off;
            sched->seg_cnt[s] = total;
            off += total;
        }
        for (int s = 0; s < n_shared; ++s) {
            sched->seg_off[local_E + s] = shared_base + s * T;
            sched->seg_cnt[local_E + s] = T;
        }
        const int n_seg = local_E + n_shared;
        int p1 = 0, p2 = 0;
        for (int s = 0; s < n_seg; ++s) {
            const int nb = (sched->seg_cnt[s] + bn - 1) / bn;
            sched->tiles1[s] = p1;
            sched->tiles2[s] = p2;
            p1 += nb * mb1;
            p2 += nb * mb2;
        }
        sched->tiles1[n_seg] = p1;
        sched->tiles2[n_seg] = p2;
        sched->n_seg = n_seg;
        sched->first_expert = first_expert;
        for (int s = 0; s < local_E; ++s) seg_off_s[first_expert + s] = sched->seg_off[s];
    }
    __syncthreads();
    if (active) {
        const bool local = e >= first_expert && e < first_expert + local_E;
        int run = part_sum[part * E + e] + (local ? seg_off_s[e] : 0);
        for (int t = lo; t < hi; ++t) {
            const size_t at = static_cast<size_t>(t) * E + e;
            const int c = tile_counts[at];
            tile_base[at] = run;
            run += c;
        }
    }
}

__global__ void __launch_bounds__(256) permute_kernel(const uint16_t* __restrict__ x,
                                                      const int32_t* __restrict__ topk_idx,
                                                      const float* __restrict__ topk_w,
                                                      const int32_t* __restrict__ tile_base, int T, int H, int K,
                                                      int E, int first_expert, int local_E,
                                                      int32_t* __restrict__ row_token,
                                                      float* __restrict__ row_weight,
                                                      int32_t* __restrict__ slot_row,
                                                      uint16_t* __restrict__ x_perm) {
    __shared__ int s_idx[kRouteTile * kMaxTopK];
    __shared__ int s_row[kRouteTile * kMaxTopK];
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x;
    const int tile = blockIdx.x;
    const int t0 = tile * kRouteTile;
    const int n_tok = min(kRouteTile, T - t0);
    const int n_pairs = n_tok * K;
    for (int q = tid; q < n_pairs; q += blockDim.x) {
        s_idx[q] = topk_idx[static_cast<size_t>(t0) * K + q];
        s_row[q] = -1;
    }
    __syncthreads();
    // Each local expert walks the tile in (token, slot) order: stable placement.
    for (int e = first_expert + tid; e < first_expert + local_E; e += blockDim.x) {
        int run = tile_base[static_cast<size_t>(tile) * E + e];
        for (int q = 0; q < n_pairs; ++q) {
            if (s_idx[q] == e) s_row[q] = run++;
        }
    }
    __syncthreads();
    if (blockIdx.y == 0) {
        for (int q = tid; q < n_pairs; q += blockDim.x) {
            const int row = s_row[q];
            const size_t slot = static_cast<size_t>(t0) * K + q;
            if (slot_row != nullptr) slot_row[slot] = row;
            if (row >= 0) {
                row_token[row] = t0 + q / K;
                row_weight[row] = topk_w[slot];
            }
        }
    }
    // Copy token rows to their expert-sorted positions, 16 bytes per thread,
    // four loads in flight before the stores.
    const int vec_per_row = H / 8;
    const int64_t total = static_cast<int64_t>(n_pairs) * vec_per_row;
    const int64_t stride = static_cast<int64_t>(blockDim.x) * gridDim.y;
    const uint4* src = reinterpret_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(x_perm);
    for (int64_t i = static_cast<int64_t>(blockIdx.y) * blockDim.x + tid; i < total; i += 4 * stride) {
        uint4 v[4];
        int64_t d[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t j = i + u * stride;
            d[u] = -1;
            if (j < total) {
                const int q = static_cast<int>(j / vec_per_row);
                const int c = static_cast<int>(j - static_cast<int64_t>(q) * vec_per_row);
                const int row = s_row[q];
                if (row >= 0) {
                    v[u] = src[static_cast<size_t>(t0 + q / K) * vec_per_row + c];
                    d[u] = static_cast<int64_t>(row) * vec_per_row + c;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (d[u] >= 0) dst[d[u]] = v[u];
    }
}

template <typename Kernel, typename... Args>
cudaError_t launch_k(Kernel kernel, dim3 grid, dim3 block, cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

cudaError_t launch_router_logits(const uint16_t* x, const float* x_f32, const float* w, const float* w_t,
                                 const float* bias, float* logits, int tokens, int hidden, int experts,
                                 cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    if (tokens >= 2048) {
        const dim3 grid((tokens + 63) / 64, (experts + 63) / 64);
        if (x_f32 != nullptr)
            return launch_k(router_logits_tiled_kernel<float>, grid, dim3(256), stream, pdl, x_f32, w_t, bias,
                            logits, tokens, hidden, experts);
        return launch_k(router_logits_tiled_kernel<uint16_t>, grid, dim3(256), stream, pdl, x, w_t, bias, logits,
                        tokens, hidden, experts);
    }
    const int groups = (experts + 7) / 8;
    const long warps = static_cast<long>(tokens) * groups;
    const dim3 grid(static_cast<unsigned>((warps + 7) / 8));
    if (x_f32 != nullptr)
        return launch_k(router_logits_warp_kernel<float>, grid, dim3(256), stream, pdl, x_f32, w, bias, logits,
                        tokens, hidden, experts);
    return launch_k(router_logits_warp_kernel<uint16_t>, grid, dim3(256), stream, pdl, x, w, bias, logits, tokens,
                    hidden, experts);
}

cudaError_t launch_router_topk(const float* logits, int tokens, RouterParams rp, int32_t* topk_idx,
                               float* topk_w, int32_t* tile_counts, cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    const dim3 grid((tokens + kRouteTile - 1) / kRouteTile);
    return launch_k(router_topk_kernel, grid, dim3(kTopkWarps * 32), stream, pdl, logits, tokens, rp, topk_idx,
                    topk_w, tile_counts);
}

cudaError_t launch_dispatch_scan(const int32_t* tile_counts, int32_t* tile_base, int32_t* expert_totals,
                                 Schedule* sched, int tokens, int top_k, int experts, int n_shared,
                                 int first_expert, int local_experts, int shared_base, int bn, int mb1,
                                 int mb2, cudaStream_t stream, bool pdl) {
    return launch_k(dispatch_scan_kernel, dim3(1), dim3(kScanThreads), stream, pdl, tile_counts, tile_base,
                    expert_totals, sched, tokens, top_k, experts, n_shared, first_expert, local_experts,
                    shared_base, bn, mb1, mb2);
}

cudaError_t launch_permute(const uint16_t* x, const int32_t* topk_idx, const float* topk_w,
                           const int32_t* tile_base, int tokens, int hidden, int top_k, int experts,
                           int first_expert, int local_experts, int32_t* row_token, float* row_weight,
                           int32_t* slot_row, uint16_t* x_perm, cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    const int tiles = (tokens + kRouteTile - 1) / kRouteTile;
    // Enough CTAs to keep the row copies bandwidth-bound at small T.
    const int split = tiles >= 128 ? 1 : min(16, (256 + tiles - 1) / tiles);
    return launch_k(permute_kernel, dim3(tiles, split), dim3(256), stream, pdl, x, topk_idx, topk_w, tile_base,
                    tokens, hidden, top_k, experts, first_expert, local_experts, row_token, row_weight,
                    slot_row, x_perm);
}

}  // namespace lm
