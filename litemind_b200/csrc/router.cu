// router.cu -- routing and dispatch kernels of the MoE path.
//
// The reference routes one token at a time: gemm::matvec_f32 for the router
// logits (src/Gemm.cpp:132-137), then MoeRouter::select (src/MoeRouter.cpp:54-107):
// softmax over every expert, optional group-limited masking, greedy top-k by
// (allowed, probability descending, index ascending), then normalise or scale.
// Here, for T tokens at once:
//   route_small       T <= 32 (decode): the whole stage below in one launch
//   router_logits_*   logits[T, E] in f32 (+ optional per-expert bias)
//   router_topk       warp per token: softmax, group mask, top-k, weights, and the
//                     per-routing-tile expert histogram
//   dispatch_scan     one CTA: per-expert totals, segment offsets, each tile's
//                     first row per expert, and the grouped GEMMs' tile tables
//   place             the row -> (token, weight) maps of the expert-sorted order,
//                     stable in token order, so the permutation is deterministic.
//   gather_rows       x_perm[r] = x[row_token[r]]: token rows in expert-sorted order,
//                     so each expert's token tile is one contiguous TMA load.
#include "moe_internal.h"
#include "ptx.cuh"
#include "route_device.cuh"

#include <algorithm>
#include <cfloat>

namespace lm {
namespace {

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
// transposed to [H, E] so expert vectors are contiguous.  The hidden axis is split
// over blockIdx.z (k_per elements each) so the grid fills the GPU; with more than
// one split each CTA writes its partial sums to partial[z][t][e] and
// router_logits_reduce adds them in z order (deterministic).
template <typename XT>
__global__ void __launch_bounds__(256) router_logits_tiled_kernel(const XT* __restrict__ x,
                                                                  const float* __restrict__ w_t,
                                                                  const float* __restrict__ bias,
                                                                  float* __restrict__ logits, int T, int H,
                                                                  int E, int k_per, float* __restrict__ partial) {
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

    const int k_begin = blockIdx.z * k_per;
    const int k_end = min(H, k_begin + k_per);
    for (int k0 = k_begin; k0 < k_end; k0 += 32) {
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
            if (e >= E) continue;
            if (partial != nullptr)
                partial[(static_cast<size_t>(blockIdx.z) * T + t) * E + e] = acc[i][j];
            else
                logits[static_cast<size_t>(t) * E + e] = bias != nullptr ? acc[i][j] + bias[e] : acc[i][j];
        }
    }
}

__global__ void __launch_bounds__(256) router_logits_reduce_kernel(const float* __restrict__ partial,
                                                                   const float* __restrict__ bias,
                                                                   float* __restrict__ logits, int T, int E,
                                                                   int splits) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t n = static_cast<int64_t>(T) * E;
    if (i >= n) return;
    float v = 0.0f;
    for (int z = 0; z < splits; ++z) v += partial[z * n + i];
    logits[i] = bias != nullptr ? v + bias[i % E] : v;
}

// Thread 0: segment offsets, counts and both GEMMs' tile prefixes from per-expert
// totals (`totals` in shared memory, global expert index).  Everything is computed
// in registers and only written to global memory, never read back.
__device__ void build_schedule(Schedule* sched, const int* totals, int T, int n_shared, int first_expert,
                               int local_E, int shared_base, int bn, int mb1, int mb2, int* seg_off_out) {
    const int n_seg = local_E + n_shared;
    int off = 0, p1 = 0, p2 = 0;
    for (int s = 0; s < n_seg; ++s) {
        int seg_off, cnt;
        if (s < local_E) {
            cnt = totals[first_expert + s];
            seg_off = off;
            if (seg_off_out != nullptr) seg_off_out[first_expert + s] = off;
            off += cnt;
        } else {
            cnt = T;
            seg_off = shared_base + (s - local_E) * T;
        }
        sched->seg_off[s] = seg_off;
        sched->seg_cnt[s] = cnt;
        sched->seg_weight[s] = s;
        sched->tiles1[s] = p1;
        sched->tiles2[s] = p2;
        const int nb = (cnt + bn - 1) / bn;
        p1 += nb * mb1;
        p2 += nb * mb2;
    }
    sched->tiles1[n_seg] = p1;
    sched->tiles2[n_seg] = p2;
    sched->n_seg = n_seg;
    sched->first_expert = first_expert;
}

constexpr int kTopkThreads = 32 * kRouteTile;  // one warp per token of a routing tile

template <int EPL>
__global__ void __launch_bounds__(kTopkThreads) router_topk_kernel(float* __restrict__ logits, int T, RouterParams rp,
                                                                   int32_t* __restrict__ topk_idx,
                                                                   float* __restrict__ topk_w,
                                                                   int32_t* __restrict__ tile_counts,
                                                                   RouterFix fix) {
    __shared__ int counts[kMaxExperts];
    __shared__ float probs[kRouteTile][kMaxExperts];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int E = rp.experts;
    const int K = rp.top_k;
    for (int e = tid; e < E; e += blockDim.x) counts[e] = 0;
    __syncthreads();
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x * kRouteTile + warp;
    if (t < T) {
        float* lg = logits + static_cast<size_t>(t) * E;
        Selection sel = route_one_token<EPL>(lg, rp, probs[warp], lane, fix.x != nullptr ? fix.margin : 0.0f);
        if (sel.ambiguous) {
            // The logits came from the tensor cores, whose f32 accumulation is
            // coarser than a CUDA-core f32 sum.  Probability order is logit order, so
            // only the experts around the cut can change the choice: recompute the
            // logits of the k+4 best-ranked experts as plain f32 dot products (lanes
            // split the hidden axis) and route again.
            RouterParams rank_rp = rp;
            rank_rp.top_k = min(E, K + 4);
            rank_rp.normalize = 0;
            rank_rp.scale = 1.0f;
            const Selection ranked = route_one_token<EPL>(lg, rank_rp, probs[warp], lane, 0.0f);
            const uint16_t* xt = fix.x + static_cast<size_t>(t) * fix.hidden;
            // kBatch experts share each pass over the hidden axis (each x chunk loaded
            // once for all of them): a pass is a chain of dependent load rounds, and one
            // ambiguous token decides when the whole launch ends.  Each dot product is
            // summed in the same order as one at a time.
            constexpr int kBatch = 2;
            const int nr = rank_rp.top_k;
            for (int r0 = 0; r0 < nr; r0 += kBatch) {
                int e[kBatch];
                const float* wr[kBatch];
                float acc[kBatch];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    e[j] = __shfl_sync(kFull, ranked.idx, min(r0 + j, nr - 1));  // past nr: recomputed, unused
                    wr[j] = fix.w + static_cast<size_t>(e[j]) * fix.hidden;
                    acc[j] = 0.0f;
                }
                for (int h = lane * 8; h < fix.hidden; h += 256) {
                    float xv[8];
                    load8(xt + h, xv);
#pragma unroll
                    for (int j = 0; j < kBatch; ++j) {
                        float wv[8];
                        load8(wr[j] + h, wv);
#pragma unroll
                        for (int i = 0; i < 8; ++i) acc[j] = fmaf(xv[i], wv[i], acc[j]);
                    }
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(kFull, acc[j], off);
                    if (lane == 0 && r0 + j < nr) lg[e[j]] = fix.bias != nullptr ? acc[j] + fix.bias[e[j]] : acc[j];
                }
            }
            __syncwarp();
            sel = route_one_token<EPL>(lg, rp, probs[warp], lane, 0.0f);
        }
        if (lane < K) {
            topk_idx[static_cast<size_t>(t) * K + lane] = sel.idx;
            topk_w[static_cast<size_t>(t) * K + lane] = sel.w;
            if (tile_counts != nullptr) atomicAdd(&counts[sel.idx], 1);
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
    __shared__ int totals[kMaxExperts];
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
        totals[tid] = run;
        seg_off_s[tid] = 0;
    }
    __syncthreads();
    if (tid == 0) build_schedule(sched, totals, T, n_shared, first_expert, local_E, shared_base, bn, mb1, mb2, seg_off_s);
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

// Permutation maps for one routing tile: each local expert walks the tile in
// (token, slot) order, so rows are stable in token order and the placement is
// deterministic.  Also zeroes the tile's rows of y when asked (the combine adds),
// and, when x_perm is given, copies each token's row to its expert-sorted places
// (the row gather, reading each token once).
__global__ void __launch_bounds__(256) place_kernel(const int32_t* __restrict__ topk_idx,
                                                    const float* __restrict__ topk_w,
                                                    const int32_t* __restrict__ tile_base, int T, int H, int K, int E,
                                                    int first_expert, int local_E, int32_t* __restrict__ row_token,
                                                    float* __restrict__ row_weight, int32_t* __restrict__ slot_row,
                                                    float* __restrict__ y_zero, const uint16_t* __restrict__ x,
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
    if (y_zero != nullptr) {
        float4* yz = reinterpret_cast<float4*>(y_zero + static_cast<size_t>(t0) * H);
        const int n4 = n_tok * H / 4;
        for (int i = tid; i < n4; i += blockDim.x) yz[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int q = tid; q < n_pairs; q += blockDim.x) {
        s_idx[q] = topk_idx[static_cast<size_t>(t0) * K + q];
        s_row[q] = -1;
    }
    __syncthreads();
    for (int e = first_expert + tid; e < first_expert + local_E; e += blockDim.x) {
        int run = tile_base[static_cast<size_t>(tile) * E + e];
        for (int q = 0; q < n_pairs; ++q) {
            if (s_idx[q] == e) s_row[q] = run++;
        }
    }
    __syncthreads();
    for (int q = tid; q < n_pairs; q += blockDim.x) {
        const int row = s_row[q];
        const size_t slot = static_cast<size_t>(t0) * K + q;
        if (slot_row != nullptr) slot_row[slot] = row;
        if (row >= 0) {
            row_token[row] = t0 + q / K;
            row_weight[row] = topk_w[slot];
        }
    }
    if (x_perm == nullptr) return;
    // One warp per token: its row is read once and written to each of its rows.
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int vec = H / 8;
    for (int tl = warp; tl < n_tok; tl += blockDim.x >> 5) {
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + tl) * H);
        for (int v0 = 0; v0 < vec; v0 += 128) {
            uint4 r[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (v0 + u * 32 + lane < vec) r[u] = src[v0 + u * 32 + lane];
            for (int k = 0; k < K; ++k) {
                const int row = s_row[tl * K + k];
                if (row < 0) continue;
                uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<size_t>(row) * H);
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (v0 + u * 32 + lane < vec) dst[v0 + u * 32 + lane] = r[u];
            }
        }
    }
}

// x_perm[r] = x[row_token[r]] for the routed rows, 16 bytes per thread with four
// loads in flight.
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ row_token, int rows, int H,
                                                          uint16_t* __restrict__ x_perm) {
    pdl_wait();
    pdl_launch_dependents();
    const int vec = H / 8;
    const int64_t total = static_cast<int64_t>(rows) * vec;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uint4* src = reinterpret_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(x_perm);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t j = i + u * stride;
            if (j < total) {
                const int r = static_cast<int>(j / vec);
                v[u] = src[static_cast<int64_t>(row_token[r]) * vec + (j - static_cast<int64_t>(r) * vec)];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t j = i + u * stride;
            if (j < total) dst[j] = v[u];
        }
    }
}

// Expert-parallel combine: y[t] += sum over slots s (in selection order) of
// w[t, s] * back[slot_row[t, s]], where `back` holds the expert outputs returned
// by the experts' ranks in this rank's send order, rounded to bf16 for the return
// trip (half the NVLink bytes; the weighted sum is in f32).  y already holds the
// shared experts' output.  One thread per 4 consecutive hidden elements of a token.
__global__ void __launch_bounds__(256) ep_combine_kernel(float* __restrict__ y, const uint16_t* __restrict__ back,
                                                         const int32_t* __restrict__ slot_row,
                                                         const float* __restrict__ topk_w, int T, int K, int H) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int per_token = H / 4;
    if (i >= static_cast<int64_t>(T) * per_token) return;
    const int t = static_cast<int>(i / per_token);
    const int c = static_cast<int>(i - static_cast<int64_t>(t) * per_token);
    float4 acc = reinterpret_cast<float4*>(y + static_cast<size_t>(t) * H)[c];
    for (int s = 0; s < K; ++s) {
        const int row = slot_row[t * K + s];
        const float w = topk_w[t * K + s];
        const uint2 b = reinterpret_cast<const uint2*>(back + static_cast<size_t>(row) * H)[c];
        acc.x = fmaf(w, __uint_as_float(b.x << 16), acc.x);
        acc.y = fmaf(w, __uint_as_float(b.x & 0xFFFF0000u), acc.y);
        acc.z = fmaf(w, __uint_as_float(b.y << 16), acc.z);
        acc.w = fmaf(w, __uint_as_float(b.y & 0xFFFF0000u), acc.w);
    }
    reinterpret_cast<float4*>(y + static_cast<size_t>(t) * H)[c] = acc;
}

// Expert parallelism: received rows arrive grouped by source rank, each source's
// rows grouped by this rank's experts.  The grouped GEMMs want each expert's rows
// contiguous, so each expert's weights stream once instead of once per source.
// Block (b, y) with b = (source r, local expert e) copies rows [16 y, 16 y + 16) of
// its group to their expert-major place and records where each came from, so the
// down projection can store its output rows back in receive order.  The copy is
// bound by the bytes in flight: each thread issues kSortUnroll 16-byte loads before
// their stores, and the small blocks give several CTAs per SM (64-row blocks with one
// load in flight per thread reached 17% of the DRAM bandwidth).
//
// A pipelined exchange moves the local experts in chunks [e_lo, e_hi): the receive
// buffer is chunk-major (all rows of earlier chunks first), source-major within a
// chunk.  One launch sorts one chunk; the whole range [0, El) is the unchunked
// source-major layout.  The expert-major destination does not depend on chunking.
constexpr int kSortRows = 16;
constexpr int kSortUnroll = 4;
// src_stride > 0: each source's rows sit in a fixed block of src_stride rows
// (the fixed-capacity exchange, one chunk) instead of back to back.
__global__ void __launch_bounds__(256) ep_sort_rows_kernel(const uint16_t* __restrict__ x_recv,
                                                           uint16_t* __restrict__ x_sorted,
                                                           int32_t* __restrict__ row_src,
                                                           const int32_t* __restrict__ recv_counts, int N, int El,
                                                           int H, int src_stride, int e_lo, int e_hi) {
    pdl_wait();
    pdl_launch_dependents();
    const int ne = e_hi - e_lo;
    const int r = blockIdx.x / ne;
    const int e = e_lo + (blockIdx.x - r * ne);
    __shared__ int s_src, s_dst, s_cnt;
    if (threadIdx.x < 32) {
        // The group's place in the receive buffer and in expert-major order: sums of
        // the (source, expert) counts before it, over the first warp.
        int src = 0, dst = 0;
        for (int i = threadIdx.x; i < N * El; i += 32) {
            const int rr = i / El, ee = i - rr * El;
            const int c = recv_counts[i];
            const bool before = src_stride > 0
                                    ? (rr == r && ee < e)
                                    : (ee < e_lo || (ee < e_hi && (rr < r || (rr == r && ee < e))));
            if (before) src += c;  // chunk-major, then source-major position
            if (ee < e || (ee == e && rr < r)) dst += c;  // expert-major position
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            src += __shfl_xor_sync(0xffffffffu, src, d);
            dst += __shfl_xor_sync(0xffffffffu, dst, d);
        }
        if (threadIdx.x == 0) {
            s_src = (src_stride > 0 ? r * src_stride : 0) + src;
            s_dst = dst;
            s_cnt = recv_counts[r * El + e];
        }
    }
    __syncthreads();
    const int vec = H / 8;
    const int nt = static_cast<int>(blockDim.x);
    // Row blocks y, y + gridDim.y, ... (the grid's y extent is capped).
    for (int j0 = blockIdx.y * kSortRows; j0 < s_cnt; j0 += gridDim.y * kSortRows) {
        const int rows = min(kSortRows, s_cnt - j0);
        const uint4* src = reinterpret_cast<const uint4*>(x_recv) + static_cast<size_t>(s_src + j0) * vec;
        uint4* dst = reinterpret_cast<uint4*>(x_sorted) + static_cast<size_t>(s_dst + j0) * vec;
        const int n = rows * vec;
        for (int base = threadIdx.x; base < n; base += nt * kSortUnroll) {
            uint4 v[kSortUnroll];
#pragma unroll
            for (int u = 0; u < kSortUnroll; ++u)
                if (base + u * nt < n) v[u] = __ldcs(src + base + u * nt);  // read once
#pragma unroll
            for (int u = 0; u < kSortUnroll; ++u)
                if (base + u * nt < n) dst[base + u * nt] = v[u];
        }
        for (int j = threadIdx.x; j < rows; j += nt) row_src[s_dst + j0 + j] = s_src + j0 + j;
    }
}

// Small T (<= kRouteTile): the whole routing stage in one launch.  CTA b computes
// expert b's logit for every token (one warp per token) and zeroes a slice of y;
// the last CTA to finish (an atomic ticket) routes every token (again one warp per
// token), counts the experts, builds the schedule and the permutation maps, and
// re-arms the ticket.
constexpr int kSmallExperts = 1;  // experts per CTA in the logits phase
constexpr int kSmallThreads = 1024;  // one warp per token of the tile in the routing step

template <typename XT, int EPL>
__global__ void __launch_bounds__(kSmallThreads) route_small_kernel(
    const XT* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias, float* __restrict__ logits,
    int T, int H, RouterParams rp, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
    int32_t* __restrict__ expert_totals, Schedule* __restrict__ sched, int32_t* __restrict__ row_token,
    float* __restrict__ row_weight, int32_t* __restrict__ slot_row, float* __restrict__ y_zero,
    unsigned int* __restrict__ ticket, int n_shared, int first_expert, int local_E, int shared_base, int bn, int mb1,
    int mb2) {
    __shared__ float probs[kSmallThreads / 32][kMaxExperts];
    __shared__ int s_idx[kRouteTile * kMaxTopK];
    __shared__ float s_w[kRouteTile * kMaxTopK];
    __shared__ int totals[kMaxExperts];
    __shared__ int seg_off_s[kMaxExperts];
    __shared__ int s_last;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    constexpr int kWarps = kSmallThreads / 32;
    const int E = rp.experts;
    const int K = rp.top_k;
    pdl_wait();
    pdl_launch_dependents();

    if (y_zero != nullptr) {  // y is accumulated into by the down GEMM
        const int n4 = T * H / 4;
        const int per = (n4 + gridDim.x - 1) / gridDim.x;
        float4* yz = reinterpret_cast<float4*>(y_zero);
        for (int i = blockIdx.x * per + tid; i < min(n4, (blockIdx.x + 1) * per); i += blockDim.x)
            yz[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // Logits of this CTA's expert(s): warp t computes token t's dot products; the
    // loop is unrolled so each lane's loads of x and of the router row are all in
    // flight together (one memory round trip instead of H / 256).
    const int e0 = blockIdx.x * kSmallExperts;
    for (int t = warp; t < T; t += kWarps) {
        float acc[kSmallExperts];
#pragma unroll
        for (int j = 0; j < kSmallExperts; ++j) acc[j] = 0.0f;
        const XT* xt = x + static_cast<size_t>(t) * H;
#pragma unroll 8
        for (int h = lane * 8; h < H; h += 256) {
            float xv[8];
            load8(xt + h, xv);
#pragma unroll
            for (int j = 0; j < kSmallExperts; ++j) {
                if (e0 + j < E) {
                    float wv[8];
                    load8(w + static_cast<size_t>(e0 + j) * H + h, wv);
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[j] = fmaf(xv[i], wv[i], acc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kSmallExperts; ++j) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(kFull, acc[j], off);
        }
        if (lane < kSmallExperts && e0 + lane < E) {
            float v = acc[0];
#pragma unroll
            for (int j = 1; j < kSmallExperts; ++j) v = (lane == j) ? acc[j] : v;
            logits[static_cast<size_t>(t) * E + e0 + lane] = bias != nullptr ? v + bias[e0 + lane] : v;
        }
    }

    // Last CTA in: route, count, schedule, place.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(ticket, 1u) == gridDim.x - 1) ? 1 : 0;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int e = tid; e < E; e += blockDim.x) {
        totals[e] = 0;
        seg_off_s[e] = 0;
    }
    __syncthreads();
    for (int t = warp; t < T; t += kWarps) {
        const Selection sel = route_one_token<EPL>(logits + static_cast<size_t>(t) * E, rp, probs[warp], lane);
        if (lane < K) {
            topk_idx[static_cast<size_t>(t) * K + lane] = sel.idx;
            topk_w[static_cast<size_t>(t) * K + lane] = sel.w;
            s_idx[t * K + lane] = sel.idx;
            s_w[t * K + lane] = sel.w;
            atomicAdd(&totals[sel.idx], 1);
        }
    }
    __syncthreads();
    const int n_pairs = T * K;
    for (int e = tid; e < E; e += blockDim.x) expert_totals[e] = totals[e];
    if (tid == 0) {
        build_schedule(sched, totals, T, n_shared, first_expert, local_E, shared_base, bn, mb1, mb2, seg_off_s);
        *ticket = 0u;  // every CTA has taken its ticket: re-arm for the next launch
    }
    __syncthreads();
    for (int e = first_expert + tid; e < first_expert + local_E; e += blockDim.x) {
        int run = seg_off_s[e];
        for (int q = 0; q < n_pairs; ++q) {
            if (s_idx[q] == e) {
                row_token[run] = q / K;
                row_weight[run] = s_w[q];
                if (slot_row != nullptr) slot_row[q] = run;
                ++run;
            }
        }
    }
    if (slot_row != nullptr && local_E < E) {
        for (int q = tid; q < n_pairs; q += blockDim.x) {
            const int e = s_idx[q];
            if (e < first_expert || e >= first_expert + local_E) slot_row[q] = -1;
        }
    }
}

// Mid-size batches (kRouteTile < T <= kRouteMidTokens): the routing stage in one
// launch, routed in parallel per 32-token block.  CTA (e, b) computes expert e's
// logits for block b's tokens (a warp per token) and zeroes a slice of y.  The last
// CTA of each block (a ticket per block) routes the block's tokens (a warp per
// token) and publishes, per expert, the block's token bit mask; the last block
// router (one more ticket) sums the masks into the expert counts, builds the
// schedule, and places each (token, slot) pair at its expert's first row plus the
// number of earlier tokens in that expert's masks -- rows in (expert, token) order,
// as the placement kernel orders them (a token picks an expert at most once) -- and
// re-arms the tickets.  tickets: kMidBlocks block tickets, then the final one.
constexpr int kMidBlocks = kRouteMidTokens / kRouteTile;
static_assert(kMidBlocks + 2 <= kRouteTickets, "route_small's ticket, the block tickets and the final one");

template <typename XT, int EPL>
__global__ void __launch_bounds__(kSmallThreads) route_mid_kernel(
    const XT* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias, float* __restrict__ logits,
    int T, int H, RouterParams rp, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
    int32_t* __restrict__ expert_totals, Schedule* __restrict__ sched, int32_t* __restrict__ row_token,
    float* __restrict__ row_weight, int32_t* __restrict__ slot_row, float* __restrict__ y_zero,
    unsigned int* __restrict__ tickets, uint32_t* __restrict__ blk_mask, int n_shared, int first_expert, int local_E,
    int shared_base, int bn, int mb1, int mb2) {
    __shared__ float probs[kSmallThreads / 32][kMaxExperts];
    __shared__ uint32_t s_mask[kMaxExperts];
    __shared__ int totals[kMaxExperts];
    __shared__ int seg_off_s[kMaxExperts];
    __shared__ int s_last;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int E = rp.experts;
    const int K = rp.top_k;
    const int nblk = (T + kRouteTile - 1) / kRouteTile;
    pdl_wait();
    pdl_launch_dependents();

    if (y_zero != nullptr) {  // y is accumulated into by the down GEMM
        const int n4 = T * H / 4;
        const int per = (n4 + gridDim.x - 1) / gridDim.x;
        float4* yz = reinterpret_cast<float4*>(y_zero);
        for (int i = blockIdx.x * per + tid; i < min(n4, (blockIdx.x + 1) * per); i += blockDim.x)
            yz[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // Logits of this CTA's expert for its block: a warp per token; the unrolled loop
    // keeps each lane's loads of x and of the router row in flight together.
    const int e = blockIdx.x / nblk;
    const int b = blockIdx.x - e * nblk;
    const int t = b * kRouteTile + warp;
    if (t < T) {
        const float* we = w + static_cast<size_t>(e) * H;
        const XT* xt = x + static_cast<size_t>(t) * H;
        float acc = 0.0f;
#pragma unroll 8
        for (int h = lane * 8; h < H; h += 256) {
            float xv[8], wv[8];
            load8(xt + h, xv);
            load8(we + h, wv);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = fmaf(xv[i], wv[i], acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(kFull, acc, off);
        if (lane == 0) logits[static_cast<size_t>(t) * E + e] = bias != nullptr ? acc + bias[e] : acc;
    }

    // Last CTA of the block: route its tokens and publish the block's expert masks.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&tickets[b], 1u) == static_cast<unsigned>(E - 1)) ? 1 : 0;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < E; i += blockDim.x) s_mask[i] = 0u;
    __syncthreads();
    if (t < T) {
        const Selection sel = route_one_token<EPL>(logits + static_cast<size_t>(t) * E, rp, probs[warp], lane);
        if (lane < K) {
            topk_idx[static_cast<size_t>(t) * K + lane] = sel.idx;
            topk_w[static_cast<size_t>(t) * K + lane] = sel.w;
            atomicOr(&s_mask[sel.idx], 1u << warp);
        }
    }
    __syncthreads();
    for (int i = tid; i < E; i += blockDim.x) blk_mask[static_cast<size_t>(b) * E + i] = s_mask[i];

    // Last block router: counts, schedule, rows; then re-arm every ticket.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&tickets[kMidBlocks], 1u) == static_cast<unsigned>(nblk - 1)) ? 1 : 0;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < E; i += blockDim.x) {
        int c = 0;
        for (int bb = 0; bb < nblk; ++bb) c += __popc(__ldcg(blk_mask + static_cast<size_t>(bb) * E + i));
        totals[i] = c;
        seg_off_s[i] = 0;
        expert_totals[i] = c;
    }
    __syncthreads();
    if (tid == 0) {
        build_schedule(sched, totals, T, n_shared, first_expert, local_E, shared_base, bn, mb1, mb2, seg_off_s);
        for (int i = 0; i <= kMidBlocks; ++i) tickets[i] = 0u;  // every CTA has taken its tickets
    }
    __syncthreads();
    const int n_pairs = T * K;
    for (int q = tid; q < n_pairs; q += blockDim.x) {
        const int tq = q / K;
        const int eq = __ldcg(topk_idx + q);  // written by the block routers, published by the ticket
        if (eq < first_expert || eq >= first_expert + local_E) {
            if (slot_row != nullptr) slot_row[q] = -1;
            continue;
        }
        const int bq = tq / kRouteTile;
        int rank = __popc(__ldcg(blk_mask + static_cast<size_t>(bq) * E + eq) & ((1u << (tq % kRouteTile)) - 1u));
        for (int bb = 0; bb < bq; ++bb) rank += __popc(__ldcg(blk_mask + static_cast<size_t>(bb) * E + eq));
        const int row = seg_off_s[eq] + rank;
        row_token[row] = tq;
        row_weight[row] = __ldcg(topk_w + q);
        if (slot_row != nullptr) slot_row[q] = row;
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
                                 float* split_ws, size_t split_ws_bytes, cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    if (tokens >= 2048 && w_t != nullptr) {
        // Split the hidden axis until the grid has about four CTAs per SM, as far as
        // the workspace holds the partial sums.
        const int tiles = ((tokens + 63) / 64) * ((experts + 63) / 64);
        int splits = 1;
        while (splits < 8 && tiles * splits < 4 * 148 && hidden % (64 * splits * 2) == 0 &&
               static_cast<size_t>(splits) * 2 * tokens * experts * sizeof(float) <= split_ws_bytes &&
               split_ws != nullptr)
            splits *= 2;
        const dim3 grid((tokens + 63) / 64, (experts + 63) / 64, splits);
        float* partial = splits > 1 ? split_ws : nullptr;
        cudaError_t e = x_f32 != nullptr
                            ? launch_k(router_logits_tiled_kernel<float>, grid, dim3(256), stream, pdl, x_f32, w_t,
                                       bias, logits, tokens, hidden, experts, hidden / splits, partial)
                            : launch_k(router_logits_tiled_kernel<uint16_t>, grid, dim3(256), stream, pdl, x, w_t,
                                       bias, logits, tokens, hidden, experts, hidden / splits, partial);
        if (e != cudaSuccess || splits == 1) return e;
        const int64_t n = static_cast<int64_t>(tokens) * experts;
        return launch_k(router_logits_reduce_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), stream,
                        true, static_cast<const float*>(split_ws), bias, logits, tokens, experts, splits);
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

int experts_per_lane(int experts) {
    const int need = (experts + 31) / 32;
    return need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : 8;
}

cudaError_t launch_router_topk(float* logits, int tokens, RouterParams rp, int32_t* topk_idx, float* topk_w,
                               int32_t* tile_counts, cudaStream_t stream, bool pdl, RouterFix fix) {
    if (tokens <= 0) return cudaSuccess;
    const dim3 grid((tokens + kRouteTile - 1) / kRouteTile);
    const dim3 block(kTopkThreads);
    switch (experts_per_lane(rp.experts)) {
        case 1: return launch_k(router_topk_kernel<1>, grid, block, stream, pdl, logits, tokens, rp, topk_idx, topk_w, tile_counts, fix);
        case 2: return launch_k(router_topk_kernel<2>, grid, block, stream, pdl, logits, tokens, rp, topk_idx, topk_w, tile_counts, fix);
        case 4: return launch_k(router_topk_kernel<4>, grid, block, stream, pdl, logits, tokens, rp, topk_idx, topk_w, tile_counts, fix);
        default: return launch_k(router_topk_kernel<8>, grid, block, stream, pdl, logits, tokens, rp, topk_idx, topk_w, tile_counts, fix);
    }
}

cudaError_t launch_dispatch_scan(const int32_t* tile_counts, int32_t* tile_base, int32_t* expert_totals,
                                 Schedule* sched, int tokens, int top_k, int experts, int n_shared,
                                 int first_expert, int local_experts, int shared_base, int bn, int mb1,
                                 int mb2, cudaStream_t stream, bool pdl) {
    return launch_k(dispatch_scan_kernel, dim3(1), dim3(kScanThreads), stream, pdl, tile_counts, tile_base,
                    expert_totals, sched, tokens, top_k, experts, n_shared, first_expert, local_experts,
                    shared_base, bn, mb1, mb2);
}

cudaError_t launch_place(const int32_t* topk_idx, const float* topk_w, const int32_t* tile_base, int tokens,
                         int hidden, int top_k, int experts, int first_expert, int local_experts, int32_t* row_token,
                         float* row_weight, int32_t* slot_row, float* y_zero, const uint16_t* x, uint16_t* x_perm,
                         cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    const int tiles = (tokens + kRouteTile - 1) / kRouteTile;
    return launch_k(place_kernel, dim3(tiles), dim3(256), stream, pdl, topk_idx, topk_w, tile_base, tokens, hidden,
                    top_k, experts, first_expert, local_experts, row_token, row_weight, slot_row, y_zero, x, x_perm);
}

cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* row_token, int rows, int hidden, uint16_t* x_perm,
                               cudaStream_t stream, bool pdl) {
    if (rows <= 0) return cudaSuccess;
    const int64_t vecs = static_cast<int64_t>(rows) * (hidden / 8);
    const int blocks = static_cast<int>(std::min<int64_t>(2048, (vecs + 1023) / 1024));
    return launch_k(gather_rows_kernel, dim3(blocks), dim3(256), stream, pdl, x, row_token, rows, hidden, x_perm);
}

cudaError_t launch_ep_combine(float* y, const uint16_t* back, const int32_t* slot_row, const float* topk_w, int tokens,
                              int top_k, int hidden, cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    const int64_t threads = static_cast<int64_t>(tokens) * (hidden / 4);
    return launch_k(ep_combine_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), stream, pdl, y,
                    back, slot_row, topk_w, tokens, top_k, hidden);
}

// The dense feed-forward's schedule -- one segment of all T tokens (read from x, as a
// shared expert's are), weight slot 0 -- and, unless the call accumulates, y zeroed
// for the down GEMM's adds: one launch, which the gate/up GEMM follows
// programmatically (its prologue overlaps this kernel).
__global__ void dense_schedule_kernel(Schedule* sched, int T, int bn, int mb1, int mb2, float4* __restrict__ y,
                                      int64_t y_vec4) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < y_vec4; i += stride)
        y[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    const int nb = (T + bn - 1) / bn;
    sched->n_seg = 1;
    sched->first_expert = 0;
    sched->seg_off[0] = 0;
    sched->seg_cnt[0] = T;
    sched->seg_weight[0] = 0;
    sched->tiles1[0] = 0;
    sched->tiles2[0] = 0;
    sched->tiles1[1] = nb * mb1;
    sched->tiles2[1] = nb * mb2;
}

cudaError_t launch_dense_schedule(Schedule* sched, int tokens, int bn, int mb1, int mb2, float* y_zero,
                                  int64_t y_count, int sms, cudaStream_t stream) {
    const int64_t vec4 = y_zero != nullptr ? y_count / 4 : 0;
    if (vec4 * 4 != (y_zero != nullptr ? y_count : 0)) return cudaErrorInvalidValue;
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((vec4 + 255) / 256, 4 * sms)));
    return launch_k(dense_schedule_kernel, dim3(grid), dim3(256), stream, false, sched, tokens, bn, mb1, mb2,
                    reinterpret_cast<float4*>(y_zero), vec4);
}

cudaError_t launch_ep_sort_rows(const uint16_t* x_recv, uint16_t* x_sorted, int32_t* row_src,
                               const int32_t* recv_counts, int nranks, int local_experts, int max_group_rows,
                               int hidden, int src_stride, int e_lo, int e_hi, cudaStream_t stream, bool pdl) {
    if (max_group_rows <= 0 || e_hi <= e_lo) return cudaSuccess;
    if (e_lo < 0 || e_hi > local_experts || (src_stride > 0 && (e_lo != 0 || e_hi != local_experts)))
        return cudaErrorInvalidValue;
    const int blocks = (max_group_rows + kSortRows - 1) / kSortRows;
    const dim3 grid(nranks * (e_hi - e_lo), std::min(blocks, 65535));
    return launch_k(ep_sort_rows_kernel, grid, dim3(256), stream, pdl, x_recv, x_sorted, row_src, recv_counts,
                    nranks, local_experts, hidden, src_stride, e_lo, e_hi);
}

// Fixed-capacity expert parallelism (small batches, no host round trip): every
// rank sends every peer a block of `cap` rows, whatever it holds.  ep_pack puts this
// rank's expert-sorted rows (sorted by global expert, so by destination) into
// destination d's block at d * cap, straight from x, and points each (token, slot)
// at its block position for the combine.  One warp per row.
__global__ void __launch_bounds__(256) ep_pack_kernel(const uint16_t* __restrict__ x,
                                                      const int32_t* __restrict__ row_token,
                                                      const int32_t* __restrict__ expert_totals,
                                                      int32_t* __restrict__ slot_row, uint16_t* __restrict__ x_send,
                                                      int T, int K, int E, int El, int cap, int H) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ int off[kMaxExperts + 1];
    if (threadIdx.x < 32) {
        // Each expert's first expert-sorted row: an exclusive scan of the totals by the
        // first warp, every total loaded in one round trip.
        const int ln = threadIdx.x;
        int cv[kMaxExperts / 32];
#pragma unroll
        for (int i = 0; i < kMaxExperts / 32; ++i) cv[i] = i * 32 + ln < E ? expert_totals[i * 32 + ln] : 0;
        int run = 0;
#pragma unroll
        for (int i = 0; i < kMaxExperts / 32; ++i) {
            int incl = cv[i];
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, d);
                if (ln >= d) incl += v;
            }
            if (i * 32 + ln < E) off[i * 32 + ln] = run + incl - cv[i];
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (ln == 0) off[E] = run;
    }
    __syncthreads();
    const int n_rows = T * K;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int n_warps = (gridDim.x * blockDim.x) >> 5;
    // Expert-sorted row r -> its destination block position.
    auto padded = [&](int r) {
        int lo = 0, hi = E;  // off[lo] <= r < off[hi]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (off[mid] <= r) lo = mid; else hi = mid;
        }
        const int d = lo / El;
        return d * cap + (r - off[d * El]);
    };
    const int vec = H / 8;
    constexpr int kPackUnroll = 8;  // a lane's 16-byte loads in flight together (a 4 KB row per warp)
    for (int r = warp; r < n_rows; r += n_warps) {
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row_token[r]) * H);
        uint4* dst = reinterpret_cast<uint4*>(x_send + static_cast<size_t>(padded(r)) * H);
        for (int v0 = 0; v0 < vec; v0 += 32 * kPackUnroll) {
            uint4 t[kPackUnroll];
#pragma unroll
            for (int u = 0; u < kPackUnroll; ++u)
                if (v0 + u * 32 + lane < vec) t[u] = src[v0 + u * 32 + lane];
#pragma unroll
            for (int u = 0; u < kPackUnroll; ++u)
                if (v0 + u * 32 + lane < vec) dst[v0 + u * 32 + lane] = t[u];
        }
    }
    for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < n_rows; q += gridDim.x * blockDim.x)
        if (slot_row[q] >= 0) slot_row[q] = padded(slot_row[q]);
}

cudaError_t launch_ep_pack(const uint16_t* x, const int32_t* row_token, const int32_t* expert_totals,
                           int32_t* slot_row, uint16_t* x_send, int tokens, int top_k, int experts,
                           int local_experts, int cap, int hidden, cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    const int rows = tokens * top_k;
    const int blocks = std::min((rows + 7) / 8, 1024);
    return launch_k(ep_pack_kernel, dim3(blocks), dim3(256), stream, pdl, x, row_token, expert_totals, slot_row,
                    x_send, tokens, top_k, experts, local_experts, cap, hidden);
}

// The receiver's schedule of a fixed-capacity exchange, on the device: one segment
// per local expert (its rows from every source, expert-major), then the shared
// experts over this rank's own T tokens at row shared_base + j * T.
__global__ void ep_schedule_kernel(const int32_t* __restrict__ recv_counts, Schedule* __restrict__ sched, int N,
                                   int El, int n_shared, int T, int shared_base, int bn, int mb1, int mb2) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    int off = 0, p1 = 0, p2 = 0, seg = 0;
    auto add = [&](int o, int cnt, int w) {
        sched->seg_off[seg] = o;
        sched->seg_cnt[seg] = cnt;
        sched->seg_weight[seg] = w;
        sched->tiles1[seg] = p1;
        sched->tiles2[seg] = p2;
        const int nb = (cnt + bn - 1) / bn;
        p1 += nb * mb1;
        p2 += nb * mb2;
        ++seg;
    };
    for (int e = 0; e < El; ++e) {
        int cnt = 0;
        for (int r = 0; r < N; ++r) cnt += recv_counts[r * El + e];
        add(off, cnt, e);
        off += cnt;
    }
    for (int j = 0; j < n_shared; ++j) add(shared_base + j * T, T, El + j);
    sched->tiles1[seg] = p1;
    sched->tiles2[seg] = p2;
    sched->n_seg = seg;
    sched->first_expert = 0;
}

cudaError_t launch_ep_schedule(const int32_t* recv_counts, Schedule* sched, int nranks, int local_experts,
                               int n_shared, int tokens, int shared_base, int bn, int mb1, int mb2,
                               cudaStream_t stream, bool pdl) {
    return launch_k(ep_schedule_kernel, dim3(1), dim3(32), stream, pdl, recv_counts, sched, nranks, local_experts,
                    n_shared, tokens, shared_base, bn, mb1, mb2);
}

template <typename XT, int EPL>
cudaError_t launch_route_small_t(const XT* x, const float* w, const float* bias, float* logits, int tokens, int hidden,
                                 RouterParams rp, int32_t* topk_idx, float* topk_w, int32_t* expert_totals,
                                 Schedule* sched, int32_t* row_token, float* row_weight, int32_t* slot_row,
                                 float* y_zero, unsigned int* ticket, int n_shared, int first_expert,
                                 int local_experts, int shared_base, int bn, int mb1, int mb2, cudaStream_t stream,
                                 bool pdl) {
    const dim3 grid((rp.experts + kSmallExperts - 1) / kSmallExperts);
    return launch_k(route_small_kernel<XT, EPL>, grid, dim3(kSmallThreads), stream, pdl, x, w, bias, logits, tokens,
                    hidden, rp, topk_idx, topk_w, expert_totals, sched, row_token, row_weight, slot_row, y_zero,
                    ticket, n_shared, first_expert, local_experts, shared_base, bn, mb1, mb2);
}

template <typename XT>
cudaError_t route_small_dispatch(const XT* x, const float* w, const float* bias, float* logits, int tokens,
                                 int hidden, RouterParams rp, int32_t* topk_idx, float* topk_w,
                                 int32_t* expert_totals, Schedule* sched, int32_t* row_token, float* row_weight,
                                 int32_t* slot_row, float* y_zero, unsigned int* ticket, int n_shared,
                                 int first_expert, int local_experts, int shared_base, int bn, int mb1, int mb2,
                                 cudaStream_t stream, bool pdl) {
#define LM_ROUTE_SMALL(EPL)                                                                                      \
    launch_route_small_t<XT, EPL>(x, w, bias, logits, tokens, hidden, rp, topk_idx, topk_w, expert_totals, sched, \
                                  row_token, row_weight, slot_row, y_zero, ticket, n_shared, first_expert,        \
                                  local_experts, shared_base, bn, mb1, mb2, stream, pdl)
    switch (experts_per_lane(rp.experts)) {
        case 1: return LM_ROUTE_SMALL(1);
        case 2: return LM_ROUTE_SMALL(2);
        case 4: return LM_ROUTE_SMALL(4);
        default: return LM_ROUTE_SMALL(8);
    }
#undef LM_ROUTE_SMALL
}

template <typename XT, int EPL>
cudaError_t launch_route_mid_t(const XT* x, const float* w, const float* bias, float* logits, int tokens, int hidden,
                               RouterParams rp, int32_t* topk_idx, float* topk_w, int32_t* expert_totals,
                               Schedule* sched, int32_t* row_token, float* row_weight, int32_t* slot_row,
                               float* y_zero, unsigned int* tickets, uint32_t* blk_mask, int n_shared,
                               int first_expert, int local_experts, int shared_base, int bn, int mb1, int mb2,
                               cudaStream_t stream, bool pdl) {
    const int nblk = (tokens + kRouteTile - 1) / kRouteTile;
    const dim3 grid(static_cast<unsigned>(rp.experts * nblk));
    return launch_k(route_mid_kernel<XT, EPL>, grid, dim3(kSmallThreads), stream, pdl, x, w, bias, logits, tokens,
                    hidden, rp, topk_idx, topk_w, expert_totals, sched, row_token, row_weight, slot_row, y_zero,
                    tickets, blk_mask, n_shared, first_expert, local_experts, shared_base, bn, mb1, mb2);
}

template <typename XT>
cudaError_t route_mid_dispatch(const XT* x, const float* w, const float* bias, float* logits, int tokens, int hidden,
                               RouterParams rp, int32_t* topk_idx, float* topk_w, int32_t* expert_totals,
                               Schedule* sched, int32_t* row_token, float* row_weight, int32_t* slot_row,
                               float* y_zero, unsigned int* tickets, uint32_t* blk_mask, int n_shared,
                               int first_expert, int local_experts, int shared_base, int bn, int mb1, int mb2,
                               cudaStream_t stream, bool pdl) {
#define LM_ROUTE_MID(EPL)                                                                                        \
    launch_route_mid_t<XT, EPL>(x, w, bias, logits, tokens, hidden, rp, topk_idx, topk_w, expert_totals, sched, \
                                row_token, row_weight, slot_row, y_zero, tickets, blk_mask, n_shared,           \
                                first_expert, local_experts, shared_base, bn, mb1, mb2, stream, pdl)
    switch (experts_per_lane(rp.experts)) {
        case 1: return LM_ROUTE_MID(1);
        case 2: return LM_ROUTE_MID(2);
        case 4: return LM_ROUTE_MID(4);
        default: return LM_ROUTE_MID(8);
    }
#undef LM_ROUTE_MID
}

cudaError_t launch_route_mid(const uint16_t* x, const float* x_f32, const float* w, const float* bias, float* logits,
                             int tokens, int hidden, RouterParams rp, int32_t* topk_idx, float* topk_w,
                             int32_t* expert_totals, Schedule* sched, int32_t* row_token, float* row_weight,
                             int32_t* slot_row, float* y_zero, unsigned int* tickets, uint32_t* blk_mask,
                             int n_shared, int first_expert, int local_experts, int shared_base, int bn, int mb1,
                             int mb2, cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    if (tokens > kRouteMidTokens || rp.experts > kMaxExperts || rp.top_k > kMaxTopK || hidden % 8 != 0)
        return cudaErrorInvalidValue;
    if (x_f32 != nullptr)
        return route_mid_dispatch<float>(x_f32, w, bias, logits, tokens, hidden, rp, topk_idx, topk_w, expert_totals,
                                         sched, row_token, row_weight, slot_row, y_zero, tickets, blk_mask, n_shared,
                                         first_expert, local_experts, shared_base, bn, mb1, mb2, stream, pdl);
    return route_mid_dispatch<uint16_t>(x, w, bias, logits, tokens, hidden, rp, topk_idx, topk_w, expert_totals,
                                        sched, row_token, row_weight, slot_row, y_zero, tickets, blk_mask, n_shared,
                                        first_expert, local_experts, shared_base, bn, mb1, mb2, stream, pdl);
}

cudaError_t launch_route_small(const uint16_t* x, const float* x_f32, const float* w, const float* bias,
                               float* logits, int tokens, int hidden, RouterParams rp, int32_t* topk_idx,
                               float* topk_w, int32_t* expert_totals, Schedule* sched, int32_t* row_token,
                               float* row_weight, int32_t* slot_row, float* y_zero, unsigned int* ticket,
                               int n_shared, int first_expert, int local_experts, int shared_base, int bn, int mb1,
                               int mb2, cudaStream_t stream, bool pdl) {
    if (tokens <= 0) return cudaSuccess;
    if (tokens > kRouteTile) return cudaErrorInvalidValue;
    if (x_f32 != nullptr)
        return route_small_dispatch<float>(x_f32, w, bias, logits, tokens, hidden, rp, topk_idx, topk_w,
                                           expert_totals, sched, row_token, row_weight, slot_row, y_zero, ticket,
                                           n_shared, first_expert, local_experts, shared_base, bn, mb1, mb2, stream,
                                           pdl);
    return route_small_dispatch<uint16_t>(x, w, bias, logits, tokens, hidden, rp, topk_idx, topk_w, expert_totals,
                                          sched, row_token, row_weight, slot_row, y_zero, ticket, n_shared,
                                          first_expert, local_experts, shared_base, bn, mb1, mb2, stream, pdl);
}

// Loads every kernel and instantiation of this file (see preload_kernels in moe_internal.h).
cudaError_t preload_router_kernels() {
    cudaFuncAttributes a{};
    const void* kernels[] = {
        reinterpret_cast<const void*>(router_logits_warp_kernel<uint16_t>),
        reinterpret_cast<const void*>(router_logits_warp_kernel<float>),
        reinterpret_cast<const void*>(router_logits_tiled_kernel<uint16_t>),
        reinterpret_cast<const void*>(router_logits_tiled_kernel<float>),
        reinterpret_cast<const void*>(router_logits_reduce_kernel),
        reinterpret_cast<const void*>(router_topk_kernel<1>),
        reinterpret_cast<const void*>(router_topk_kernel<2>),
        reinterpret_cast<const void*>(router_topk_kernel<4>),
        reinterpret_cast<const void*>(router_topk_kernel<8>),
        reinterpret_cast<const void*>(dispatch_scan_kernel),
        reinterpret_cast<const void*>(place_kernel),
        reinterpret_cast<const void*>(gather_rows_kernel),
        reinterpret_cast<const void*>(ep_combine_kernel),
        reinterpret_cast<const void*>(ep_sort_rows_kernel),
        reinterpret_cast<const void*>(ep_pack_kernel),
        reinterpret_cast<const void*>(ep_schedule_kernel),
        reinterpret_cast<const void*>(dense_schedule_kernel),
        reinterpret_cast<const void*>(route_small_kernel<uint16_t, 1>),
        reinterpret_cast<const void*>(route_small_kernel<uint16_t, 2>),
        reinterpret_cast<const void*>(route_small_kernel<uint16_t, 4>),
        reinterpret_cast<const void*>(route_small_kernel<uint16_t, 8>),
        reinterpret_cast<const void*>(route_small_kernel<float, 1>),
        reinterpret_cast<const void*>(route_small_kernel<float, 2>),
        reinterpret_cast<const void*>(route_small_kernel<float, 4>),
        reinterpret_cast<const void*>(route_small_kernel<float, 8>),
        reinterpret_cast<const void*>(route_mid_kernel<uint16_t, 1>),
        reinterpret_cast<const void*>(route_mid_kernel<uint16_t, 2>),
        reinterpret_cast<const void*>(route_mid_kernel<uint16_t, 4>),
        reinterpret_cast<const void*>(route_mid_kernel<uint16_t, 8>),
        reinterpret_cast<const void*>(route_mid_kernel<float, 1>),
        reinterpret_cast<const void*>(route_mid_kernel<float, 2>),
        reinterpret_cast<const void*>(route_mid_kernel<float, 4>),
        reinterpret_cast<const void*>(route_mid_kernel<float, 8>),
    };
    for (const void* k : kernels)
        if (const cudaError_t e = cudaFuncGetAttributes(&a, k); e != cudaSuccess) return e;
    return cudaSuccess;
}

}  // namespace lm
