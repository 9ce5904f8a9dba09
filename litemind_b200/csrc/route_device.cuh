// route_device.cuh -- per-token routing and small load helpers shared by the
// routing kernels (router.cu) and the fused decode kernel (decode_fused.cu).
#pragma once

#include <cfloat>
#include <cstdint>

#include "moe_internal.h"

namespace lm {

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

constexpr uint32_t kFull = 0xffffffffu;

// One token's routing by one warp: MoeRouter::select (src/MoeRouter.cpp:54-107).
// Softmax over every expert before the cut (:61-64, src/Gemm.cpp:209-223), optional
// group-limited masking (:66-84), greedy top-k ordered by (allowed, probability
// descending, index ascending) as top_k_indices orders them (:21-32), then
// normalise or scale, never both (:96-106).  Each round of the top-k packs
// (allowed, probability) into one 32-bit key -- probabilities are non-negative, so
// their bit patterns order like their values -- and takes the warp's maximum key,
// then the lowest expert index holding it, with two redux.sync reductions.
// Lane s < K returns selection s.  `lg` holds the token's E logits; `probs` is E
// floats of per-warp shared scratch (group-limited routing only).
struct Selection {
    int idx;
    float w;
    bool ambiguous;  // two of the first k+1 ranked probabilities are closer than the margin
};

// kShared: `lg` points to shared memory (plain loads) instead of global memory
// written by other CTAs (L2 loads).
template <int EPL, bool kShared = false>  // experts per lane: ceil(E / 32) rounded up to 1, 2, 4 or 8
__device__ __forceinline__ Selection route_one_token(const float* lg, const RouterParams& rp, float* probs, int lane,
                                                     float margin = 0.0f) {
    const int E = rp.experts;
    const int K = rp.top_k;
    float p[EPL];
    float m = -FLT_MAX;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? (kShared ? lg[e] : __ldcg(lg + e)) : -FLT_MAX;
        m = fmaxf(m, p[j]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? expf(p[j] - m) : 0.0f;
        sum += p[j];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(kFull, sum, off);
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) p[j] *= inv;

    uint32_t group_mask = 0xffffffffu;
    int per_group = E;
    if (rp.group_limited && rp.n_group > 1) {
        per_group = E / rp.n_group;
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
            const int e = lane + 32 * j;
            if (e < E) probs[e] = p[j];
        }
        __syncwarp();
        uint32_t gkey = 0;
        bool g_avail = lane < rp.n_group;
        if (g_avail) {
            float best = probs[lane * per_group];
            for (int o = 1; o < per_group; ++o) best = fmaxf(best, probs[lane * per_group + o]);
            gkey = __float_as_uint(best);
        }
        __syncwarp();
        group_mask = 0u;
        const int keep = min(rp.topk_group, rp.n_group);
        for (int r = 0; r < keep; ++r) {
            const uint32_t gmax = __reduce_max_sync(kFull, g_avail ? gkey : 0u);
            const uint32_t gc = (g_avail && gkey == gmax) ? static_cast<uint32_t>(lane) : 0xffffffffu;
            const uint32_t g = __reduce_min_sync(kFull, gc);
            if (g < 32u) {
                group_mask |= 1u << g;
                if (g == static_cast<uint32_t>(lane)) g_avail = false;
            }
        }
    }

    uint32_t key[EPL];
    uint32_t avail = 0;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        const int e = lane + 32 * j;
        key[j] = 0;
        if (e < E) {
            const uint32_t allowed = (group_mask >> (e / per_group)) & 1u;
            key[j] = (allowed << 31) | __float_as_uint(p[j]);
            avail |= 1u << j;
        }
    }
    Selection mine{-1, 0.0f, false};
    // One round past K when a margin is asked for: the (k+1)-th probability decides
    // whether an approximate logit could have moved the cut.
    const int rounds = (margin > 0.0f && K < E) ? K + 1 : K;
    float prev = 0.0f;
    float min_gap = 1.0f;
    for (int s = 0; s < rounds; ++s) {
        uint32_t best = 0;
        int bj = -1;
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
            if (((avail >> j) & 1u) && (bj < 0 || key[j] > best)) {
                best = key[j];
                bj = j;
            }
        }
        const uint32_t wmax = __reduce_max_sync(kFull, bj >= 0 ? best : 0u);
        const uint32_t cand = (bj >= 0 && best == wmax) ? static_cast<uint32_t>(lane + 32 * bj) : 0xffffffffu;
        const uint32_t win = __reduce_min_sync(kFull, cand);
        if ((win & 31u) == static_cast<uint32_t>(lane)) avail &= ~(1u << (win >> 5));
        const float pw = __uint_as_float(wmax & 0x7fffffffu);
        if (s > 0) min_gap = fminf(min_gap, prev - pw);
        prev = pw;
        if (lane == s && s < K) {
            mine.idx = static_cast<int>(win);
            mine.w = pw;
        }
    }
    mine.ambiguous = margin > 0.0f && min_gap < margin;
    if (K > 1 && rp.normalize) {
        float selected = 0.0f;  // in selection order, as the reference sums it
        for (int s = 0; s < K; ++s) selected += __shfl_sync(kFull, mine.w, s);
        mine.w = mine.w / (selected + 1e-20f);
    } else if (rp.scale != 1.0f) {
        mine.w = mine.w * rp.scale;
    }
    return mine;
}

}  // namespace lm
