/*
 * moe_oracle.c -- CPU restatement of LiteMind's MoE feed-forward path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).  See moe_oracle.h.
 *
 * Compiled with -ffp-contract=off so that the only fused multiply-adds are the
 * explicit fmaf() calls below; they sit exactly where GCC contracts the
 * reference's `a += b * c` statements when it builds src/Gemm.cpp with FMA
 * enabled (the reference's -march=native build on any AVX2 machine): the AVX2
 * intrinsics, matvec_bf16_accumulate and axpy.  The scalar reductions in dot()
 * and in dot_bf16's tail stay a separate multiply and add, as GCC emits them.
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

float orc_bf16_to_f32(uint16_t bits) {
    /* src/Gemm.cpp:18-20: bf16 shares float32's exponent layout. */
    uint32_t wide = (uint32_t)bits << 16;
    float value;
    memcpy(&value, &wide, sizeof value);
    return value;
}

uint16_t orc_f32_to_bf16(float value) {
    /* tests/KernelTest.cpp:15-20: round to nearest, ties to even. */
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    uint32_t rounded = bits + 0x7fffU + ((bits >> 16) & 1U);
    return (uint16_t)(rounded >> 16);
}

float orc_dot(const float* left, const float* right, size_t count) {
    /* src/Gemm.cpp:183-189: one sequential fp32 accumulator.  As GCC compiles it
     * with AVX2+FMA, the products of the leading multiple-of-4 elements are
     * rounded before each add (vector multiplies, scalar adds in order), and the
     * last count % 4 elements are fused multiply-adds. */
    float total = 0.0f;
    const size_t plain = count & ~(size_t)3;
    size_t i = 0;
    for (; i < plain; ++i) {
        total += left[i] * right[i];
    }
    for (; i < count; ++i) {
        total = fmaf(left[i], right[i], total);
    }
    return total;
}

float orc_dot_bf16(const uint16_t* weights, const float* input, size_t count) {
    /* src/Gemm.cpp:46-102, AVX2+FMA branch: four 8-lane accumulators over 32-wide
     * steps, an 8-wide step into accumulator 0, then (a0+a1)+(a2+a3), the
     * 8->4->2->1 horizontal sum of :25-32 and a fused scalar tail. */
    float acc[4][8];
    memset(acc, 0, sizeof acc);
    size_t i = 0;
    for (; i + 32 <= count; i += 32) {
        for (int j = 0; j < 4; ++j) {
            for (int l = 0; l < 8; ++l) {
                const size_t at = i + 8 * (size_t)j + (size_t)l;
                acc[j][l] = fmaf(orc_bf16_to_f32(weights[at]), input[at], acc[j][l]);
            }
        }
    }
    for (; i + 8 <= count; i += 8) {
        for (int l = 0; l < 8; ++l) {
            acc[0][l] = fmaf(orc_bf16_to_f32(weights[i + l]), input[i + l], acc[0][l]);
        }
    }
    float s[8];
    for (int l = 0; l < 8; ++l) {
        const float a01 = acc[0][l] + acc[1][l];
        const float a23 = acc[2][l] + acc[3][l];
        s[l] = a01 + a23;
    }
    float t[4];
    for (int l = 0; l < 4; ++l) {
        t[l] = s[l] + s[l + 4];
    }
    float total = (t[0] + t[2]) + (t[1] + t[3]);
    for (; i < count; ++i) {
        total += orc_bf16_to_f32(weights[i]) * input[i]; /* not contracted, as in the reference */
    }
    return total;
}

void orc_matvec_f32(const float* weights, const float* input, float* out, size_t out_dim,
                    size_t in_dim) {
    for (size_t row = 0; row < out_dim; ++row) {
        out[row] = orc_dot(weights + row * in_dim, input, in_dim);
    }
}

void orc_matvec_bf16(const uint16_t* weights, const float* input, float* out, size_t out_dim,
                     size_t in_dim) {
    /* Rows are independent; the reference's 32-row tasks (:16, :147-153) do not
     * change any row's arithmetic, so a plain loop is the same function. */
    for (size_t row = 0; row < out_dim; ++row) {
        out[row] = orc_dot_bf16(weights + row * in_dim, input, in_dim);
    }
}

void orc_matvec_bf16_accumulate(const uint16_t* weights, const float* input, float* out,
                                size_t out_dim, size_t in_dim, float scale) {
    /* :156-175: out[row] += scale * dot, contracted to one fused multiply-add. */
    for (size_t row = 0; row < out_dim; ++row) {
        out[row] = fmaf(scale, orc_dot_bf16(weights + row * in_dim, input, in_dim), out[row]);
    }
}

void orc_axpy(float scale, const float* source, float* destination, size_t count) {
    for (size_t i = 0; i < count; ++i) {
        destination[i] = fmaf(scale, source[i], destination[i]);
    }
}

void orc_rms_norm(float* values, const float* weight, size_t count, float epsilon) {
    /* :197-207: sum of squares in double, then x * inverse * weight. */
    double sum_of_squares = 0.0;
    for (size_t i = 0; i < count; ++i) {
        sum_of_squares = fma((double)values[i], (double)values[i], sum_of_squares);
    }
    const float inverse =
        (float)(1.0 / sqrt(sum_of_squares / (double)count + (double)epsilon));
    for (size_t i = 0; i < count; ++i) {
        values[i] = values[i] * inverse * weight[i];
    }
}

void orc_softmax(float* values, size_t count) {
    /* :209-223: max-subtracted exponentials, fp32 sum, multiply by 1/sum. */
    if (count == 0) {
        return;
    }
    float maximum = values[0];
    for (size_t i = 1; i < count; ++i) {
        if (values[i] > maximum) {
            maximum = values[i];
        }
    }
    float total = 0.0f;
    for (size_t i = 0; i < count; ++i) {
        values[i] = expf(values[i] - maximum);
        total += values[i];
    }
    const float inverse = total > 0.0f ? 1.0f / total : 0.0f;
    for (size_t i = 0; i < count; ++i) {
        values[i] *= inverse;
    }
}

void orc_silu_multiply(const float* gate, const float* up, float* destination, size_t count) {
    /* :225-231 */
    for (size_t i = 0; i < count; ++i) {
        const float value = gate[i];
        destination[i] = value / (1.0f + expf(-value)) * up[i];
    }
}

/* ── Routing ─────────────────────────────────────────────────────────────── */

void orc_router_init(orc_router* router, int64_t n_routed_experts, int64_t num_experts_per_tok,
                     int64_t n_group, int64_t topk_group, int32_t group_limited_greedy,
                     int32_t norm_topk_prob, float routed_scaling_factor) {
    router->expert_count = n_routed_experts;
    router->top_k = num_experts_per_tok;
    router->n_group = n_group > 1 ? n_group : 1;
    router->topk_group = topk_group > 1 ? topk_group : 1;
    router->group_limited = group_limited_greedy != 0;
    router->normalize = norm_topk_prob != 0;
    router->routed_scaling_factor = routed_scaling_factor;
    if (router->expert_count % router->n_group != 0) {
        /* src/MoeRouter.cpp:46-51 */
        router->group_limited = 0;
        router->n_group = 1;
    }
}

/* True when a ranks ahead of b under top_k_indices' comparator
 * (src/MoeRouter.cpp:21-32): allowed first, then higher score, then lower index. */
static int ranks_ahead(const float* scores, const unsigned char* allowed, int64_t a, int64_t b) {
    const int a_allowed = allowed == NULL || allowed[a];
    const int b_allowed = allowed == NULL || allowed[b];
    if (a_allowed != b_allowed) {
        return a_allowed;
    }
    if (scores[a] != scores[b]) {
        return scores[a] > scores[b];
    }
    return a < b;
}

/* top_k_indices, src/MoeRouter.cpp:14-34.  The comparator is a total order, so
 * repeated selection of the leading element gives partial_sort's prefix. */
static int64_t top_k_indices(const float* scores, const unsigned char* allowed, int64_t count,
                             int64_t top_k, int64_t* order, unsigned char* taken) {
    const int64_t keep = top_k < count ? top_k : count;
    memset(taken, 0, (size_t)count);
    for (int64_t slot = 0; slot < keep; ++slot) {
        int64_t best = -1;
        for (int64_t e = 0; e < count; ++e) {
            if (taken[e]) {
                continue;
            }
            if (best < 0 || ranks_ahead(scores, allowed, e, best)) {
                best = e;
            }
        }
        taken[best] = 1;
        order[slot] = best;
    }
    return keep;
}

int64_t orc_router_select(const orc_router* router, const float* logits, int64_t count,
                          int64_t* expert_index, float* weight) {
    const int64_t E = router->expert_count;
    if (count != E || router->top_k == 0 || E == 0) {
        return 0; /* src/MoeRouter.cpp:57-59 */
    }
    float* scores = (float*)malloc((size_t)E * sizeof(float));
    unsigned char* allowed = NULL;
    unsigned char* taken = (unsigned char*)malloc((size_t)E);
    int64_t* order = (int64_t*)malloc((size_t)E * sizeof(int64_t));
    memcpy(scores, logits, (size_t)E * sizeof(float));
    orc_softmax(scores, (size_t)E); /* :63-64, softmax before the cut */

    if (router->group_limited && router->n_group > 1) {
        /* :66-84: group score = max probability in the group, keep topk_group groups. */
        const int64_t G = router->n_group;
        const int64_t per_group = E / G;
        float* group_scores = (float*)malloc((size_t)G * sizeof(float));
        int64_t* group_order = (int64_t*)malloc((size_t)G * sizeof(int64_t));
        unsigned char* group_taken = (unsigned char*)malloc((size_t)G);
        for (int64_t g = 0; g < G; ++g) {
            float best = scores[g * per_group];
            for (int64_t o = 1; o < per_group; ++o) {
                if (scores[g * per_group + o] > best) {
                    best = scores[g * per_group + o];
                }
            }
            group_scores[g] = best;
        }
        const int64_t keep_groups = router->topk_group < G ? router->topk_group : G;
        const int64_t kept = top_k_indices(group_scores, NULL, G, keep_groups, group_order, group_taken);
        allowed = (unsigned char*)calloc((size_t)E, 1);
        for (int64_t i = 0; i < kept; ++i) {
            for (int64_t o = 0; o < per_group; ++o) {
                allowed[group_order[i] * per_group + o] = 1;
            }
        }
        free(group_scores);
        free(group_order);
        free(group_taken);
    }

    const int64_t n = top_k_indices(scores, allowed, E, router->top_k, order, taken);
    float selected_sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        expert_index[i] = order[i];
        weight[i] = scores[order[i]];
        selected_sum += scores[order[i]];
    }
    /* :96-106: normalise or scale, never both. */
    if (router->top_k > 1 && router->normalize) {
        const float denominator = selected_sum + 1e-20f;
        for (int64_t i = 0; i < n; ++i) {
            weight[i] /= denominator;
        }
    } else if (router->routed_scaling_factor != 1.0f) {
        for (int64_t i = 0; i < n; ++i) {
            weight[i] *= router->routed_scaling_factor;
        }
    }
    free(scores);
    free(allowed);
    free(taken);
    free(order);
    return n;
}

int64_t orc_select_top_k(const float* logits, int64_t logit_count, int64_t expert_count,
                         int64_t top_k, int32_t normalize, int64_t* expert_index, float* weight) {
    if (expert_count == 0 || top_k == 0 || top_k > expert_count || logit_count != expert_count) {
        return -1; /* src/MoeRouter.cpp:119-121 throws std::invalid_argument */
    }
    orc_router router;
    orc_router_init(&router, expert_count, top_k, 1, 1, 0, normalize, 1.0f);
    return orc_router_select(&router, logits, logit_count, expert_index, weight);
}

/* ── The MoE block ───────────────────────────────────────────────────────── */

/* Impl::feed_forward, src/DeepSeekRunner.cpp:228-240. */
static void feed_forward(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                         int64_t inter, int64_t hidden, const float* x, float* out, float scale,
                         float* gate_buf, float* up_buf, float* act_buf) {
    orc_matvec_bf16(gate, x, gate_buf, (size_t)inter, (size_t)hidden);
    orc_matvec_bf16(up, x, up_buf, (size_t)inter, (size_t)hidden);
    orc_silu_multiply(gate_buf, up_buf, act_buf, (size_t)inter);
    orc_matvec_bf16_accumulate(down, act_buf, out, (size_t)hidden, (size_t)inter, scale);
}

int orc_moe_layer(const orc_moe_shape* shape, int64_t tokens, const float* x,
                  const float* router, const float* bias,
                  const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                  const uint16_t* sh_gate, const uint16_t* sh_up, const uint16_t* sh_down,
                  float* y, int64_t* idx, float* w, float* logits_out, int threads) {
    const int64_t H = shape->hidden;
    const int64_t I = shape->inter;
    const int64_t E = shape->router.expert_count;
    const int64_t K = shape->router.top_k;
    const int64_t S = I * shape->n_shared;
    const int64_t widest = S > I ? S : I;
    const int64_t expert_elems = I * H;
    if (H <= 0 || I <= 0 || E <= 0 || K <= 0 || tokens < 0) {
        return -1;
    }
#ifdef _OPENMP
    if (threads > 0) {
        omp_set_num_threads(threads);
    }
#else
    (void)threads;
#endif
    int status = 0;
#pragma omp parallel
    {
        float* gate_buf = (float*)malloc((size_t)widest * sizeof(float));
        float* up_buf = (float*)malloc((size_t)widest * sizeof(float));
        float* act_buf = (float*)malloc((size_t)widest * sizeof(float));
        float* logits = (float*)malloc((size_t)E * sizeof(float));
        int64_t* sel_idx = (int64_t*)malloc((size_t)K * sizeof(int64_t));
        float* sel_w = (float*)malloc((size_t)K * sizeof(float));
#pragma omp for schedule(dynamic, 1)
        for (int64_t t = 0; t < tokens; ++t) {
            const float* xt = x + t * H;
            float* out = y + t * H;
            /* :273-275: router logits, then selection. */
            orc_matvec_f32(router, xt, logits, (size_t)E, (size_t)H);
            if (bias != NULL) {
                for (int64_t e = 0; e < E; ++e) {
                    logits[e] = logits[e] + bias[e];
                }
            }
            if (logits_out != NULL) {
                memcpy(logits_out + t * E, logits, (size_t)E * sizeof(float));
            }
            const int64_t n = orc_router_select(&shape->router, logits, E, sel_idx, sel_w);
            if (n != K) {
#pragma omp atomic write
                status = -2;
            }
            /* :268: the output starts at zero; :277-284 experts in selection order. */
            memset(out, 0, (size_t)H * sizeof(float));
            for (int64_t s = 0; s < n; ++s) {
                const int64_t e = sel_idx[s];
                feed_forward(gate + e * expert_elems, up + e * expert_elems, down + e * expert_elems,
                             I, H, xt, out, sel_w[s], gate_buf, up_buf, act_buf);
                if (idx != NULL) {
                    idx[t * K + s] = e;
                }
                if (w != NULL) {
                    w[t * K + s] = sel_w[s];
                }
            }
            /* :285-288: the shared experts, weight 1.0. */
            if (S > 0) {
                feed_forward(sh_gate, sh_up, sh_down, S, H, xt, out, 1.0f, gate_buf, up_buf,
                             act_buf);
            }
        }
        free(gate_buf);
        free(up_buf);
        free(act_buf);
        free(logits);
        free(sel_idx);
        free(sel_w);
    }
    return status;
}

/* ── ExpertCache bookkeeping ─────────────────────────────────────────────── */

uint64_t orc_cache_make_key(uint64_t layer, uint64_t expert) {
    /* include/ExpertCache.hpp:67-69 */
    return (layer << 32) | (uint32_t)expert;
}

void orc_cache_configure(orc_expert_cache* cache, uint64_t budget_bytes) {
    cache->budget_bytes = budget_bytes; /* src/ExpertCache.cpp:5-7 */
}

static void cache_evict_oldest(orc_expert_cache* cache) {
    /* src/ExpertCache.cpp:49-68: drop the least recently used entry. */
    if (cache->count == 0) {
        return;
    }
    cache->count -= 1;
    cache->resident_bytes -= cache->bytes[cache->count];
    cache->evictions += 1;
}

void orc_cache_touch(orc_expert_cache* cache, uint64_t key, uint64_t block_bytes) {
    /* src/ExpertCache.cpp:9-47 */
    if (cache->budget_bytes == 0) {
        return;
    }
    for (int64_t i = 0; i < cache->count; ++i) {
        if (cache->keys[i] == key) {
            const uint64_t bytes = cache->bytes[i];
            memmove(&cache->keys[1], &cache->keys[0], (size_t)i * sizeof(uint64_t));
            memmove(&cache->bytes[1], &cache->bytes[0], (size_t)i * sizeof(uint64_t));
            cache->keys[0] = key;
            cache->bytes[0] = bytes;
            cache->hits += 1;
            return;
        }
    }
    while (cache->resident_bytes + block_bytes > cache->budget_bytes && cache->count > 0) {
        cache_evict_oldest(cache);
    }
    if (cache->count == ORC_CACHE_CAPACITY) {
        cache_evict_oldest(cache);
    }
    memmove(&cache->keys[1], &cache->keys[0], (size_t)cache->count * sizeof(uint64_t));
    memmove(&cache->bytes[1], &cache->bytes[0], (size_t)cache->count * sizeof(uint64_t));
    cache->keys[0] = key;
    cache->bytes[0] = block_bytes;
    cache->count += 1;
    cache->resident_bytes += block_bytes;
    cache->bytes_streamed += block_bytes;
    cache->loads += 1;
}

void orc_cache_clear(orc_expert_cache* cache) {
    /* src/ExpertCache.cpp:70-76 */
    while (cache->count > 0) {
        cache_evict_oldest(cache);
    }
    cache->resident_bytes = 0;
}
