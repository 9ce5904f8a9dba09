/*
 * moe_oracle.h -- CPU restatement of LiteMind's MoE feed-forward path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * litemind_b200: only tests/, __graft_entry__.smoke() and the cpu_baseline leg of
 * bench.py may load it.  Nothing in the product links or calls it.
 *
 * Every function restates one piece of the reference (ragavanperarasu/LiteMind),
 * cited as file:line relative to the reference checkout.  The arithmetic order of
 * the reference's compiled AVX2+FMA build is reproduced (four 8-lane FMA
 * accumulators, the same horizontal sum, fused multiply-adds where GCC contracts
 * `a += b * c`), so on the same inputs this oracle is bit-identical to the
 * reference's own code built from its sources by oracle/Makefile into oracle/_ref.
 * The pin is tested in tests/test_oracle_pin.py against that build and against
 * the golden vectors in tests/golden/.
 */
#ifndef LITEMIND_MOE_ORACLE_H
#define LITEMIND_MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* bf16 helpers: widen by shifting (src/Gemm.cpp:18-20), round to nearest even
 * as tests/KernelTest.cpp:15-20 does. */
float orc_bf16_to_f32(uint16_t bits);
uint16_t orc_f32_to_bf16(float value);

/* Dense kernels, src/Gemm.cpp. */
float orc_dot(const float* left, const float* right, size_t count);              /* :183-189 */
float orc_dot_bf16(const uint16_t* weights, const float* input, size_t count);  /* :46-102  */
void orc_matvec_f32(const float* weights, const float* input, float* out,
                    size_t out_dim, size_t in_dim);                              /* :132-137 */
void orc_matvec_bf16(const uint16_t* weights, const float* input, float* out,
                     size_t out_dim, size_t in_dim);                             /* :139-154 */
void orc_matvec_bf16_accumulate(const uint16_t* weights, const float* input, float* out,
                                size_t out_dim, size_t in_dim, float scale);     /* :156-175 */
void orc_axpy(float scale, const float* source, float* destination, size_t count); /* :191-195 */
void orc_rms_norm(float* values, const float* weight, size_t count, float epsilon); /* :197-207 */
void orc_softmax(float* values, size_t count);                                   /* :209-223 */
void orc_silu_multiply(const float* gate, const float* up, float* destination,
                       size_t count);                                            /* :225-231 */

/* Router configuration, the fields MoeRouter latches in its constructor
 * (src/MoeRouter.cpp:38-52). */
typedef struct orc_router {
    int64_t expert_count;
    int64_t top_k;
    int64_t n_group;
    int64_t topk_group;
    int32_t group_limited;
    int32_t normalize;
    float routed_scaling_factor;
} orc_router;

/* MoeRouter::MoeRouter(const Config&), src/MoeRouter.cpp:38-52, including the
 * fall-back to greedy routing when n_group does not divide the experts. */
void orc_router_init(orc_router* router, int64_t n_routed_experts, int64_t num_experts_per_tok,
                     int64_t n_group, int64_t topk_group, int32_t group_limited_greedy,
                     int32_t norm_topk_prob, float routed_scaling_factor);

/* MoeRouter::select, src/MoeRouter.cpp:54-107.  Writes up to top_k selections in
 * the reference's order (descending weight, lower index first on ties) and
 * returns how many were written; 0 when the logit count does not match, as the
 * reference returns an empty selection (:57-59). */
int64_t orc_router_select(const orc_router* router, const float* logits, int64_t count,
                          int64_t* expert_index, float* weight);

/* MoeRouter::select_top_k, src/MoeRouter.cpp:115-133.  Returns -1 where the
 * reference throws std::invalid_argument (:119-121). */
int64_t orc_select_top_k(const float* logits, int64_t logit_count, int64_t expert_count,
                         int64_t top_k, int32_t normalize, int64_t* expert_index, float* weight);

/* Shape of one MoE layer (include/Config.hpp:59-71). */
typedef struct orc_moe_shape {
    int64_t hidden;        /* hidden_size */
    int64_t inter;         /* moe_intermediate_size */
    int64_t n_shared;      /* n_shared_experts; the shared FFN is inter * n_shared wide */
    orc_router router;
} orc_moe_shape;

/*
 * One MoE feed-forward block over T tokens, as DeepSeekRunner::Impl::forward runs
 * it per token (src/DeepSeekRunner.cpp:268-288) with Impl::feed_forward
 * (src/DeepSeekRunner.cpp:228-240):
 *   logits = matvec_f32(router, x) [+ bias]; select; out = 0;
 *   for each selection (descending weight): out += w * down(silu(gate x) * up x);
 *   then the shared FFN with weight 1.0.
 * The optional per-expert logit bias (may be NULL) is added between the logits and
 * select; the reference has no such input, it is how a skewed expert load is made.
 *
 * Layouts (row-major, bf16 as raw uint16 bits):
 *   x        [T, hidden] f32       router [E, hidden] f32
 *   gate, up [E, inter, hidden]    down   [E, hidden, inter]
 *   sh_gate, sh_up [S, hidden]     sh_down [hidden, S]          S = inter * n_shared
 * Outputs: y [T, hidden] f32 (overwritten), and when non-NULL idx/w [T, top_k]
 * and logits [T, E] (after the bias).
 * Tokens are independent, so threads > 1 splits tokens across OpenMP threads
 * without changing any token's arithmetic.
 */
int orc_moe_layer(const orc_moe_shape* shape, int64_t tokens, const float* x,
                  const float* router, const float* bias,
                  const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                  const uint16_t* sh_gate, const uint16_t* sh_up, const uint16_t* sh_down,
                  float* y, int64_t* idx, float* w, float* logits, int threads);

/*
 * ExpertCache bookkeeping, include/ExpertCache.hpp:29-89 and
 * src/ExpertCache.cpp:5-76: an LRU working set under a byte budget, with the
 * same counters.  Fixed capacity (ORC_CACHE_CAPACITY entries) is enough for tests.
 */
#define ORC_CACHE_CAPACITY 4096
typedef struct orc_expert_cache {
    uint64_t budget_bytes;
    uint64_t resident_bytes;
    uint64_t loads, hits, evictions, bytes_streamed;
    int64_t count;                         /* entries, most recent first */
    uint64_t keys[ORC_CACHE_CAPACITY];
    uint64_t bytes[ORC_CACHE_CAPACITY];
} orc_expert_cache;

void orc_cache_configure(orc_expert_cache* cache, uint64_t budget_bytes);
void orc_cache_touch(orc_expert_cache* cache, uint64_t key, uint64_t block_bytes);
void orc_cache_clear(orc_expert_cache* cache);
uint64_t orc_cache_make_key(uint64_t layer, uint64_t expert);

#ifdef __cplusplus
}
#endif

#endif /* LITEMIND_MOE_ORACLE_H */
