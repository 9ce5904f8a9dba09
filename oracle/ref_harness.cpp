// ref_harness.cpp -- C entry points onto the reference's own compiled code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's sources, where they lie in the reference checkout, into
// oracle/_ref/libref_litemind.so.  It lets the tests pin the C restatement
// (moe_oracle.c) against the reference itself, and lets bench.py's reference
// arm time the reference's CPU path.  Nothing in the product links it.
//
// The MoE block of DeepSeekRunner::Impl::forward is private to the runner's
// pimpl (include/DeepSeekRunner.hpp:110-112), so ref_moe_layer restates those
// few lines (src/DeepSeekRunner.cpp:228-240 and :268-288) over the reference's
// public gemm:: and MoeRouter API; every arithmetic step runs in reference code.

#include "Config.hpp"
#include "ExpertCache.hpp"
#include "Gemm.hpp"
#include "MoeRouter.hpp"
#include "SafeTensor.hpp"
#include "Tensor.hpp"
#include "Threading.hpp"

#include <algorithm>
#include <bit>
#include <cstdint>
#include <random>
#include <cstring>
#include <memory>
#include <span>
#include <stdexcept>
#include <vector>

using namespace litemind;

namespace {

Config routing_config(int64_t experts, int64_t top_k, int64_t n_group, int64_t topk_group,
                      int32_t group_limited, int32_t normalize, float scale) {
    Config config;
    config.n_routed_experts = static_cast<std::size_t>(experts);
    config.num_experts_per_tok = static_cast<std::size_t>(top_k);
    config.n_group = static_cast<std::size_t>(n_group);
    config.topk_group = static_cast<std::size_t>(topk_group);
    config.topk_method = group_limited != 0 ? "group_limited_greedy" : "greedy";
    config.norm_topk_prob = normalize != 0;
    config.routed_scaling_factor = scale;
    return config;
}

std::unique_ptr<ThreadPool>& shared_pool() {
    static std::unique_ptr<ThreadPool> pool;
    return pool;
}

ThreadPool& pool_with(int threads) {
    auto& pool = shared_pool();
    const std::size_t want = threads <= 0 ? ThreadPool::hardware_threads() : static_cast<std::size_t>(threads);
    if (!pool || pool->worker_count() != want) {
        pool = std::make_unique<ThreadPool>(want);
    }
    return *pool;
}

}  // namespace

extern "C" {

// The inputs tests/KernelTest.cpp:28-51 draws: a 67x253 bf16 matrix (round to
// nearest even of U(-1,1) from std::mt19937(12345)), its widened copy, and the
// U(-1,1) input vector, in the same draw order.
void ref_kerneltest_inputs(float* weights_f32, uint16_t* weights_bf16, float* input) {
    constexpr std::size_t out_dim = 67U, in_dim = 253U;
    std::mt19937 generator(12345U);
    std::uniform_real_distribution<float> distribution(-1.0F, 1.0F);
    for (std::size_t i = 0; i < out_dim * in_dim; ++i) {
        const std::uint32_t bits = std::bit_cast<std::uint32_t>(distribution(generator));
        weights_bf16[i] = static_cast<uint16_t>((bits + 0x7fffU + ((bits >> 16U) & 1U)) >> 16U);
        weights_f32[i] = std::bit_cast<float>(static_cast<std::uint32_t>(weights_bf16[i]) << 16U);
    }
    for (std::size_t i = 0; i < in_dim; ++i) input[i] = distribution(generator);
}

int64_t ref_hardware_threads() { return static_cast<int64_t>(ThreadPool::hardware_threads()); }

const char* ref_kernel_description() {
    static std::string text = gemm::kernel_description();
    return text.c_str();
}

void ref_matvec_bf16(const uint16_t* w, const float* x, float* out, int64_t rows, int64_t cols,
                     int threads) {
    gemm::matvec_bf16(pool_with(threads), w, x, out, static_cast<std::size_t>(rows),
                      static_cast<std::size_t>(cols));
}

void ref_matvec_bf16_serial(const uint16_t* w, const float* x, float* out, int64_t rows, int64_t cols) {
    gemm::matvec_bf16_serial(w, x, out, static_cast<std::size_t>(rows), static_cast<std::size_t>(cols));
}

void ref_matvec_bf16_accumulate(const uint16_t* w, const float* x, float* out, int64_t rows,
                                int64_t cols, float scale, int threads) {
    gemm::matvec_bf16_accumulate(pool_with(threads), w, x, out, static_cast<std::size_t>(rows),
                                 static_cast<std::size_t>(cols), scale);
}

void ref_matvec_f32(const float* w, const float* x, float* out, int64_t rows, int64_t cols) {
    gemm::matvec_f32(w, x, out, static_cast<std::size_t>(rows), static_cast<std::size_t>(cols));
}

void ref_softmax(float* v, int64_t n) { gemm::softmax(v, static_cast<std::size_t>(n)); }

void ref_silu_multiply(const float* g, const float* u, float* d, int64_t n) {
    gemm::silu_multiply(g, u, d, static_cast<std::size_t>(n));
}

void ref_rms_norm(float* v, const float* w, int64_t n, float eps) {
    gemm::rms_norm(v, w, static_cast<std::size_t>(n), eps);
}

void ref_axpy(float scale, const float* src, float* dst, int64_t n) {
    gemm::axpy(scale, src, dst, static_cast<std::size_t>(n));
}

// MoeRouter(Config).select; returns the number of selections written.
int64_t ref_router_select(const float* logits, int64_t count, int64_t experts, int64_t top_k,
                          int64_t n_group, int64_t topk_group, int32_t group_limited,
                          int32_t normalize, float scale, int64_t* idx, float* w) {
    const MoeRouter router(routing_config(experts, top_k, n_group, topk_group, group_limited,
                                          normalize, scale));
    const auto selection = router.select(std::span<const float>(logits, static_cast<std::size_t>(count)));
    for (std::size_t i = 0; i < selection.size(); ++i) {
        idx[i] = static_cast<int64_t>(selection[i].expert_index);
        w[i] = selection[i].weight;
    }
    return static_cast<int64_t>(selection.size());
}

// MoeRouter::select_top_k; returns -1 where the reference throws.
int64_t ref_select_top_k(const float* logits, int64_t count, int64_t experts, int64_t top_k,
                         int32_t normalize, int64_t* idx, float* w) {
    try {
        const auto selection = MoeRouter::select_top_k(
            std::span<const float>(logits, static_cast<std::size_t>(count)),
            static_cast<std::size_t>(experts), static_cast<std::size_t>(top_k), normalize != 0);
        for (std::size_t i = 0; i < selection.size(); ++i) {
            idx[i] = static_cast<int64_t>(selection[i].expert_index);
            w[i] = selection[i].weight;
        }
        return static_cast<int64_t>(selection.size());
    } catch (const std::invalid_argument&) {
        return -1;
    }
}

// The MoE block over T tokens, one token at a time exactly as the runner does.
// Layouts match orc_moe_layer in moe_oracle.h.
int ref_moe_layer(int64_t hidden, int64_t inter, int64_t n_shared, int64_t experts, int64_t top_k,
                  int64_t n_group, int64_t topk_group, int32_t group_limited, int32_t normalize,
                  float scale, int64_t tokens, const float* x, const float* router_w,
                  const float* bias, const uint16_t* gate, const uint16_t* up,
                  const uint16_t* down, const uint16_t* sh_gate, const uint16_t* sh_up,
                  const uint16_t* sh_down, float* y, int64_t* idx, float* w, float* logits_out,
                  int threads) {
    ThreadPool& pool = pool_with(threads);
    const MoeRouter router(routing_config(experts, top_k, n_group, topk_group, group_limited,
                                          normalize, scale));
    const std::size_t H = static_cast<std::size_t>(hidden);
    const std::size_t I = static_cast<std::size_t>(inter);
    const std::size_t S = I * static_cast<std::size_t>(n_shared);
    const std::size_t widest = std::max(I, S);
    const std::size_t expert_elems = I * H;
    std::vector<float> gate_buffer(widest), up_buffer(widest), activation(widest);
    std::vector<float> logits(static_cast<std::size_t>(experts));
    std::vector<ExpertSelection> selection;

    auto feed_forward = [&](const uint16_t* g, const uint16_t* u, const uint16_t* d, std::size_t width,
                            const float* input, float* output, float weight) {
        gemm::matvec_bf16(pool, g, input, gate_buffer.data(), width, H);
        gemm::matvec_bf16(pool, u, input, up_buffer.data(), width, H);
        gemm::silu_multiply(gate_buffer.data(), up_buffer.data(), activation.data(), width);
        gemm::matvec_bf16_accumulate(pool, d, activation.data(), output, H, width, weight);
    };

    for (int64_t t = 0; t < tokens; ++t) {
        const float* xt = x + static_cast<std::size_t>(t) * H;
        float* out = y + static_cast<std::size_t>(t) * H;
        std::fill(out, out + H, 0.0F);
        gemm::matvec_f32(router_w, xt, logits.data(), static_cast<std::size_t>(experts), H);
        if (bias != nullptr) {
            for (std::size_t e = 0; e < logits.size(); ++e) {
                logits[e] = logits[e] + bias[e];
            }
        }
        if (logits_out != nullptr) {
            std::memcpy(logits_out + static_cast<std::size_t>(t) * logits.size(), logits.data(),
                        logits.size() * sizeof(float));
        }
        router.select(logits, selection);
        if (selection.size() != static_cast<std::size_t>(top_k)) {
            return -2;
        }
        for (std::size_t s = 0; s < selection.size(); ++s) {
            const std::size_t e = selection[s].expert_index;
            feed_forward(gate + e * expert_elems, up + e * expert_elems, down + e * expert_elems, I, xt,
                         out, selection[s].weight);
            if (idx != nullptr) {
                idx[static_cast<std::size_t>(t) * selection.size() + s] = static_cast<int64_t>(e);
            }
            if (w != nullptr) {
                w[static_cast<std::size_t>(t) * selection.size() + s] = selection[s].weight;
            }
        }
        if (S != 0U) {
            feed_forward(sh_gate, sh_up, sh_down, S, xt, out, 1.0F);
        }
    }
    return 0;
}

// ExpertCache driven with metadata-only views: no shard, so prefetch/release
// are no-ops (src/WeightStore.cpp:40-50) and only the bookkeeping runs.
struct RefCache {
    ExpertCache cache;
    std::vector<std::unique_ptr<Tensor>> metas;
};

void* ref_cache_new() { return new RefCache(); }
void ref_cache_free(void* handle) { delete static_cast<RefCache*>(handle); }
void ref_cache_configure(void* handle, uint64_t budget) {
    static_cast<RefCache*>(handle)->cache.configure(budget);
}
void ref_cache_touch(void* handle, uint64_t key, uint64_t gate_elems, uint64_t up_elems,
                     uint64_t down_elems) {
    auto* ref = static_cast<RefCache*>(handle);
    auto make = [&](uint64_t elems) {
        ref->metas.push_back(std::make_unique<Tensor>("w", std::vector<std::size_t>{elems},
                                                      DataType::BFloat16, 0U));
        return WeightView{nullptr, ref->metas.back().get(), nullptr};
    };
    ExpertCache::Block block{make(gate_elems), make(up_elems), make(down_elems)};
    ref->cache.touch(key, block);
}
void ref_cache_clear(void* handle) { static_cast<RefCache*>(handle)->cache.clear(); }
void ref_cache_stats(void* handle, uint64_t* out6) {
    const ExpertCache& c = static_cast<RefCache*>(handle)->cache;
    out6[0] = c.resident_bytes();
    out6[1] = c.resident_experts();
    out6[2] = c.loads();
    out6[3] = c.hits();
    out6[4] = c.evictions();
    out6[5] = c.bytes_streamed();
}
uint64_t ref_cache_make_key(uint64_t layer, uint64_t expert) {
    return ExpertCache::make_key(static_cast<std::size_t>(layer), static_cast<std::size_t>(expert));
}

// SafeTensor::open + find (src/SafeTensor.cpp:87-157) on one shard: 0 found, 1 the
// shard was rejected (message in err), 2 no such tensor.  dtype: 1 BF16, 2 F16,
// 3 F32, 4 any other known type (the codes of lm_safetensors_info).
int ref_safetensor_info(const char* path, const char* name, int32_t* dtype, int32_t* ndim, int64_t* shape,
                        uint64_t* offset, uint64_t* nbytes, char* err, int32_t err_len) {
    SafeTensor shard;
    std::string error;
    if (!shard.open(path, error)) {
        if (err != nullptr && err_len > 0) {
            const size_t n = std::min(error.size(), static_cast<size_t>(err_len - 1));
            std::memcpy(err, error.data(), n);
            err[n] = '\0';
        }
        return 1;
    }
    const Tensor* t = shard.find(name);
    if (t == nullptr) return 2;
    switch (t->data_type()) {
        case DataType::BFloat16: *dtype = 1; break;
        case DataType::Float16: *dtype = 2; break;
        case DataType::Float32: *dtype = 3; break;
        default: *dtype = 4; break;
    }
    *ndim = static_cast<int32_t>(t->shape().size());
    for (size_t i = 0; i < t->shape().size() && i < 8; ++i) shape[i] = static_cast<int64_t>(t->shape()[i]);
    *offset = t->offset();
    *nbytes = t->byte_size();
    return 0;
}

}  // extern "C"
