// MoeLayer.hpp -- the MoE feed-forward block of DeepSeekRunner::Impl::forward
// (src/DeepSeekRunner.cpp:264-290 of the reference) for T tokens on one B200, as an
// owning C++ object over the C ABI in litemind_moe.h.  Every method throws
// litemind::b200::Error with the library's message when the call fails, matching
// the reference's exception-based error reporting at its C++ boundary.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "litemind_moe.h"

namespace litemind::b200 {

class Error final : public std::runtime_error {
public:
    Error(lm_status status, const std::string& message) : std::runtime_error(message), status_(status) {}
    [[nodiscard]] lm_status status() const noexcept { return status_; }

private:
    lm_status status_;
};

class MoeLayer final {
public:
    /** Takes the MoE fields of any Config-like object (litemind::Config included). */
    template <class ConfigLike>
    MoeLayer(const ConfigLike& c, int device, int32_t num_layers, int32_t max_tokens) {
        lm_moe_config cfg;
        lm_moe_config_default(&cfg);
        cfg.hidden_size = static_cast<int32_t>(c.hidden_size);
        cfg.moe_intermediate_size = static_cast<int32_t>(c.moe_intermediate_size);
        cfg.n_routed_experts = static_cast<int32_t>(c.n_routed_experts);
        cfg.n_shared_experts = static_cast<int32_t>(c.n_shared_experts);
        cfg.num_experts_per_tok = static_cast<int32_t>(c.num_experts_per_tok);
        cfg.norm_topk_prob = c.norm_topk_prob ? 1 : 0;
        cfg.routed_scaling_factor = c.routed_scaling_factor;
        cfg.topk_method = c.topk_method == "group_limited_greedy" ? LM_TOPK_GROUP_LIMITED_GREEDY : LM_TOPK_GREEDY;
        cfg.n_group = static_cast<int32_t>(c.n_group);
        cfg.topk_group = static_cast<int32_t>(c.topk_group);
        cfg.rms_norm_eps = c.rms_norm_eps;
        cfg.num_layers = num_layers;
        cfg.max_tokens = max_tokens;
        create(cfg, device);
    }
    MoeLayer(const lm_moe_config& cfg, int device) { create(cfg, device); }
    ~MoeLayer() { lm_moe_destroy(ctx_); }
    MoeLayer(const MoeLayer&) = delete;
    MoeLayer& operator=(const MoeLayer&) = delete;
    MoeLayer(MoeLayer&& o) noexcept
        : ctx_(std::exchange(o.ctx_, nullptr)), routed_experts_(std::exchange(o.routed_experts_, 0)) {}
    MoeLayer& operator=(MoeLayer&& o) noexcept {
        std::swap(ctx_, o.ctx_);
        std::swap(routed_experts_, o.routed_experts_);
        return *this;
    }

    void upload_layer(int32_t layer, const float* router, const uint16_t* gate, const uint16_t* up,
                      const uint16_t* down, const uint16_t* shared_gate, const uint16_t* shared_up,
                      const uint16_t* shared_down, const float* norm_weight = nullptr) {
        check(lm_moe_upload_layer(ctx_, layer, router, gate, up, down, shared_gate, shared_up, shared_down,
                                  norm_weight));
    }
    void upload_expert(int32_t layer, int32_t expert, const uint16_t* gate, const uint16_t* up,
                       const uint16_t* down) {
        check(lm_moe_upload_expert(ctx_, layer, expert, gate, up, down));
    }
    /** Layer slot `layer` from SafeTensors shards, tensors model.layers.{checkpoint_layer}.* */
    void load_safetensors(int32_t layer, const std::vector<std::string>& shards, int32_t checkpoint_layer) {
        std::vector<const char*> paths;
        paths.reserve(shards.size());
        for (const std::string& p : shards) paths.push_back(p.c_str());
        check(lm_moe_load_safetensors(ctx_, layer, checkpoint_layer, paths.data(), static_cast<int32_t>(paths.size())));
    }

    // Dense feed-forward layers (their own index space): DeepSeek's first layer.
    void ffn_upload(int32_t layer, int32_t intermediate, const uint16_t* gate, const uint16_t* up,
                    const uint16_t* down, const float* norm_weight = nullptr) {
        check(lm_ffn_upload(ctx_, layer, intermediate, gate, up, down, norm_weight));
    }
    void ffn_load_safetensors(int32_t layer, const std::vector<std::string>& shards, int32_t checkpoint_layer,
                              int32_t intermediate) {
        std::vector<const char*> paths;
        paths.reserve(shards.size());
        for (const std::string& p : shards) paths.push_back(p.c_str());
        check(lm_ffn_load_safetensors(ctx_, layer, checkpoint_layer, intermediate, paths.data(),
                                      static_cast<int32_t>(paths.size())));
    }
    void ffn_forward(int32_t layer, const uint16_t* x, int32_t tokens, float* y, bool accumulate = false,
                     void* stream = nullptr) {
        check(lm_ffn_forward(ctx_, layer, x, tokens, y, accumulate ? 1 : 0, stream));
    }
    /** hidden (device f32 [T, H]) += FFN(rms_norm(hidden)). */
    void ffn_block_forward(int32_t layer, float* hidden, int32_t tokens, void* stream = nullptr) {
        check(lm_ffn_block_forward(ctx_, layer, hidden, tokens, stream));
    }
    /** x device bf16 [T, H] -> y device f32 [T, H] (asynchronous on `stream`). */
    void forward(int32_t layer, const uint16_t* x, int32_t tokens, float* y, bool accumulate = false,
                 const float* logit_bias = nullptr, void* stream = nullptr) {
        check(lm_moe_forward(ctx_, layer, x, tokens, logit_bias, y, accumulate ? 1 : 0, stream));
    }
    /** Host buffers in and out; returns when y_host is written. */
    void forward_host(int32_t layer, const uint16_t* x_host, int32_t tokens, float* y_host,
                      const float* logit_bias_host = nullptr) {
        check(lm_moe_forward_host(ctx_, layer, x_host, tokens, logit_bias_host, y_host));
    }
    /** hidden (device f32 [T, H]) += MoE(rms_norm(hidden)). */
    void block_forward(int32_t layer, float* hidden, int32_t tokens, void* stream = nullptr) {
        check(lm_moe_block_forward(ctx_, layer, hidden, tokens, stream));
    }
    void route(int32_t layer, const uint16_t* x, int32_t tokens, int32_t* topk_idx, float* topk_w,
               const float* logit_bias = nullptr, float* logits = nullptr, void* stream = nullptr) {
        check(lm_moe_route(ctx_, layer, x, tokens, logit_bias, topk_idx, topk_w, logits, stream));
    }
    void ep_init(const void* nccl_unique_id, int32_t rank, int32_t nranks) {
        check(lm_moe_ep_init(ctx_, nccl_unique_id, rank, nranks));
    }
    /** A fresh 128-byte NCCL id for ep_init (rank 0 makes it and shares it). */
    static std::vector<char> ep_unique_id() {
        std::vector<char> id(128);
        const lm_status st = lm_moe_ep_unique_id(id.data());
        if (st != LM_OK) throw Error(st, std::string("lm_moe_ep_unique_id: ") + lm_status_string(st));
        return id;
    }
    void sync(void* stream = nullptr) { check(lm_moe_sync(ctx_, stream)); }

    /** Tokens routed to each routed expert by the last route or forward. */
    [[nodiscard]] std::vector<int32_t> expert_counts() const {
        std::vector<int32_t> counts(static_cast<size_t>(routed_experts_));
        check(lm_moe_expert_counts(ctx_, counts.data(), routed_experts_));
        return counts;
    }
    [[nodiscard]] int32_t routed_experts() const noexcept { return routed_experts_; }
    /** Per-slot device time (ms) and launch counts while profiling (lm_moe_profile_*). */
    void profile(bool enable) { check(lm_moe_profile_enable(ctx_, enable ? 1 : 0)); }
    std::vector<double> profile_read(bool reset = true, std::vector<int64_t>* launches = nullptr) {
        std::vector<double> ms(LM_PROFILE_SLOTS);
        std::vector<int64_t> n(LM_PROFILE_SLOTS);
        check(lm_moe_profile_read(ctx_, ms.data(), n.data(), reset ? 1 : 0));
        if (launches != nullptr) *launches = std::move(n);
        return ms;
    }
    /** Step times of the last profiled chunked expert-parallel forward (empty if none). */
    std::vector<float> profile_ep_timeline() {
        std::vector<float> ms(LM_EP_TIMELINE_MAX);
        int32_t chunks = 0;
        check(lm_moe_profile_ep_timeline(ctx_, ms.data(), LM_EP_TIMELINE_MAX, &chunks));
        ms.resize(chunks > 0 ? static_cast<size_t>(4 * chunks + 2) : 0);
        return ms;
    }

    [[nodiscard]] lm_moe_ctx* handle() const noexcept { return ctx_; }

private:
    void create(const lm_moe_config& cfg, int device) {
        const lm_status st = lm_moe_create(&cfg, device, &ctx_);
        if (st != LM_OK) throw Error(st, std::string("lm_moe_create: ") + lm_status_string(st));
        routed_experts_ = cfg.n_routed_experts;
    }
    void check(lm_status st) const {
        if (st != LM_OK) throw Error(st, lm_moe_last_error(ctx_));
    }

    lm_moe_ctx* ctx_{nullptr};
    int32_t routed_experts_{0};
};

/** The exchange plan of one expert-parallel forward, or of one chunk of it (host only;
 *  lm_moe_ep_plan / lm_moe_ep_chunk_plan).  send counts: [E] this rank's rows per
 *  expert; recv counts: [nranks, E / nranks] rows each rank sends to this rank's experts. */
inline lm_ep_plan ep_plan(int32_t nranks, const std::vector<int32_t>& send_expert_counts,
                          const std::vector<int32_t>& recv_expert_counts, int32_t chunks = 1, int32_t chunk = 0) {
    lm_ep_plan plan{};
    if (send_expert_counts.size() != recv_expert_counts.size())
        throw Error(LM_ERR_INVALID_ARGUMENT, "ep_plan: send and receive counts differ in length");
    const auto experts = static_cast<int32_t>(send_expert_counts.size());
    const lm_status st = lm_moe_ep_chunk_plan(nranks, experts, chunks, chunk, send_expert_counts.data(),
                                              recv_expert_counts.data(), &plan);
    if (st != LM_OK) throw Error(st, std::string("lm_moe_ep_chunk_plan: ") + lm_status_string(st));
    return plan;
}

}  // namespace litemind::b200
