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
    MoeLayer(MoeLayer&& o) noexcept : ctx_(std::exchange(o.ctx_, nullptr)) {}
    MoeLayer& operator=(MoeLayer&& o) noexcept {
        std::swap(ctx_, o.ctx_);
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
    void sync(void* stream = nullptr) { check(lm_moe_sync(ctx_, stream)); }

    [[nodiscard]] lm_moe_ctx* handle() const noexcept { return ctx_; }

private:
    void create(const lm_moe_config& cfg, int device) {
        const lm_status st = lm_moe_create(&cfg, device, &ctx_);
        if (st != LM_OK) throw Error(st, std::string("lm_moe_create: ") + lm_status_string(st));
    }
    void check(lm_status st) const {
        if (st != LM_OK) throw Error(st, lm_moe_last_error(ctx_));
    }

    lm_moe_ctx* ctx_{nullptr};
};

}  // namespace litemind::b200
