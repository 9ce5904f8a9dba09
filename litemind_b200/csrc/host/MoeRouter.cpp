// MoeRouter.cpp -- litemind::b200::MoeRouter: the reference's MoeRouter contract
// (src/MoeRouter.cpp:38-133) on top of the router_topk kernel via lm_moe_select.
#include "litemind_b200/MoeRouter.hpp"

#include <cuda_runtime.h>

#include <stdexcept>

namespace litemind::b200 {

struct MoeRouter::State {
    lm_moe_ctx* ctx{nullptr};
    int device{0};
    std::size_t selected{0};  // min(top_k, experts): the reference's partial_sort prefix
    float* logits{nullptr};
    int32_t* idx{nullptr};
    float* weights{nullptr};

    ~State() {
        if (ctx != nullptr) {
            cudaSetDevice(device);
            cudaFree(logits);
            cudaFree(idx);
            cudaFree(weights);
            lm_moe_destroy(ctx);
        }
    }
};

MoeRouter::MoeRouter() : MoeRouter(RoutingConfig{}, 0) {}

MoeRouter::MoeRouter(const RoutingConfig& config, int device) : config_(config), state_(std::make_unique<State>()) {
    state_->device = device;
    const std::size_t E = config.n_routed_experts;
    const std::size_t K = config.num_experts_per_tok;
    if (E == 0 || K == 0) return;  // select() then returns nothing, as the reference's does (:57-59)
    state_->selected = K < E ? K : E;
    lm_moe_config cfg;
    lm_moe_config_default(&cfg);
    cfg.hidden_size = 128;  // the router context holds no expert weights
    cfg.moe_intermediate_size = 64;
    cfg.n_shared_experts = 0;
    cfg.n_routed_experts = static_cast<int32_t>(E);
    cfg.num_experts_per_tok = static_cast<int32_t>(state_->selected);
    cfg.norm_topk_prob = config.norm_topk_prob ? 1 : 0;
    cfg.routed_scaling_factor = config.routed_scaling_factor;
    cfg.topk_method = config.topk_method == "group_limited_greedy" ? LM_TOPK_GROUP_LIMITED_GREEDY : LM_TOPK_GREEDY;
    cfg.n_group = static_cast<int32_t>(config.n_group);
    cfg.topk_group = static_cast<int32_t>(config.topk_group);
    cfg.num_layers = 1;
    cfg.max_tokens = 1;
    if (const lm_status st = lm_moe_create(&cfg, device, &state_->ctx); st != LM_OK)
        throw std::runtime_error(std::string("MoeRouter: ") + lm_status_string(st));
    if (cudaMalloc(&state_->logits, E * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&state_->idx, state_->selected * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&state_->weights, state_->selected * sizeof(float)) != cudaSuccess)
        throw std::runtime_error("MoeRouter: device allocation failed");
}

MoeRouter::~MoeRouter() = default;
MoeRouter::MoeRouter(MoeRouter&&) noexcept = default;
MoeRouter& MoeRouter::operator=(MoeRouter&&) noexcept = default;

void MoeRouter::select(std::span<const float> gate_logits, std::vector<ExpertSelection>& selection) const {
    selection.clear();
    if (state_->ctx == nullptr || gate_logits.size() != config_.n_routed_experts) return;
    const std::size_t K = state_->selected;
    cudaSetDevice(state_->device);
    std::vector<int32_t> idx(K);
    std::vector<float> w(K);
    if (cudaMemcpy(state_->logits, gate_logits.data(), gate_logits.size() * sizeof(float), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        lm_moe_select(state_->ctx, state_->logits, 1, state_->idx, state_->weights, nullptr) != LM_OK ||
        cudaMemcpy(idx.data(), state_->idx, K * sizeof(int32_t), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(w.data(), state_->weights, K * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
        throw std::runtime_error("MoeRouter::select: device routing failed");
    selection.reserve(K);
    for (std::size_t i = 0; i < K; ++i) selection.push_back(ExpertSelection{static_cast<std::size_t>(idx[i]), w[i]});
}

std::vector<ExpertSelection> MoeRouter::select(std::span<const float> gate_logits) const {
    std::vector<ExpertSelection> selection;
    select(gate_logits, selection);
    return selection;
}

std::vector<ExpertSelection> MoeRouter::select_top_k(std::span<const float> gate_logits, std::size_t expert_count,
                                                     std::size_t top_k, bool normalize_selected_weights) {
    if (expert_count == 0U || top_k == 0U || top_k > expert_count || gate_logits.size() != expert_count)
        throw std::invalid_argument("MoE routing requires one logit per expert and a valid top-k value.");
    RoutingConfig config;
    config.n_routed_experts = expert_count;
    config.num_experts_per_tok = top_k;
    config.norm_topk_prob = normalize_selected_weights;
    config.routed_scaling_factor = 1.0F;
    config.topk_method = "greedy";
    return MoeRouter(config).select(gate_logits);
}

lm_status MoeRouter::select_device(const float* logits, int32_t tokens, int32_t* topk_idx, float* topk_w,
                                   void* stream) const {
    if (state_->ctx == nullptr) return LM_ERR_INVALID_ARGUMENT;
    return lm_moe_select(state_->ctx, logits, tokens, topk_idx, topk_w, stream);
}

}  // namespace litemind::b200
