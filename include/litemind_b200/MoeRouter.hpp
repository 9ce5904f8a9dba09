// MoeRouter.hpp -- litemind::MoeRouter's interface (include/MoeRouter.hpp:27-55 of the
// reference) with routing on the B200.
//
// select() keeps the reference's contract exactly: softmax over every expert before
// the cut, optional group-limited masking, greedy top-k in descending weight with
// the lower index first on ties, then normalise *or* scale; an empty selection when
// the logit count is wrong (src/MoeRouter.cpp:57-59); select_top_k throws
// std::invalid_argument where the reference does (src/MoeRouter.cpp:119-121).
// select_device() is the batched form the MoE block uses: T tokens of device logits.
//
// Like the reference's router, one object is not safe to use from two threads at once.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <span>
#include <string>
#include <vector>

#include "litemind_moe.h"

namespace litemind::b200 {

/** One routed-expert decision (include/MoeRouter.hpp:12-15). */
struct ExpertSelection final {
    std::size_t expert_index{};
    float weight{};
};

/** The routing fields of the reference's Config (include/Config.hpp:59-71). */
struct RoutingConfig final {
    std::size_t n_routed_experts{64U};
    std::size_t num_experts_per_tok{6U};
    bool norm_topk_prob{false};
    float routed_scaling_factor{1.0F};
    std::string topk_method{"greedy"};
    std::size_t n_group{1U};
    std::size_t topk_group{1U};

    /** Reads the same-named fields of any Config-like object (litemind::Config included). */
    template <class ConfigLike>
    static RoutingConfig from(const ConfigLike& c) {
        RoutingConfig r;
        r.n_routed_experts = c.n_routed_experts;
        r.num_experts_per_tok = c.num_experts_per_tok;
        r.norm_topk_prob = c.norm_topk_prob;
        r.routed_scaling_factor = c.routed_scaling_factor;
        r.topk_method = c.topk_method;
        r.n_group = c.n_group;
        r.topk_group = c.topk_group;
        return r;
    }
};

class MoeRouter final {
public:
    /** DeepSeek-V2-Lite routing on device 0. */
    MoeRouter();
    explicit MoeRouter(const RoutingConfig& config, int device = 0);
    template <class ConfigLike>
    explicit MoeRouter(const ConfigLike& config, int device = 0) : MoeRouter(RoutingConfig::from(config), device) {}
    ~MoeRouter();
    MoeRouter(MoeRouter&&) noexcept;
    MoeRouter& operator=(MoeRouter&&) noexcept;

    /** Selects experts for one token from its router logits (host memory). */
    void select(std::span<const float> gate_logits, std::vector<ExpertSelection>& selection) const;
    [[nodiscard]] std::vector<ExpertSelection> select(std::span<const float> gate_logits) const;

    /** The reference's static entry point; throws std::invalid_argument on bad sizes. */
    [[nodiscard]] static std::vector<ExpertSelection> select_top_k(std::span<const float> gate_logits,
                                                                   std::size_t expert_count, std::size_t top_k,
                                                                   bool normalize_selected_weights);

    /** Batched: logits device f32 [tokens, E] -> idx device int32 [tokens, k], weights f32 [tokens, k]. */
    lm_status select_device(const float* logits, int32_t tokens, int32_t* topk_idx, float* topk_w,
                            void* stream = nullptr) const;

    [[nodiscard]] const RoutingConfig& config() const noexcept { return config_; }

private:
    struct State;
    RoutingConfig config_;
    std::unique_ptr<State> state_;
};

}  // namespace litemind::b200
