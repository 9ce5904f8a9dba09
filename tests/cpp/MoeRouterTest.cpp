// MoeRouterTest.cpp -- the reference's routing checks (tests/MoeRouterSamplerTest.cpp:
// 26-93) against litemind::b200::MoeRouter, which routes on the GPU.  The router is
// built from a Config-like struct with the reference's field names, as
// DeepSeekRunner builds its router from litemind::Config.
#include <cmath>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include "Expect.hpp"
#include "litemind_b200/MoeRouter.hpp"

namespace {

struct Config {  // the fields of include/Config.hpp:59-71 that MoeRouter reads
    std::size_t n_routed_experts{8U};
    std::size_t num_experts_per_tok{3U};
    bool norm_topk_prob{false};
    float routed_scaling_factor{1.0F};
    std::string topk_method{"greedy"};
    std::size_t n_group{1U};
    std::size_t topk_group{1U};
};

}  // namespace

int main() {
    Expect expect("MoeRouterTest (B200)");
    using litemind::b200::MoeRouter;
    const std::vector<float> logits{0.0F, 5.0F, 1.0F, 4.0F, 2.0F, 3.0F, -1.0F, -2.0F};
    const Config lite{};
    const MoeRouter router(lite);
    const auto selection = router.select(logits);
    expect(selection.size() == 3U, "three experts are selected");
    expect(selection.size() == 3U && selection[0].expert_index == 1U, "the highest logit is chosen first");
    expect(selection.size() == 3U && selection[1].expert_index == 3U, "the second highest follows");
    expect(selection.size() == 3U && selection[2].expert_index == 5U, "the third highest follows");
    if (selection.size() == 3U) {
        expect(selection[0].weight > selection[1].weight, "weights follow the score order");
        const double total = selection[0].weight + selection[1].weight + selection[2].weight;
        expect(total < 1.0 && total > 0.5, "softmax over all experts before the cut");
        double denominator = 0.0;
        for (const float v : logits) denominator += std::exp(static_cast<double>(v) - 5.0);
        expect.near(selection[0].weight, 1.0 / denominator, 1e-6, "the top weight is the full-softmax probability");
    }

    Config normalising = lite;
    normalising.norm_topk_prob = true;
    const auto normalised = MoeRouter(normalising).select(logits);
    expect.near(normalised[0].weight + normalised[1].weight + normalised[2].weight, 1.0, 1e-5,
                "normalised weights sum to one");

    Config scaled = lite;
    scaled.routed_scaling_factor = 2.0F;
    const auto scaled_selection = MoeRouter(scaled).select(logits);
    expect.near(scaled_selection[0].weight, selection[0].weight * 2.0, 1e-6, "the scaling factor multiplies");

    Config both = lite;
    both.norm_topk_prob = true;
    both.routed_scaling_factor = 2.0F;
    const auto both_selection = MoeRouter(both).select(logits);
    expect.near(both_selection[0].weight + both_selection[1].weight + both_selection[2].weight, 1.0, 1e-5,
                "normalisation wins over the scaling factor");

    Config grouped = lite;
    grouped.topk_method = "group_limited_greedy";
    grouped.n_group = 2U;
    grouped.topk_group = 1U;
    grouped.num_experts_per_tok = 2U;
    const auto grouped_selection = MoeRouter(grouped).select(logits);
    expect(grouped_selection.size() == 2U, "group-limited routing still selects top-k");
    for (const auto& choice : grouped_selection) expect(choice.expert_index < 4U, "stays in the winning group");

    const auto legacy = MoeRouter::select_top_k(logits, 8U, 3U, true);
    expect.near(legacy[0].weight + legacy[1].weight + legacy[2].weight, 1.0, 1e-5, "select_top_k normalises");
    bool threw = false;
    try {
        (void)MoeRouter::select_top_k(logits, 8U, 9U, false);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    expect(threw, "select_top_k rejects top_k > experts with std::invalid_argument");
    expect(router.select(std::vector<float>(7U, 0.0F)).empty(), "a wrong logit count gives an empty selection");

    // Ties: equal probabilities go to the lower index.
    const auto tied = MoeRouter(lite).select(std::vector<float>(8U, 0.5F));
    expect(tied.size() == 3U && tied[0].expert_index == 0U && tied[1].expert_index == 1U && tied[2].expert_index == 2U,
          "equal logits select the lowest indices in order");
    return expect.finish();
}
