// PrefillTest.cpp -- BatchedPrefill (include/litemind_b200/Prefill.hpp) as
// DeepSeekRunner would drive it for a prompt: the layer plan from a Config-like struct
// with the reference's field names (layer 0 dense, the rest MoE), every layer's
// feed-forward sub-layer loaded from SafeTensors shards, then all T prompt positions
// through every layer, one call per layer.  The attention sub-layer is left out (no
// callback): the pytest driver compares the result with the reference's per-token
// loop of the same sub-layers on the CPU oracle.
//   PrefillTest <tokens> <hidden_in.f32> <hidden_out.f32> <shard>...
#include <cuda_runtime.h>

#include <cstdint>
#include <fstream>
#include <string>
#include <vector>

#include "Expect.hpp"
#include "litemind_b200/MoeLayer.hpp"
#include "litemind_b200/Prefill.hpp"

namespace {

struct Config {  // the fields of the reference's include/Config.hpp that the feed-forward path reads
    std::size_t hidden_size{256U};
    std::size_t intermediate_size{512U};
    std::size_t moe_intermediate_size{128U};
    std::size_t n_routed_experts{16U};
    std::size_t n_shared_experts{2U};
    std::size_t num_experts_per_tok{4U};
    std::size_t num_hidden_layers{3U};
    std::size_t first_k_dense_replace{1U};
    std::size_t moe_layer_freq{1U};
    bool norm_topk_prob{false};
    float routed_scaling_factor{1.0F};
    std::string topk_method{"greedy"};
    std::size_t n_group{1U};
    std::size_t topk_group{1U};
    float rms_norm_eps{1e-6F};
};

}  // namespace

int main(int argc, char** argv) {
    using litemind::b200::BatchedPrefill;
    using litemind::b200::MoeLayer;
    Expect expect("PrefillTest (B200)");
    if (argc < 5) return 2;
    const int32_t T = std::stoi(argv[1]);
    const Config config{};
    const std::vector<std::string> shards(argv + 4, argv + argc);

    const auto plan = BatchedPrefill::plan(config);
    expect(plan.size() == 3U && plan[0].dense && !plan[1].dense && !plan[2].dense, "layer 0 dense, then MoE");
    expect(plan[1].slot == 0 && plan[2].slot == 1, "MoE layers numbered in their own slot space");
    int32_t moe_layers = 0;
    for (const auto& s : plan) moe_layers += s.dense ? 0 : 1;

    MoeLayer ffn(config, /*device=*/0, moe_layers, /*max_tokens=*/T);
    for (std::size_t l = 0; l < plan.size(); ++l) {
        if (plan[l].dense) {
            ffn.ffn_load_safetensors(plan[l].slot, shards, static_cast<int32_t>(l),
                                     static_cast<int32_t>(config.intermediate_size));
        } else {
            ffn.load_safetensors(plan[l].slot, shards, static_cast<int32_t>(l));
        }
    }

    const std::size_t n = static_cast<std::size_t>(T) * config.hidden_size;
    std::vector<float> hidden(n);
    std::ifstream(argv[2], std::ios::binary).read(reinterpret_cast<char*>(hidden.data()),
                                                 static_cast<std::streamsize>(n * sizeof(float)));
    float* dev = nullptr;
    expect(cudaMalloc(&dev, n * sizeof(float)) == cudaSuccess, "device hidden state");
    cudaMemcpy(dev, hidden.data(), n * sizeof(float), cudaMemcpyHostToDevice);

    int calls = 0;
    BatchedPrefill prefill(ffn, plan);
    prefill.run(dev, T, [&](std::size_t, float*, int32_t tokens, void*) { calls += tokens == T ? 1 : 0; });
    expect(calls == 3, "the attention callback ran once per layer over every prompt position");
    ffn.sync();
    cudaMemcpy(hidden.data(), dev, n * sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(dev);
    std::ofstream(argv[3], std::ios::binary).write(reinterpret_cast<const char*>(hidden.data()),
                                                  static_cast<std::streamsize>(n * sizeof(float)));
    return expect.finish();
}
