// Prefill.hpp -- batched prefill of the feed-forward sub-layers, for
// DeepSeekRunner::generate (src/DeepSeekRunner.cpp:472-482 of the reference).
//
// The reference reads a prompt one position at a time: for each position, every
// layer's attention sub-layer, then its feed-forward sub-layer -- RMSNorm, the dense
// FFN (layers before first_k_dense_replace) or the MoE block, the residual add
// (src/DeepSeekRunner.cpp:242-290).  The feed-forward sub-layer treats each position
// on its own, so once a layer's attention has run for all T prompt positions (a causal
// attention over the prompt does), its feed-forward sub-layer runs for all T positions
// in one call: one cooperative launch up to 256 tokens, the grouped tensor-core GEMMs
// above.  BatchedPrefill drives that loop; the hidden states stay on the device as f32
// [T, hidden], and the caller's attention sub-layer is a callback.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <utility>
#include <vector>

#include "litemind_b200/MoeLayer.hpp"

namespace litemind::b200 {

class BatchedPrefill final {
public:
    /** Where one decoder layer's feed-forward sub-layer lives in the MoeLayer context:
     *  a dense slot (ffn_* calls) or a MoE slot (upload_layer / load_safetensors). */
    struct LayerSlot final {
        bool dense{false};
        int32_t slot{0};
    };

    /** hidden (device f32 [tokens, hidden]) += attention(rms_norm(hidden)) for every prompt
     *  position of `layer`, on `stream`: the caller's attention sub-layer. */
    using Attention = std::function<void(std::size_t layer, float* hidden, int32_t tokens, void* stream)>;

    BatchedPrefill(MoeLayer& ffn, std::vector<LayerSlot> layers) : ffn_(ffn), layers_(std::move(layers)) {}

    /** The reference's layer plan (Config::is_moe_layer): layers before
     *  first_k_dense_replace, and those off the moe_layer_freq grid, are dense; dense
     *  and MoE layers are numbered in their own slot spaces, in layer order. */
    template <class ConfigLike>
    static std::vector<LayerSlot> plan(const ConfigLike& c) {
        std::vector<LayerSlot> out;
        int32_t dense = 0, moe = 0;
        for (std::size_t l = 0; l < static_cast<std::size_t>(c.num_hidden_layers); ++l) {
            const bool is_moe = c.n_routed_experts > 0 && l >= c.first_k_dense_replace &&
                                (c.moe_layer_freq == 0 || l % c.moe_layer_freq == 0);
            out.push_back(is_moe ? LayerSlot{false, moe++} : LayerSlot{true, dense++});
        }
        return out;
    }

    /** Every layer for all `tokens` prompt positions: attention (if given), then the
     *  feed-forward sub-layer in one call.  Asynchronous on `stream`. */
    void run(float* hidden, int32_t tokens, const Attention& attention = {}, void* stream = nullptr) {
        for (std::size_t l = 0; l < layers_.size(); ++l) {
            if (attention) attention(l, hidden, tokens, stream);
            const LayerSlot& s = layers_[l];
            if (s.dense) {
                ffn_.ffn_block_forward(s.slot, hidden, tokens, stream);
            } else {
                ffn_.block_forward(s.slot, hidden, tokens, stream);
            }
        }
    }

    [[nodiscard]] const std::vector<LayerSlot>& layers() const noexcept { return layers_; }

private:
    MoeLayer& ffn_;
    std::vector<LayerSlot> layers_;
};

}  // namespace litemind::b200
