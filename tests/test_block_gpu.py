"""Stacked decoder feed-forward sub-layers (RMSNorm, MoE layer, residual add) against the oracle.

Each block is DeepSeekRunner::Impl::forward's feed-forward half
(src/DeepSeekRunner.cpp:264-290): normalised = rms_norm(hidden, weight) with the sum
of squares in double, feed_forward_output = MoE(normalised), hidden += output.
On the GPU that is lm_moe_block_forward: the router reads the f32 normalised
activations, the experts read them rounded to bf16, and the down projection adds
straight into the residual.  Parity uses the criteria of tests/parity.py on the
final hidden state, and the routing of every layer must match.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import synthetic as syn  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer  # noqa: E402
from oracle.oracle import RouterConfig  # noqa: E402
from tests.parity import MAX_REL, MIN_COS, output_errors  # noqa: E402

SMALL = syn.MoeShape(hidden=256, inter=128, n_routed_experts=16, n_shared_experts=2, top_k=4)


def oracle_block(oracle_lib, shape, W, norm, hidden, eps=1e-6):
    """One sub-layer on the CPU: returns (increment y, idx, w, logits)."""
    xn = np.stack([oracle_lib.rms_norm(row, norm, eps) for row in hidden])
    return oracle_lib.moe_layer(xn, W, RouterConfig(shape.n_routed_experts, shape.top_k), shape.n_shared_experts,
                                threads=0)


# T >= 2048 routes the f32 activations through the tiled router kernel with its
# hidden axis split over CTAs.
@pytest.mark.parametrize("shape_name,layers,T", [("small", 3, 50), ("small", 2, 300), ("v2lite", 2, 24),
                                                 ("small", 1, 2500)])
def test_block_stack_matches_oracle(oracle_lib, shape_name, layers, T):
    """Each layer from the same input: the oracle gets the GPU's hidden state before
    the layer (a stack of layers would otherwise compare routings of inputs that have
    already drifted apart by the bf16 expert activations)."""
    shape = SMALL if shape_name == "small" else syn.V2_LITE
    std = 0.1 if shape_name == "small" else 0.02
    weights = [syn.layer_weights(shape, seed=4, layer=l, std=std) for l in range(layers)]
    rng = np.random.default_rng(44)
    norms = [(1.0 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32) for _ in range(layers)]
    hidden0 = rng.standard_normal((T, shape.hidden)).astype(np.float32)

    layer = MoeLayer(MoeConfig.from_shape(shape, num_layers=layers, max_tokens=max(T, 32)))
    for l in range(layers):
        layer.upload_layer(l, weights[l], norm_weight=norms[l])
    hidden = torch.from_numpy(hidden0.copy()).cuda()
    for l in range(layers):
        before = hidden.cpu().numpy()
        layer.block_forward(l, hidden)
        layer.sync()
        counts = layer.expert_counts()
        increment = hidden.cpu().numpy() - before
        y, idx, w, logits = oracle_block(oracle_lib, shape, weights[l], norms[l], before)
        ref_counts = np.bincount(idx.reshape(-1), minlength=shape.n_routed_experts)
        # A near-tie may swap one token's last choice between two experts.
        assert np.abs(counts - ref_counts).sum() <= 2, f"layer {l}: expert histogram {counts} vs {ref_counts}"
        if np.array_equal(counts, ref_counts):
            rel, cos = output_errors(increment, y)
            assert rel.max() <= MAX_REL, f"layer {l}: max relative error {rel.max():.3e}"
            assert cos.min() >= MIN_COS, f"layer {l}: min cosine {cos.min():.7f}"
            print(f"{shape_name} layer {l} T={T}: max_rel {rel.max():.2e} min_cos {cos.min():.7f}")
