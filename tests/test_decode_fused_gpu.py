"""The fused decode kernel (one cooperative launch per layer for T <= 256 on one GPU).

Parity against the oracle across the token counts that change its work split: in
direct mode (by default below 16 tokens; up to 32 when forced: one token, a token-tile
boundary, 32) and in gather mode (16-256 tokens: column-tile boundaries at 32, 64, 96,
128 and above, more tokens than CTAs, the largest batch), with a
logit bias, with group-limited and renormalised routing, with accumulation into y,
with f32 router activations (the block path), with gather mode forced down to a
single token, and against the grouped multi-launch path it replaces.  Its phase
trace is checked for ordering in both modes.  The grouped path's single-launch
routing for mid-size batches is checked here the same way.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import synthetic as syn  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor  # noqa: E402
from oracle.oracle import RouterConfig  # noqa: E402
from tests.parity import MAX_REL, MIN_COS, assert_layer_parity, output_errors  # noqa: E402

V2 = syn.V2_LITE
# A shape with enough experts for group-limited routing (8 groups of 8).
GROUPED = syn.MoeShape(hidden=512, inter=256, n_routed_experts=64, n_shared_experts=2, top_k=6)


@pytest.fixture(scope="module")
def v2(v2lite_weights):
    layer = MoeLayer(MoeConfig(max_tokens=256))
    layer.upload_layer(0, v2lite_weights)
    yield layer
    layer.close()


def _layer_with_env(cfg, **env):
    """A context created under the given LITEMIND_B200_* settings (read at creation)."""
    old = {k: os.environ.get(k) for k in env}
    os.environ.update({k: str(v) for k, v in env.items()})
    try:
        return MoeLayer(cfg)
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


def _oracle(oracle_lib, shape, W, x_bits, cfg=None, bias=None):
    x = syn.bf16_to_f32(x_bits).reshape(x_bits.shape)
    cfg = cfg or RouterConfig(shape.n_routed_experts, shape.top_k)
    return oracle_lib.moe_layer(x, W, cfg, shape.n_shared_experts, bias=bias, threads=0)


def _gpu(layer, x_bits, bias=None):
    x = bf16_tensor(x_bits)
    b = None if bias is None else torch.from_numpy(bias).cuda()
    layer.profile(True)
    layer.profile_read(reset=True)
    y = layer.forward(0, x, bias=b)
    prof = layer.profile_read(reset=True)
    layer.profile(False)
    idx, w, logits = layer.route(0, x, bias=b)
    layer.sync()
    return y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), logits.cpu().numpy(), prof


@pytest.mark.parametrize("T", [1, 2, 15, 16, 17, 31, 32])
def test_fused_parity_across_token_counts(oracle_lib, v2lite_weights, v2, T):
    x = syn.tokens(V2, T, seed=50 + T)
    y, idx, w, _, prof = _gpu(v2, x)
    assert "decode_fused" in prof and "gemm_gate_up" not in prof, prof
    ry, ridx, rw, rlog = _oracle(oracle_lib, V2, v2lite_weights, x)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"fused T={T}")


@pytest.mark.parametrize("T", [33, 48, 63, 64, 65, 96, 127, 128, 129, 160, 200, 255, 256])
def test_fused_gather_parity_across_token_counts(oracle_lib, v2lite_weights, v2, T):
    x = syn.tokens(V2, T, seed=150 + T)
    y, idx, w, _, prof = _gpu(v2, x)
    assert "decode_fused" in prof and "gemm_gate_up" not in prof, prof
    ry, ridx, rw, rlog = _oracle(oracle_lib, V2, v2lite_weights, x)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"fused gather T={T}")
    counts = v2.expert_counts()
    assert np.abs(counts - np.bincount(ridx.reshape(-1), minlength=64)).sum() <= 2


def test_fused_gather_forced_at_small_batches(oracle_lib, v2lite_weights):
    """Gather mode (routing once per token, rows gathered, 32-row column tiles) forced
    down to one token: the same parity as direct mode gives."""
    layer = _layer_with_env(MoeConfig(max_tokens=128), LITEMIND_B200_FUSED_GATHER_FROM=1)
    layer.upload_layer(0, v2lite_weights)
    for T in (1, 7, 32):
        x = syn.tokens(V2, T, seed=170 + T)
        y, idx, w, _, prof = _gpu(layer, x)
        assert "decode_fused" in prof
        ry, ridx, rw, rlog = _oracle(oracle_lib, V2, v2lite_weights, x)
        assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"forced gather T={T}")
    layer.close()


def test_fused_direct_forced_up_to_its_limit(oracle_lib, v2lite_weights):
    """Direct mode (every expert reads x itself) kept up to its 32-token limit."""
    layer = _layer_with_env(MoeConfig(max_tokens=128), LITEMIND_B200_FUSED_GATHER_FROM=33)
    layer.upload_layer(0, v2lite_weights)
    for T in (16, 17, 31, 32):
        x = syn.tokens(V2, T, seed=180 + T)
        y, idx, w, _, prof = _gpu(layer, x)
        assert "decode_fused" in prof
        ry, ridx, rw, rlog = _oracle(oracle_lib, V2, v2lite_weights, x)
        assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"forced direct T={T}")
    layer.close()


def test_fused_modes_alternate_on_one_context(oracle_lib, v2lite_weights, v2):
    """Direct and gather launches back to back on one context (the grid counters are
    re-armed by each launch's last CTA), each call's output against the oracle."""
    for T in (128, 96, 8, 128, 32, 40):
        x = syn.tokens(V2, T, seed=190 + T)
        y, idx, w, _, _ = _gpu(v2, x)
        ry, ridx, rw, rlog = _oracle(oracle_lib, V2, v2lite_weights, x)
        assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"alternating T={T}")


def test_fused_gather_with_zipf_bias_and_accumulate(oracle_lib, v2lite_weights, v2):
    x = syn.tokens(V2, 112, seed=2)
    bias = syn.zipf_bias(V2, seed=2)
    y, idx, w, _, _ = _gpu(v2, x, bias)
    ry, ridx, rw, rlog = _oracle(oracle_lib, V2, v2lite_weights, x, bias=bias)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what="fused gather + bias")
    xt = bf16_tensor(x)
    b = torch.from_numpy(bias).cuda()
    y0 = v2.forward(0, xt, bias=b)
    y1 = torch.full_like(y0, -1.0)
    v2.forward(0, xt, bias=b, y=y1, accumulate=True)
    v2.sync()
    torch.testing.assert_close(y1 + 1.0, y0, rtol=1e-5, atol=1e-5)


def test_fused_with_zipf_bias(oracle_lib, v2lite_weights, v2):
    x = syn.tokens(V2, 32, seed=2)
    bias = syn.zipf_bias(V2, seed=2)
    y, idx, w, _, _ = _gpu(v2, x, bias)
    ry, ridx, rw, rlog = _oracle(oracle_lib, V2, v2lite_weights, x, bias=bias)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what="fused + bias")


def test_fused_accumulates(v2):
    x = bf16_tensor(syn.tokens(V2, 20, seed=9))
    y0 = v2.forward(0, x)
    y1 = torch.full_like(y0, 2.0)
    v2.forward(0, x, y=y1, accumulate=True)
    v2.sync()
    torch.testing.assert_close(y1 - 2.0, y0, rtol=1e-5, atol=1e-5)


def test_fused_matches_grouped_path(v2lite_weights, v2):
    """The grouped multi-launch path (LITEMIND_B200_FUSED_DECODE=0) on the same inputs."""
    old = os.environ.get("LITEMIND_B200_FUSED_DECODE")
    os.environ["LITEMIND_B200_FUSED_DECODE"] = "0"
    try:
        grouped = MoeLayer(MoeConfig(max_tokens=128))
    finally:
        if old is None:
            del os.environ["LITEMIND_B200_FUSED_DECODE"]
        else:
            os.environ["LITEMIND_B200_FUSED_DECODE"] = old
    grouped.upload_layer(0, v2lite_weights)
    for T in (1, 8, 32, 64, 128):
        x = syn.tokens(V2, T, seed=70 + T)
        y, _, _, _, _ = _gpu(v2, x)
        counts = v2.expert_counts()
        gy, _, _, _, gprof = _gpu(grouped, x)
        gcounts = grouped.expert_counts()
        assert "decode_fused" not in gprof
        # The two paths sum the router logits in different orders: a near-tie may move
        # one choice; otherwise both routings and outputs agree.
        assert np.abs(counts - gcounts).sum() <= 2
        if np.array_equal(counts, gcounts):
            rel = np.abs(y - gy).max() / np.abs(gy).max()
            assert rel < 1e-2, rel
    grouped.close()


def test_group_limited_routing_large_batch(oracle_lib):
    """Group-limited routing at T >= 2048 takes the CUDA-core tiled router (split over
    the hidden axis) instead of the tensor-core one; sampled tokens against the oracle."""
    W = syn.layer_weights(GROUPED, seed=23, std=0.05)
    cfg = MoeConfig.from_shape(GROUPED, max_tokens=3000, topk_method="group_limited_greedy", n_group=8,
                               topk_group=3)
    layer = MoeLayer(cfg)
    layer.upload_layer(0, W)
    T = 3000
    x = syn.tokens(GROUPED, T, seed=24)
    y, idx, w, _, _ = _gpu(layer, x)
    sample = np.sort(np.random.default_rng(3).choice(T, 64, replace=False))
    rcfg = RouterConfig(64, 6, n_group=8, topk_group=3, group_limited=True)
    ry, ridx, rw, rlog = _oracle(oracle_lib, GROUPED, W, x[sample], cfg=rcfg)
    assert_layer_parity(y[sample], idx[sample], w[sample], ry, ridx, rw, rlog, what="group-limited T=3000")
    layer.close()


@pytest.mark.parametrize("T,normalize", [(24, False), (24, True), (80, False), (128, True)])
def test_fused_group_limited_routing(oracle_lib, T, normalize):
    W = syn.layer_weights(GROUPED, seed=21, std=0.05)
    cfg = MoeConfig.from_shape(GROUPED, max_tokens=128, topk_method="group_limited_greedy", n_group=8,
                               topk_group=3, norm_topk_prob=normalize, routed_scaling_factor=1.0)
    layer = MoeLayer(cfg)
    layer.upload_layer(0, W)
    x = syn.tokens(GROUPED, T, seed=22)
    bias = np.linspace(-0.5, 0.5, GROUPED.n_routed_experts).astype(np.float32)
    y, idx, w, _, prof = _gpu(layer, x, bias=bias)
    assert "decode_fused" in prof
    rcfg = RouterConfig(64, 6, n_group=8, topk_group=3, group_limited=True, norm_topk_prob=normalize)
    ry, ridx, rw, rlog = _oracle(oracle_lib, GROUPED, W, x, cfg=rcfg, bias=bias)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"fused group-limited T={T} normalize={normalize}")
    layer.close()


@pytest.mark.parametrize("experts,T", [(12, 40), (12, 128), (16, 40), (16, 97)])
def test_fused_gather_logit_inputs(oracle_lib, experts, T):
    """Gather mode computes the router logits from inputs each CTA pulls into shared
    memory with bulk copies when its tasks are one token group against 8 consecutive
    experts (expert counts a multiple of 8), and from global memory otherwise: both,
    with partial last token groups, against the oracle."""
    shape = syn.MoeShape(hidden=512, inter=256, n_routed_experts=experts, n_shared_experts=2, top_k=3)
    W = syn.layer_weights(shape, seed=51 + experts, std=0.05)
    layer = MoeLayer(MoeConfig.from_shape(shape, max_tokens=128))
    layer.upload_layer(0, W)
    x = syn.tokens(shape, T, seed=52 + T)
    y, idx, w, _, prof = _gpu(layer, x)
    assert "decode_fused" in prof
    ry, ridx, rw, rlog = _oracle(oracle_lib, shape, W, x, cfg=RouterConfig(experts, 3))
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"fused gather E={experts} T={T}")
    layer.close()


@pytest.mark.parametrize("T,normalize", [(33, False), (100, True), (128, False), (256, True)])
def test_mid_batch_single_launch_routing(oracle_lib, T, normalize):
    """32 < T <= 256 routes in one launch (logits and routing per 32-token block,
    then counts, schedule and rows), then the grouped GEMMs: group-limited routing
    with a logit bias, and the forward's own expert histogram against the oracle's."""
    W = syn.layer_weights(GROUPED, seed=41, std=0.05)
    cfg = MoeConfig.from_shape(GROUPED, max_tokens=256, topk_method="group_limited_greedy", n_group=8,
                               topk_group=3, norm_topk_prob=normalize, routed_scaling_factor=1.0)
    # The fused kernel would take batches up to 128 tokens: keep them on the grouped path.
    layer = _layer_with_env(cfg, LITEMIND_B200_FUSED_MAX_TOKENS=32)
    layer.upload_layer(0, W)
    x = syn.tokens(GROUPED, T, seed=42 + T)
    bias = np.linspace(-0.5, 0.5, GROUPED.n_routed_experts).astype(np.float32)
    y, idx, w, _, prof = _gpu(layer, x, bias=bias)
    assert "route" in prof and "router_topk" not in prof and "decode_fused" not in prof, prof
    rcfg = RouterConfig(64, 6, n_group=8, topk_group=3, group_limited=True, norm_topk_prob=normalize)
    ry, ridx, rw, rlog = _oracle(oracle_lib, GROUPED, W, x, cfg=rcfg, bias=bias)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"mid-batch route T={T}")
    counts = layer.expert_counts()
    ref_counts = np.bincount(ridx.reshape(-1), minlength=GROUPED.n_routed_experts)
    assert np.abs(counts - ref_counts).sum() <= 2, (counts, ref_counts)
    layer.close()


@pytest.mark.parametrize("T", [12, 72])
def test_fused_block_forward(oracle_lib, T):
    """RMSNorm -> MoE -> residual with the router on the f32 normalised activations."""
    shape = syn.MoeShape(hidden=512, inter=256, n_routed_experts=16, n_shared_experts=2, top_k=4)
    W = syn.layer_weights(shape, seed=31, std=0.05)
    norm = np.linspace(0.5, 1.5, shape.hidden).astype(np.float32)
    layer = MoeLayer(MoeConfig.from_shape(shape, max_tokens=128))
    layer.upload_layer(0, W, norm_weight=norm)
    hidden0 = np.random.default_rng(32).standard_normal((T, shape.hidden)).astype(np.float32)
    hidden = torch.from_numpy(hidden0.copy()).cuda()
    layer.profile(True)
    layer.profile_read(reset=True)
    layer.block_forward(0, hidden)
    prof = layer.profile_read(reset=True)
    layer.profile(False)
    layer.sync()
    assert "decode_fused" in prof
    xn = np.stack([oracle_lib.rms_norm(row, norm, 1e-6) for row in hidden0])
    y, idx, _, _ = oracle_lib.moe_layer(xn, W, RouterConfig(shape.n_routed_experts, shape.top_k),
                                        shape.n_shared_experts, threads=0)
    counts = layer.expert_counts()
    ref_counts = np.bincount(idx.reshape(-1), minlength=shape.n_routed_experts)
    assert np.abs(counts - ref_counts).sum() <= 2
    if np.array_equal(counts, ref_counts):
        rel, cos = output_errors(hidden.cpu().numpy() - hidden0, y)
        assert rel.max() <= MAX_REL and cos.min() >= MIN_COS, (rel.max(), cos.min())
    layer.close()


def test_fused_phase_trace_is_ordered(v2):
    x = bf16_tensor(syn.tokens(V2, 8, seed=3))
    v2.profile(True)
    v2.forward(0, x)
    tr = v2.profile_trace().astype(np.int64)
    v2.profile(False)
    v2.sync()
    assert tr.shape[0] == torch.cuda.get_device_properties(0).multi_processor_count
    start, logits, seen, sched, gate_up, down = (tr[:, k] for k in (0, 1, 2, 3, 4, 7))
    for a, b in ((start, logits), (logits, seen), (seen, sched), (sched, gate_up), (gate_up, down)):
        assert (a > 0).all() and (b >= a).all()
    # No CTA leaves routing before the last CTA has written its logits (each CTA
    # stamps "written" just after its arrival, hence the slack).
    assert seen.min() >= logits.max() - 2000


def test_fused_gather_phase_trace_is_ordered(v2):
    x = bf16_tensor(syn.tokens(V2, 128, seed=4))
    v2.profile(True)
    v2.forward(0, x)
    tr = v2.profile_trace().astype(np.int64)
    v2.profile(False)
    v2.sync()
    start, logits, seen, topk, topk_seen, sched, gathered, gate_up, down = (
        tr[:, k] for k in (0, 1, 2, 9, 13, 3, 14, 4, 7))
    for a, b in ((start, logits), (logits, seen), (seen, topk), (topk, topk_seen), (topk_seen, sched),
                 (sched, gathered), (gathered, gate_up), (gate_up, down)):
        assert (a > 0).all() and (b >= a).all()
    assert topk_seen.min() >= topk.max() - 2000
