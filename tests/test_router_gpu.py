"""Routing on the GPU against the reference's routing tests and the oracle.

The first group restates tests/MoeRouterSamplerTest.cpp:26-93 of the reference
(same logits, same configurations, same assertions) against litemind_b200's
MoeRouter, which runs the router_topk kernel.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200.moe import MoeConfig, MoeRouter  # noqa: E402
from oracle.oracle import RouterConfig  # noqa: E402

LOGITS = [0.0, 5.0, 1.0, 4.0, 2.0, 3.0, -1.0, -2.0]  # tests/MoeRouterSamplerTest.cpp:30


def lite_routing(**kw) -> MoeConfig:
    base = dict(n_routed_experts=8, num_experts_per_tok=3, norm_topk_prob=False, routed_scaling_factor=1.0,
                topk_method="greedy", n_group=1, topk_group=1, max_tokens=4096)
    base.update(kw)
    return MoeConfig(**base)


def test_greedy_top_k_over_full_softmax():
    sel = MoeRouter(lite_routing()).select(LOGITS)
    assert len(sel) == 3
    assert [s.expert_index for s in sel] == [1, 3, 5]
    assert sel[0].weight > sel[1].weight
    total = sum(s.weight for s in sel)
    assert 0.5 < total < 1.0
    denominator = sum(math.exp(v - 5.0) for v in LOGITS)
    assert abs(sel[0].weight - 1.0 / denominator) <= 1e-6


def test_normalisation_and_scaling_rules():
    base = MoeRouter(lite_routing()).select(LOGITS)
    norm = MoeRouter(lite_routing(norm_topk_prob=True)).select(LOGITS)
    assert abs(sum(s.weight for s in norm) - 1.0) <= 1e-5
    scaled = MoeRouter(lite_routing(routed_scaling_factor=2.0)).select(LOGITS)
    assert abs(scaled[0].weight - 2.0 * base[0].weight) <= 1e-6
    both = MoeRouter(lite_routing(norm_topk_prob=True, routed_scaling_factor=2.0)).select(LOGITS)
    assert abs(sum(s.weight for s in both) - 1.0) <= 1e-5


def test_group_limited_routing_stays_in_winning_group():
    cfg = lite_routing(topk_method="group_limited_greedy", n_group=2, topk_group=1, num_experts_per_tok=2)
    sel = MoeRouter(cfg).select(LOGITS)
    assert len(sel) == 2
    assert all(s.expert_index < 4 for s in sel)


def test_select_top_k_legacy_entry():
    legacy = MoeRouter.select_top_k(LOGITS, 8, 3, True)
    assert abs(sum(s.weight for s in legacy) - 1.0) <= 1e-5
    with pytest.raises(ValueError):
        MoeRouter.select_top_k(LOGITS, 8, 0, False)
    with pytest.raises(ValueError):
        MoeRouter.select_top_k(LOGITS, 8, 9, False)
    with pytest.raises(ValueError):
        MoeRouter.select_top_k(LOGITS[:4], 8, 2, False)


def test_wrong_logit_count_gives_empty_selection():
    assert MoeRouter(lite_routing()).select(LOGITS[:7]) == []


@pytest.mark.parametrize("E,K,group", [(64, 6, None), (8, 3, None), (16, 4, (4, 2)), (64, 6, (8, 3)),
                                       (160, 6, (8, 3)), (256, 8, (8, 4)), (12, 12, None)])
def test_batched_select_matches_oracle(oracle_lib, E, K, group):
    rng = np.random.default_rng(E * 100 + K)
    T = 1000
    logits = (rng.standard_normal((T, E)) * 2).astype(np.float32)
    logits[::3] = np.round(logits[::3])  # exact ties: lower index must win
    logits[1::7, :] = 0.5  # all equal
    for norm, scale in [(False, 1.0), (True, 1.0), (False, 2.5), (True, 3.0)]:
        kw = dict(n_routed_experts=E, num_experts_per_tok=K, norm_topk_prob=norm, routed_scaling_factor=scale,
                  max_tokens=T)
        rc = RouterConfig(E, K, 1, 1, False, norm, scale)
        if group is not None:
            kw.update(topk_method="group_limited_greedy", n_group=group[0], topk_group=group[1])
            rc = RouterConfig(E, K, group[0], group[1], True, norm, scale)
        router = MoeRouter(MoeConfig(**kw))
        idx, w = router.select_batch(torch.from_numpy(logits).cuda())
        torch.cuda.synchronize()
        idx, w = idx.cpu().numpy(), w.cpu().numpy()
        for t in range(T):
            ri, rw = oracle_lib.router_select(logits[t], rc)
            # Same f32 logits in, so only the softmax's summation order differs:
            # probabilities may move by an ulp, never across a 1e-6 gap.
            if not np.array_equal(idx[t], ri):
                p = np.exp(logits[t].astype(np.float64) - logits[t].max())
                p /= p.sum()
                for a, b in zip(idx[t], ri):
                    assert abs(p[a] - p[b]) <= 1e-6, (t, idx[t], ri)
            np.testing.assert_allclose(w[t], rw, rtol=1e-5, atol=1e-8)  # softmax sums of up to 256 terms
