"""The expert-parallel exchange on ONE B200: an expert-parallel context of one rank
(LITEMIND_B200_EP_SINGLE=1 at lm_moe_ep_init) runs the whole exchange path -- routing
over all experts, the row counts and rows through NCCL (sending to itself), the
expert-major sort, the grouped GEMMs on the received rows, the return and the weighted
combine -- where a plain one-rank context would take the local path.  Its outputs must
match the oracle's MoE block, in the fixed-block mode (small batches: ep_pack_kernel,
ep_schedule_kernel, ep_sort_rows_kernel with a fixed source stride) and the
host-planned mode, in one piece or in chunks of local experts.  The 2-GPU tests cover
the exchange between ranks; these need one GPU.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import synthetic as syn  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor  # noqa: E402
from oracle.oracle import RouterConfig  # noqa: E402
from tests.parity import assert_layer_parity  # noqa: E402

SMALL = syn.MoeShape(hidden=256, inter=128, n_routed_experts=8, n_shared_experts=1, top_k=2)


def _ep_layer(monkeypatch, shape, max_tokens, chunks, W):
    monkeypatch.setenv("LITEMIND_B200_EP_SINGLE", "1")
    monkeypatch.setenv("LITEMIND_B200_EP_CHUNKS", str(chunks))
    layer = MoeLayer(MoeConfig.from_shape(shape, max_tokens=max_tokens), device=0)
    layer.ep_init(MoeLayer.ep_unique_id(), 0, 1)
    layer.upload_layer(0, W)
    return layer


# (37, 64): 64 x min(2, 8) = 128 rows per rank pair, the fixed-block exchange.
# (5000, 5000): 10000 rows exceed the fixed blocks' limit, so the host plans the
# exchange: in one piece, or in 4 chunks of 2 local experts.
@pytest.mark.parametrize("T,max_tokens,chunks", [(37, 64, 1), (5000, 5000, 1), (5000, 5000, 4)])
def test_single_rank_exchange_small(oracle_lib, monkeypatch, T, max_tokens, chunks):
    W = syn.layer_weights(SMALL, seed=5, std=0.1)
    layer = _ep_layer(monkeypatch, SMALL, max_tokens, chunks, W)
    try:
        xb = syn.tokens(SMALL, T, seed=T)
        x = bf16_tensor(xb)
        for _ in range(2):  # a second call reuses every exchange buffer
            y = layer.forward(0, x)
            layer.sync()
        idx, w, _ = layer.route(0, x)
        layer.sync()
        counts = layer.expert_counts()
        assert counts.sum() == T * SMALL.top_k
        sample = np.arange(T) if T <= 64 else np.sort(np.random.default_rng(T).choice(T, 64, replace=False))
        xs = syn.bf16_to_f32(xb).reshape(T, -1)[sample]
        ry, ridx, rw, rlog = oracle_lib.moe_layer(xs, W, RouterConfig(SMALL.n_routed_experts, SMALL.top_k),
                                                  SMALL.n_shared_experts, threads=0)
        assert_layer_parity(y.cpu().numpy()[sample], idx.cpu().numpy()[sample], w.cpu().numpy()[sample], ry, ridx,
                            rw, rlog, what=f"one-rank exchange T={T} chunks={chunks}")
    finally:
        layer.close()


def test_single_rank_exchange_v2lite_chunked(oracle_lib, v2lite_weights, monkeypatch):
    """V2-Lite, 2048 tokens (12288 rows: host-planned), in the default 2 chunks of 32
    experts: a sample of tokens against the oracle."""
    T = 2048
    layer = _ep_layer(monkeypatch, syn.V2_LITE, T, 2, v2lite_weights)
    try:
        xb = syn.tokens(syn.V2_LITE, T, seed=4)
        x = bf16_tensor(xb)
        y = layer.forward(0, x)
        idx, w, _ = layer.route(0, x)
        layer.sync()
        sample = np.sort(np.random.default_rng(4).choice(T, 32, replace=False))
        xs = syn.bf16_to_f32(xb).reshape(T, -1)[sample]
        ry, ridx, rw, rlog = oracle_lib.moe_layer(xs, v2lite_weights, RouterConfig(64, 6), 2, threads=0)
        assert_layer_parity(y.cpu().numpy()[sample], idx.cpu().numpy()[sample], w.cpu().numpy()[sample], ry, ridx,
                            rw, rlog, what="one-rank exchange V2-Lite T=2048")
    finally:
        layer.close()
