"""Expert-parallel host logic on CPU: two gloo ranks run the exchange protocol of
lm_moe_forward's expert-parallel path around lm_moe_ep_plan (the library's own
plan function) and must reproduce the single-process oracle.

Each rank routes its own tokens with the oracle, orders its (token, slot) rows by
expert (token order within an expert, as the place kernel does), exchanges the
per-expert counts, asks lm_moe_ep_plan for the send/recv counts and offsets, sends
the rows with all_to_all_single, computes its local experts, returns the outputs in
receive order, and combines them by slot with the routing weights, plus the shared
experts.  No GPU is used.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from litemind_b200 import synthetic as syn

SHAPE = syn.MoeShape(hidden=64, inter=32, n_routed_experts=8, n_shared_experts=1, top_k=3)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ffn(gate, up, down, x):
    """One SwiGLU expert in float64 (rows of x)."""
    g = x @ gate.T
    u = x @ up.T
    h = g / (1.0 + np.exp(-g)) * u
    return h @ down.T


def _worker(rank, world, port, token_counts):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from litemind_b200.moe import ep_plan
        from oracle.oracle import Oracle, RouterConfig

        orc = Oracle()
        W = syn.layer_weights(SHAPE, seed=3, std=0.1)
        Wf = {k: (syn.bf16_to_f32(v).reshape(v.shape).astype(np.float64) if v.dtype == np.uint16 else v)
              for k, v in W.items()}
        E, K, H = SHAPE.n_routed_experts, SHAPE.top_k, SHAPE.hidden
        El = E // world
        T = token_counts[rank]
        x = syn.bf16_to_f32(syn.tokens(SHAPE, max(T, 1), seed=10 + rank)).reshape(-1, H)[:T]
        cfg = RouterConfig(E, K)
        if T > 0:
            ref_y, idx, w, _ = orc.moe_layer(x, W, cfg, SHAPE.n_shared_experts)
        else:
            ref_y, idx, w = np.zeros((0, H), np.float32), np.zeros((0, K), np.int64), np.zeros((0, K), np.float32)
        # Send order: by expert, then (token, slot) order.
        pairs = [(int(idx[t, s]), t, s) for t in range(T) for s in range(K)]
        order = sorted(range(len(pairs)), key=lambda i: (pairs[i][0], i))
        slot_row = np.zeros(T * K, np.int64)
        for row, i in enumerate(order):
            slot_row[i] = row
        send_rows = np.array([x[pairs[i][1]] for i in order], np.float64).reshape(-1, H)
        send_expert = np.array([pairs[i][0] for i in order], np.int64)
        counts = np.bincount(idx.reshape(-1), minlength=E).astype(np.int32)
        recv_counts = torch.zeros(E, dtype=torch.int32)
        dist.all_to_all_single(recv_counts, torch.from_numpy(counts))  # El per peer
        plan = ep_plan(world, counts, recv_counts.numpy())
        assert plan["n_send"] == T * K
        assert plan["send_offset"][0] == 0 and plan["recv_offset"][0] == 0
        # Rows and their experts to the experts' ranks.
        recv_x = torch.zeros((plan["n_recv"], H), dtype=torch.float64)
        dist.all_to_all_single(recv_x, torch.from_numpy(send_rows), plan["recv_count"], plan["send_count"])
        recv_e = torch.zeros(plan["n_recv"], dtype=torch.int64)
        dist.all_to_all_single(recv_e, torch.from_numpy(send_expert), plan["recv_count"], plan["send_count"])
        # Received rows are grouped by source, each source's rows by local expert.
        rc = recv_counts.numpy().reshape(world, El)
        for src in range(world):
            seg = recv_e.numpy()[plan["recv_offset"][src]:plan["recv_offset"][src] + plan["recv_count"][src]]
            assert np.array_equal(seg, np.repeat(rank * El + np.arange(El), rc[src]))
        out = np.zeros((plan["n_recv"], H))
        for r in range(plan["n_recv"]):
            e = int(recv_e[r])
            assert rank * El <= e < (rank + 1) * El
            out[r] = _ffn(Wf["gate"][e], Wf["up"][e], Wf["down"][e], recv_x[r].numpy()[None])[0]
        back = torch.zeros((T * K, H), dtype=torch.float64)
        dist.all_to_all_single(back, torch.from_numpy(out), plan["send_count"], plan["recv_count"])
        y = _ffn(Wf["shared_gate"], Wf["shared_up"], Wf["shared_down"], x.astype(np.float64))
        for t in range(T):
            for s in range(K):
                y[t] += float(w[t, s]) * back[slot_row[t * K + s]].numpy()
        if T > 0:
            np.testing.assert_allclose(y, ref_y, rtol=1e-4, atol=1e-5)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("token_counts", [(13, 7), (0, 9), (16, 16)])
def test_ep_protocol_two_gloo_ranks(token_counts):
    mp.spawn(_worker, args=(2, _free_port(), token_counts), nprocs=2, join=True)


def test_ep_plan_rejects_bad_input():
    from litemind_b200._lib import LiteMindError
    from litemind_b200.moe import ep_plan

    with pytest.raises(LiteMindError):
        ep_plan(3, np.zeros(8, np.int32), np.zeros(8, np.int32))  # 3 ranks do not divide 8 experts
    with pytest.raises(LiteMindError):
        ep_plan(2, np.array([1, -1, 0, 0], np.int32), np.zeros(4, np.int32))
