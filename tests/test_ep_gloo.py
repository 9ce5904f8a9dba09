"""Expert-parallel host logic on CPU: two gloo ranks run the exchange protocol of
lm_moe_forward's expert-parallel path around lm_moe_ep_plan (the library's own
plan function) and must reproduce the single-process oracle.

Each rank routes its own tokens with the oracle, orders its (token, slot) rows by
expert (token order within an expert, as the place kernel does), exchanges the
per-expert counts, asks lm_moe_ep_plan for the send/recv counts and offsets, sends
the rows with all_to_all_single, computes its local experts, returns the outputs in
receive order, and combines them by slot with the routing weights, plus the shared
experts.  With chunks > 1 the rows move in chunks of local experts planned by
lm_moe_ep_chunk_plan, as lm_moe_forward's pipelined exchange moves them.  The
small-batch fixed-block exchange (one block of rows per rank pair, planned on the
device) runs the same way through a restatement of its kernels' index math.  No GPU
is used.
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


def _worker(rank, world, port, token_counts, chunks):
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
        # The local experts move in `chunks` exchanges (one when chunks = 1); the
        # receive buffer holds the chunks one after another, each by source rank.
        plans = [ep_plan(world, counts, recv_counts.numpy(), chunks, k) for k in range(chunks)]
        assert sum(p["n_send"] for p in plans) == plan["n_send"]
        assert sum(p["n_recv"] for p in plans) == plan["n_recv"]
        rc = recv_counts.numpy().reshape(world, El)
        recv_x = np.zeros((plan["n_recv"], H))
        recv_e = np.zeros(plan["n_recv"], np.int64)
        for k, pk in enumerate(plans):
            base = pk["recv_offset"][0]
            assert base == sum(p["n_recv"] for p in plans[:k])
            assert pk["recv_offset"] == [base + sum(pk["recv_count"][:d]) for d in range(world)]
            take = np.concatenate([np.arange(pk["send_offset"][d], pk["send_offset"][d] + pk["send_count"][d])
                                   for d in range(world)]).astype(np.int64)
            got_x = torch.zeros((pk["n_recv"], H), dtype=torch.float64)
            dist.all_to_all_single(got_x, torch.from_numpy(send_rows[take].reshape(-1, H)), pk["recv_count"],
                                   pk["send_count"])
            got_e = torch.zeros(pk["n_recv"], dtype=torch.int64)
            dist.all_to_all_single(got_e, torch.from_numpy(send_expert[take]), pk["recv_count"], pk["send_count"])
            recv_x[base:base + pk["n_recv"]] = got_x.numpy()
            recv_e[base:base + pk["n_recv"]] = got_e.numpy()
            # Chunk k carries this rank's local experts [lo, hi), each source's rows by expert.
            lo, hi = k * El // chunks, (k + 1) * El // chunks
            for src in range(world):
                seg = recv_e[pk["recv_offset"][src]:pk["recv_offset"][src] + pk["recv_count"][src]]
                assert np.array_equal(seg, np.repeat(rank * El + np.arange(lo, hi), rc[src, lo:hi]))
        out = np.zeros((plan["n_recv"], H))
        for r in range(plan["n_recv"]):
            e = int(recv_e[r])
            assert rank * El <= e < (rank + 1) * El
            out[r] = _ffn(Wf["gate"][e], Wf["up"][e], Wf["down"][e], recv_x[r][None])[0]
        # Outputs go back chunk by chunk with the offsets reversed.
        back = np.zeros((T * K, H))
        for pk in plans:
            base = pk["recv_offset"][0]
            got = torch.zeros((pk["n_send"], H), dtype=torch.float64)
            dist.all_to_all_single(got, torch.from_numpy(out[base:base + pk["n_recv"]].reshape(-1, H)),
                                   pk["send_count"], pk["recv_count"])
            pos = 0
            for d in range(world):
                n = pk["send_count"][d]
                back[pk["send_offset"][d]:pk["send_offset"][d] + n] = got.numpy()[pos:pos + n]
                pos += n
        y = _ffn(Wf["shared_gate"], Wf["shared_up"], Wf["shared_down"], x.astype(np.float64))
        for t in range(T):
            for s in range(K):
                y[t] += float(w[t, s]) * back[slot_row[t * K + s]]
        if T > 0:
            np.testing.assert_allclose(y, ref_y, rtol=1e-4, atol=1e-5)
    finally:
        dist.destroy_process_group()


def _worker_fixed(rank, world, port, token_counts, max_tokens):
    """The fixed-block exchange (small batches, no host round trip): every rank sends
    every peer one block of `cap` = max_tokens x min(k, local experts) rows with the
    per-expert counts beside it.  The index math restates the device kernels: the
    pack into destination blocks (ep_pack_kernel), the receiver's expert-major sort
    with its row map (ep_sort_rows_kernel with a fixed source stride), the receiver's
    schedule (ep_schedule_kernel), outputs stored back at their receive positions
    (the down epilogue's y_rows_map), the blocks returned and the slot-ordered
    weighted combine (ep_combine_kernel)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.oracle import Oracle, RouterConfig

        orc = Oracle()
        W = syn.layer_weights(SHAPE, seed=5, std=0.1)
        Wf = {k: (syn.bf16_to_f32(v).reshape(v.shape).astype(np.float64) if v.dtype == np.uint16 else v)
              for k, v in W.items()}
        E, K, H = SHAPE.n_routed_experts, SHAPE.top_k, SHAPE.hidden
        El = E // world
        cap = max_tokens * min(K, El)
        T = token_counts[rank]
        x = syn.bf16_to_f32(syn.tokens(SHAPE, max(T, 1), seed=20 + rank)).reshape(-1, H)[:T]
        if T > 0:
            ref_y, idx, w, _ = orc.moe_layer(x, W, RouterConfig(E, K), SHAPE.n_shared_experts)
        else:
            ref_y, idx, w = np.zeros((0, H), np.float32), np.zeros((0, K), np.int64), np.zeros((0, K), np.float32)
        # Expert-sorted rows (token order within an expert) and each slot's row.
        pairs = [(int(idx[t, s]), t) for t in range(T) for s in range(K)]
        order = sorted(range(len(pairs)), key=lambda i: (pairs[i][0], i))
        row_token = np.array([pairs[i][1] for i in order], np.int64)
        slot_row = np.zeros(T * K, np.int64)
        for row, i in enumerate(order):
            slot_row[i] = row
        counts = np.bincount(idx.reshape(-1), minlength=E).astype(np.int64)
        off = np.concatenate([[0], np.cumsum(counts)])
        # ep_pack: row r of expert e goes to destination d = e // El, at d * cap + its
        # rank among the rows bound for d.
        def padded(r):
            e = int(np.searchsorted(off, r, side="right") - 1)
            d = e // El
            assert r - off[d * El] < cap, "a destination's rows exceed the fixed block"
            return d * cap + (r - off[d * El])
        x_send = np.zeros((world * cap, H))
        for r in range(T * K):
            x_send[padded(r)] = x[row_token[r]]
        slot_row = np.array([padded(int(r)) for r in slot_row], np.int64)
        # One exchange of counts and blocks.
        recv_counts = torch.zeros(E, dtype=torch.int64)
        dist.all_to_all_single(recv_counts, torch.from_numpy(counts))
        rc = recv_counts.numpy().reshape(world, El)
        x_recv = torch.zeros((world * cap, H), dtype=torch.float64)
        dist.all_to_all_single(x_recv, torch.from_numpy(x_send))
        x_recv = x_recv.numpy()
        # ep_sort_rows with source stride cap: block (source r, local expert e).
        n_recv = int(rc.sum())
        x_sorted = np.zeros((n_recv, H))
        row_src = np.full(n_recv, -1, np.int64)
        for r in range(world):
            for e in range(El):
                src = r * cap + int(rc[r, :e].sum())
                dst = int(rc[:, :e].sum()) + int(rc[:r, e].sum())
                n = int(rc[r, e])
                x_sorted[dst:dst + n] = x_recv[src:src + n]
                row_src[dst:dst + n] = np.arange(src, src + n)
        assert (row_src >= 0).all() and len(set(row_src.tolist())) == n_recv
        # ep_schedule: one segment per local expert, expert-major, then the shared experts.
        seg_off = np.concatenate([[0], np.cumsum(rc.sum(axis=0))])[:-1]
        seg_cnt = rc.sum(axis=0)
        assert seg_off[-1] + seg_cnt[-1] == n_recv if El else True
        # Local experts; outputs stored at their receive positions.
        y_ret = np.zeros((world * cap, H))
        for e in range(El):
            rows = slice(int(seg_off[e]), int(seg_off[e] + seg_cnt[e]))
            ge = rank * El + e
            y_ret[row_src[rows]] = _ffn(Wf["gate"][ge], Wf["up"][ge], Wf["down"][ge], x_sorted[rows])
        y_back = torch.zeros((world * cap, H), dtype=torch.float64)
        dist.all_to_all_single(y_back, torch.from_numpy(y_ret))
        y_back = y_back.numpy()
        # ep_combine: shared experts first, then the slots in selection order.
        y = _ffn(Wf["shared_gate"], Wf["shared_up"], Wf["shared_down"], x.astype(np.float64))
        for t in range(T):
            for s in range(K):
                y[t] += float(w[t, s]) * y_back[slot_row[t * K + s]]
        if T > 0:
            np.testing.assert_allclose(y, ref_y, rtol=1e-4, atol=1e-5)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,token_counts,max_tokens", [(2, (13, 7), 16), (2, (0, 5), 8), (4, (3, 0, 8, 8), 8)])
def test_ep_fixed_block_protocol_gloo_ranks(world, token_counts, max_tokens):
    mp.spawn(_worker_fixed, args=(world, _free_port(), token_counts, max_tokens), nprocs=world, join=True)


# chunks > 1: the chunked exchange of lm_moe_ep_chunk_plan (4 local experts per rank
# here; 3 chunks split them 1 + 1 + 2).
@pytest.mark.parametrize("token_counts,chunks", [((13, 7), 1), ((0, 9), 1), ((16, 16), 1), ((13, 7), 2),
                                                 ((16, 16), 3), ((0, 9), 4)])
def test_ep_protocol_two_gloo_ranks(token_counts, chunks):
    mp.spawn(_worker, args=(2, _free_port(), token_counts, chunks), nprocs=2, join=True)


# Four ranks of 2 local experts each, in one piece and in 2 chunks of one expert.
@pytest.mark.parametrize("chunks", [1, 2])
def test_ep_protocol_four_gloo_ranks(chunks):
    mp.spawn(_worker, args=(4, _free_port(), (11, 0, 6, 19), chunks), nprocs=4, join=True)


def test_ep_chunk_plan_layout():
    """Chunk plans partition the whole plan: per destination, the chunks' send ranges
    tile the whole send range in order; the receive buffer holds the chunks back to back."""
    from litemind_b200.moe import ep_plan

    rng = np.random.default_rng(0)
    world, E = 4, 16
    El = E // world
    send = rng.integers(0, 9, E).astype(np.int32)
    recv = rng.integers(0, 9, E).astype(np.int32)
    whole = ep_plan(world, send, recv)
    for chunks in (1, 2, 3, 4):
        plans = [ep_plan(world, send, recv, chunks, k) for k in range(chunks)]
        for d in range(world):
            pos = whole["send_offset"][d]
            for k, pk in enumerate(plans):
                assert pk["send_offset"][d] == pos
                lo, hi = k * El // chunks, (k + 1) * El // chunks
                assert pk["send_count"][d] == send[d * El + lo:d * El + hi].sum()
                assert pk["recv_count"][d] == recv[d * El + lo:d * El + hi].sum()
                pos += pk["send_count"][d]
            assert pos == whole["send_offset"][d] + whole["send_count"][d]
        base = 0
        for pk in plans:
            assert pk["recv_offset"][0] == base
            base += pk["n_recv"]
        assert base == whole["n_recv"]
    assert ep_plan(world, send, recv, 1, 0) == whole


def test_ep_plan_rejects_bad_input():
    from litemind_b200._lib import LiteMindError
    from litemind_b200.moe import ep_plan

    with pytest.raises(LiteMindError):
        ep_plan(3, np.zeros(8, np.int32), np.zeros(8, np.int32))  # 3 ranks do not divide 8 experts
    with pytest.raises(LiteMindError):
        ep_plan(2, np.array([1, -1, 0, 0], np.int32), np.zeros(4, np.int32))
    for chunks, chunk in ((0, 0), (3, 0), (2, 2), (2, -1)):  # 2 local experts: 1 or 2 chunks
        with pytest.raises(LiteMindError):
            ep_plan(2, np.zeros(4, np.int32), np.zeros(4, np.int32), chunks, chunk)
