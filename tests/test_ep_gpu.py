"""Expert parallelism on two B200s: each rank holds half of the routed experts,
runs lm_moe_forward on its own tokens over NCCL, and its outputs must match the
oracle's single-process MoE block for those tokens.  Needs 2 GPUs on one machine;
gloo carries only the NCCL unique id.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from litemind_b200 import synthetic as syn  # noqa: E402

SMALL = syn.MoeShape(hidden=256, inter=128, n_routed_experts=8, n_shared_experts=1, top_k=2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shape_name, token_counts, chunks, copy=True):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LITEMIND_B200_EP_CHUNKS=str(chunks),
                      LITEMIND_B200_EP_COPY="1" if copy else "0")
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor
        from oracle.oracle import Oracle, RouterConfig
        from tests.parity import assert_layer_parity

        torch.cuda.set_device(rank)
        shape = SMALL if shape_name == "small" else syn.V2_LITE
        W = syn.layer_weights(shape, seed=5, std=0.1 if shape_name == "small" else 0.02)
        uid = [MoeLayer.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        layer = MoeLayer(MoeConfig.from_shape(shape, max_tokens=max(token_counts)), device=rank)
        layer.ep_init(uid[0], rank, world)
        layer.upload_layer(0, W)
        T = token_counts[rank]
        xb = syn.tokens(shape, max(T, 1), seed=100 + rank)[:T]
        x = bf16_tensor(xb) if T > 0 else torch.zeros((0, shape.hidden), dtype=torch.bfloat16, device="cuda")
        for _ in range(3):  # calls in a row reuse every exchange buffer (and advance the flags' epoch)
            y = layer.forward(0, x)
            layer.sync()
        if T > 0:
            idx, w, _ = layer.route(0, x)
            layer.sync()
            ref = Oracle().moe_layer(syn.bf16_to_f32(xb).reshape(T, -1), W,
                                     RouterConfig(shape.n_routed_experts, shape.top_k), shape.n_shared_experts)
            stats = assert_layer_parity(y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), *ref,
                                        what=f"EP rank {rank} T={T}")
            print(f"rank {rank}: {stats}")
        dist.barrier()
        layer.close()
    finally:
        dist.destroy_process_group()


# Up to max_tokens x min(k, local experts) rows per rank pair, ranks exchange fixed
# blocks with the plan made on the device; (5000, 4100) and V2-Lite (700, 450) exceed
# that and take the host-planned exchange: in one piece (chunks 1) or pipelined in
# chunks of local experts (4 chunks of 1 expert, 3 uneven chunks, V2-Lite's 4 chunks of
# 8 experts).  The host-planned rows move by copy engines out of IPC-mapped peer
# buffers (the default) or by NCCL (copy=False).
@pytest.mark.parametrize("shape_name,token_counts,chunks", [("small", (37, 11), 4), ("small", (0, 20), 4),
                                                            ("small", (300, 300), 4), ("v2lite", (32, 64), 4),
                                                            ("small", (5000, 4100), 1), ("small", (5000, 4100), 4),
                                                            ("small", (3000, 0), 3), ("v2lite", (700, 450), 4)])
def test_expert_parallel_two_gpus(shape_name, token_counts, chunks):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_worker, args=(2, _free_port(), shape_name, token_counts, chunks), nprocs=2, join=True)


@pytest.mark.parametrize("shape_name,token_counts,chunks", [("small", (5000, 4100), 1), ("small", (3000, 0), 3),
                                                            ("v2lite", (700, 450), 4)])
def test_expert_parallel_two_gpus_nccl_exchange(shape_name, token_counts, chunks):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_worker, args=(2, _free_port(), shape_name, token_counts, chunks, False), nprocs=2, join=True)


def _silent_peer_worker(rank, world, port, tokens, copy, status_dir):
    """Both ranks forward once; then each in turn stops taking part while staying alive
    (no kernel or exchange of its own in flight), and the other's next forward must end
    with LM_ERR_COMM within the shortened wait limit instead of waiting for ever."""
    import json
    import time
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LITEMIND_B200_EP_CHUNKS="2",
                      LITEMIND_B200_EP_COPY="1" if copy else "0", NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from litemind_b200 import _lib
        from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor

        torch.cuda.set_device(rank)
        W = syn.layer_weights(SMALL, seed=5, std=0.1)
        uid = [MoeLayer.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        layer = MoeLayer(MoeConfig.from_shape(SMALL, max_tokens=tokens), device=rank)
        layer.ep_init(uid[0], rank, world)
        layer.upload_layer(0, W)
        x = bf16_tensor(syn.tokens(SMALL, tokens, seed=100 + rank))
        layer.forward(0, x)
        layer.sync()
        dist.barrier()
        record = {}
        for turn in range(world):  # rank `turn` forwards alone; its peer stays silent
            if rank == turn:
                layer.debug_set(_lib.LM_DEBUG_WAIT_LIMIT_NS, 300_000_000)
                t0 = time.monotonic()
                try:
                    layer.forward(0, x)
                    layer.sync()
                    record["first"] = "no error"
                except _lib.LiteMindError as e:
                    record["first"] = e.status
                record["seconds"] = time.monotonic() - t0
                try:  # the context's expert parallelism is over: the next call fails at once
                    layer.forward(0, x)
                    layer.sync()
                    record["second"] = "no error"
                except _lib.LiteMindError as e:
                    record["second"] = e.status
            dist.barrier()
        with open(os.path.join(status_dir, f"rank{rank}.json"), "w") as f:
            json.dump(record, f)
        layer.close()
    finally:
        dist.destroy_process_group()


# 300 tokens: fixed blocks, the exchange enqueued without a host wait (the sync reports
# it); 5000: the host-planned exchange, whose row counts the host waits for.
@pytest.mark.parametrize("tokens,copy", [(300, False), (5000, True), (5000, False)])
def test_silent_peer_ends_the_forward_with_an_error(tmp_path, tokens, copy):
    import json

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_silent_peer_worker, args=(2, _free_port(), tokens, copy, str(tmp_path)), nprocs=2, join=True)
    from litemind_b200._lib import LM_ERR_COMM, LM_ERR_DEVICE_TIMEOUT

    for r in range(2):
        rec = json.load(open(tmp_path / f"rank{r}.json"))
        # The host's wait for the exchange gives up (LM_ERR_COMM), or -- when the exchange
        # ends early because the peer's communicator is gone -- a device-side wait for the
        # peer's readiness flag does (LM_ERR_DEVICE_TIMEOUT); either way within the limit.
        assert rec["first"] in (LM_ERR_COMM, LM_ERR_DEVICE_TIMEOUT), (r, rec)
        assert rec["second"] in (LM_ERR_COMM, LM_ERR_DEVICE_TIMEOUT), (r, rec)
        assert rec["seconds"] < 20.0, (r, rec)
