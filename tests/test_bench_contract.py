"""bench.py's JSON contract on CPU: the reference arm (the reference's own CPU code,
oracle/_ref) prints one line with the keys the round driver reads, and the launch
count it reports for our arm follows the library's dispatch rules."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _run(*args):
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    from oracle import oracle as orc

    if not orc.reference_available():
        pytest.skip("reference library not built here")
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "0", "--tokens", "8")
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["metric"] == bench.METRIC and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_loader_reference_arm_is_unavailable():
    d = _run("--impl", "reference", "--workload", "load")
    assert d["impl"] == "reference" and "unavailable" in d


def _window_worker(rank, world, port, result_dir):
    import time

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # Rank 0's window closed long ago; rank 1's is still open.  Both must stop
        # together, or rank 1 would enter a collective forward that rank 0 never joins.
        t0 = time.perf_counter() - (100.0 if rank == 0 else 0.0)
        answers = [bench.load_window_open(t0, 10.0, world, torch) for _ in range(3)]
        with open(os.path.join(result_dir, f"rank{rank}.json"), "w") as f:
            json.dump(answers, f)
    finally:
        dist.destroy_process_group()


def test_load_window_is_agreed_across_ranks(tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_window_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    answers = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    assert answers[0] == answers[1] == [False, False, False]


def test_launch_counts_follow_dispatch_rules():
    k = bench.kernels_per_forward
    assert k(32, 1) == k(128, 1) == k(256, 1) == 1  # the fused decode kernel (direct and gather modes)
    assert k(257, 1) == 7  # logits, top-k, scan, placement, gather, two GEMMs
    assert k(16384, 1) == 6  # the placement copies the rows itself
    assert k(32, 8) == 7  # fixed-block exchange: route, pack, sort, schedule, two GEMMs, combine
    # Host-planned, 2 chunks (the default): four routing kernels, per chunk a sort and two
    # GEMMs, the shared experts' two GEMMs, the combine.
    os.environ.pop("LITEMIND_B200_EP_CHUNKS", None)
    os.environ.pop("LITEMIND_B200_EP_COPY", None)
    assert k(8192, 8) == 4 + 2 * 3 + 2 + 1
    # Two ranks move the rows by copy engines by default: a signal for the rows and one
    # per chunk, and the peer's wait for its rows and one per chunk.
    assert k(8192, 2) == 4 + 2 * 3 + 2 + 1 + (1 + 2) + (1 + 2)
    os.environ["LITEMIND_B200_EP_CHUNKS"] = "1"
    try:
        assert k(8192, 8) == 4 + 3 + 1
        os.environ["LITEMIND_B200_EP_COPY"] = "0"
        assert k(8192, 2) == 4 + 3 + 1
        os.environ["LITEMIND_B200_EP_COPY"] = "1"
        assert k(8192, 4) == 4 + 3 + 1 + (1 + 1) + 3 * (1 + 1)
    finally:
        os.environ.pop("LITEMIND_B200_EP_CHUNKS", None)
        os.environ.pop("LITEMIND_B200_EP_COPY", None)
