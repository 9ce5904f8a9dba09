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


def test_launch_counts_follow_dispatch_rules():
    k = bench.kernels_per_forward
    assert k(32, 1) == k(128, 1) == 1  # the fused decode kernel (direct and gather modes)
    assert k(129, 1) == k(256, 1) == 4  # single-launch route, row gather, two GEMMs
    assert k(257, 1) == 7  # logits, top-k, scan, placement, gather, two GEMMs
    assert k(16384, 1) == 6  # the placement copies the rows itself
    assert k(32, 8) == 7  # fixed-block exchange: route, pack, sort, schedule, two GEMMs, combine
    # Host-planned, 2 chunks (the default): four routing kernels, per chunk a sort and two
    # GEMMs, the shared experts' two GEMMs, the combine.
    os.environ.pop("LITEMIND_B200_EP_CHUNKS", None)
    assert k(8192, 8) == 4 + 2 * 3 + 2 + 1
    os.environ["LITEMIND_B200_EP_CHUNKS"] = "1"
    try:
        assert k(8192, 8) == 4 + 3 + 1
    finally:
        os.environ.pop("LITEMIND_B200_EP_CHUNKS", None)
