"""The C++20 host mirror (include/litemind_b200/*.hpp) compiled as a user would:
g++ against include/ and liblitemind_b200.so.  ExpertCacheTest replays the
reference's ExpertCache statistics (CPU); SafeTensorsTest looks up checkpoint tensors
through the C ABI (CPU); MoeRouterTest runs the reference's routing checks on the GPU.
CopyPoolTest checks the weight upload's host copy threads (CPU, built from source
under ThreadSanitizer); EpPlanTest the expert-parallel plans through MoeLayer.hpp (CPU)."""
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPP = os.path.join(ROOT, "tests", "cpp")
LIBDIR = os.path.join(ROOT, "litemind_b200")


def _compile(name, tmp_path):
    from litemind_b200 import build

    build.build()
    exe = tmp_path / name
    cuda_inc = os.path.join(build._cuda_home(), "include")
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", f"-I{ROOT}/include", f"-I{CPP}", f"-I{cuda_inc}",
           os.path.join(CPP, name + ".cpp"), f"-L{LIBDIR}", "-llitemind_b200", f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return str(exe)


def test_expert_cache_mirror_matches_reference_counters(tmp_path):
    with open(os.path.join(ROOT, "tests", "golden", "cache.json")) as f:
        g = json.load(f)
    seq = tmp_path / "sequence.txt"
    with open(seq, "w") as f:
        f.write(f"{g['budget_blocks'] * g['block_bytes']} {g['block_bytes']}\n")
        for (layer, expert), st in zip(g["touches"], g["stats"]):
            f.write(" ".join(str(v) for v in [layer, expert, *st]) + "\n")
        f.write(" ".join(str(v) for v in [999999, 0, *g["after_clear"]]) + "\n")
    exe = _compile("ExpertCacheTest", tmp_path)
    res = subprocess.run([exe, str(seq)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr


@pytest.mark.gpu
def test_moe_router_mirror_reference_checks(tmp_path):
    exe = _compile("MoeRouterTest", tmp_path)
    res = subprocess.run([exe], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr


def test_safetensors_lookup_from_cpp(tmp_path):
    import numpy as np

    from litemind_b200.checkpoint import write_safetensors

    shard = tmp_path / "shard.safetensors"
    write_safetensors(shard, {"w": ("BF16", np.arange(48, dtype=np.uint16).reshape(6, 8)),
                              "b": ("F32", np.ones(4, np.float32))})
    raw = shard.read_bytes()
    cut = tmp_path / "cut.safetensors"
    cut.write_bytes(raw[:-20])
    exe = _compile("SafeTensorsTest", tmp_path)
    res = subprocess.run([exe, str(shard), str(cut)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr



def test_copy_pool_threads(tmp_path):
    exe = tmp_path / "CopyPoolTest"
    host = os.path.join(ROOT, "litemind_b200", "csrc", "host")
    cmd = ["g++", "-std=c++20", "-O1", "-g", "-Wall", "-Wextra", "-pthread", "-fsanitize=thread", f"-I{host}", f"-I{CPP}",
           os.path.join(CPP, "CopyPoolTest.cpp"), os.path.join(host, "CopyPool.cpp"), "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "CopyPoolTest: all" in res.stdout


def test_ep_plan_from_cpp(tmp_path):
    exe = _compile("EpPlanTest", tmp_path)
    res = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stdout + res.stderr
