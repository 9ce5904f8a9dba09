"""The oracle against the reference: golden vectors made by the reference's own
code (tests/golden/make_golden.py) and the reference's own known-answer tests
(tests/KernelTest.cpp, tests/MoeRouterSamplerTest.cpp), restated.  CPU only."""
import json
import math
import os

import numpy as np
import pytest

from litemind_b200 import synthetic as syn
from oracle.oracle import RouterConfig

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


# ── tests/KernelTest.cpp, restated against the oracle ──────────────────────

def test_kerneltest_matvec(oracle_lib):
    g = load("kernels.npz")
    out = oracle_lib.matvec_bf16(g["kt_w_bf16"], g["kt_x"])
    np.testing.assert_array_equal(out, g["kt_matvec"])               # bit-exact with the reference
    np.testing.assert_allclose(out, g["kt_expected"], atol=1e-3, rtol=0)  # KernelTest.cpp:60-63
    np.testing.assert_allclose(g["kt_serial"], out, atol=1e-4, rtol=0)    # :66-70
    acc = oracle_lib.matvec_bf16_accumulate(g["kt_w_bf16"], g["kt_x"], np.ones(67, np.float32), 0.5)
    np.testing.assert_array_equal(acc, g["kt_accumulate"])
    np.testing.assert_allclose(acc, 1.0 + 0.5 * g["kt_expected"], atol=1e-3, rtol=0)  # :73-79


def test_kerneltest_rms_softmax_silu(oracle_lib):
    g = load("kernels.npz")
    v = oracle_lib.rms_norm(np.array([1, 2, 3, 4], np.float32), np.full(4, 2.0, np.float32), 1e-6)
    scale = 2.0 / math.sqrt(7.5 + 1e-6)
    np.testing.assert_allclose(v, np.arange(1, 5) * scale, atol=1e-5, rtol=0)  # :82-90
    np.testing.assert_array_equal(v, g["rms_known_out"])
    np.testing.assert_array_equal(oracle_lib.rms_norm(g["rms_in"], g["rms_w"], 1e-6), g["rms_out"])
    s = oracle_lib.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert abs(s.sum() - 1.0) <= 1e-6 and s[2] > s[1] > s[0]  # :93-97
    e = oracle_lib.softmax(np.array([1000.0, 1001.0], np.float32))
    assert np.isfinite(e).all() and abs(e.sum() - 1.0) <= 1e-6  # :99-102
    for i in range(3):
        np.testing.assert_array_equal(oracle_lib.softmax(g[f"softmax_in_{i}"]), g[f"softmax_out_{i}"])
    p = oracle_lib.silu_multiply(np.array([0.0, 1.0], np.float32), np.array([3.0, 2.0], np.float32))
    assert abs(p[0]) <= 1e-6 and abs(p[1] - 2.0 / (1.0 + math.exp(-1.0))) <= 1e-6  # :105-110
    np.testing.assert_array_equal(oracle_lib.silu_multiply(g["silu_gate"], g["silu_up"]), g["silu_out"])
    np.testing.assert_array_equal(oracle_lib.axpy(0.37, g["axpy_src"], g["axpy_dst"]), g["axpy_out"])
    np.testing.assert_array_equal(oracle_lib.matvec_f32(g["router_w"], g["router_x"]), g["router_logits"])


# ── tests/MoeRouterSamplerTest.cpp, restated against the oracle ────────────

LOGITS = np.array([0.0, 5.0, 1.0, 4.0, 2.0, 3.0, -1.0, -2.0], np.float32)


def lite(**kw):
    base = dict(n_routed_experts=8, num_experts_per_tok=3)
    base.update(kw)
    return RouterConfig(**base)


def test_moerouter_known_answers(oracle_lib):
    idx, w = oracle_lib.router_select(LOGITS, lite())
    assert list(idx) == [1, 3, 5] and w[0] > w[1]                     # :34-38
    assert 0.5 < w.sum() < 1.0                                          # :43-45
    assert abs(w[0] - 1.0 / sum(math.exp(v - 5.0) for v in LOGITS)) <= 1e-6  # :48-53
    _, wn = oracle_lib.router_select(LOGITS, lite(norm_topk_prob=True))
    assert abs(wn.sum() - 1.0) <= 1e-5                                  # :56-61
    _, ws = oracle_lib.router_select(LOGITS, lite(routed_scaling_factor=2.0))
    assert abs(ws[0] - 2.0 * w[0]) <= 1e-6                              # :64-68
    _, wb = oracle_lib.router_select(LOGITS, lite(norm_topk_prob=True, routed_scaling_factor=2.0))
    assert abs(wb.sum() - 1.0) <= 1e-5                                  # :70-76
    gi, _ = oracle_lib.router_select(LOGITS, lite(num_experts_per_tok=2, n_group=2, topk_group=1,
                                                  group_limited=True))
    assert len(gi) == 2 and (gi < 4).all()                              # :79-88
    _, wl = oracle_lib.select_top_k(LOGITS, 8, 3, True)
    assert abs(wl.sum() - 1.0) <= 1e-5                                  # :91-93
    with pytest.raises(ValueError):
        oracle_lib.select_top_k(LOGITS, 8, 0, False)
    assert oracle_lib.router_select(LOGITS[:7], lite())[0].size == 0    # src/MoeRouter.cpp:57-59


def test_router_golden(oracle_lib):
    g = load("router.npz")
    for c in range(g["params"].shape[0]):
        E, K, ng, tg, gl, norm = (int(v) for v in g["params"][c])
        cfg = RouterConfig(E, K, ng, tg, bool(gl), bool(norm), float(g["scale"][c]))
        idx, w = oracle_lib.router_select(g["logits"][c, :E], cfg)
        n = int(g["count"][c])
        np.testing.assert_array_equal(idx, g["idx"][c, :n], err_msg=f"case {c}")
        np.testing.assert_array_equal(w, g["w"][c, :n], err_msg=f"case {c}")


@pytest.mark.parametrize("name", ["testmodel", "grouped", "biased"])
def test_moe_small_golden(oracle_lib, name):
    g = load("moe_small.npz")
    H, I, E, S, K = (int(v) for v in g[f"{name}_shape"])
    ng, tg, gl, norm = (int(v) for v in g[f"{name}_routing"])
    cfg = RouterConfig(E, K, ng, tg, bool(gl), bool(norm), float(g[f"{name}_scale"]))
    W = {k: g[f"{name}_{k}"] for k in ("router", "gate", "up", "down", "shared_gate", "shared_up", "shared_down")}
    bias = g[f"{name}_bias"] if f"{name}_bias" in g.files else None
    y, idx, w, logits = oracle_lib.moe_layer(g[f"{name}_x"], W, cfg, S, bias=bias, threads=2)
    np.testing.assert_array_equal(logits, g[f"{name}_logits"])
    np.testing.assert_array_equal(idx, g[f"{name}_idx"])
    np.testing.assert_array_equal(w, g[f"{name}_w"])
    np.testing.assert_array_equal(y, g[f"{name}_y"])


def test_moe_v2lite_golden(oracle_lib, v2lite_weights):
    g = load("moe_v2lite.npz")
    W = v2lite_weights
    fp = np.array([int(W[k].astype(np.uint64).sum()) for k in ("gate", "up", "down", "shared_gate", "shared_up",
                                                                 "shared_down")], np.uint64)
    np.testing.assert_array_equal(fp, g["weight_fingerprint"])  # the synthetic generator has not drifted
    np.testing.assert_array_equal(syn.tokens(syn.V2_LITE, 3, seed=1), g["x_bits"])
    x = syn.bf16_to_f32(g["x_bits"]).reshape(3, -1)
    y, idx, w, logits = oracle_lib.moe_layer(x, W, RouterConfig(), 2, threads=0)
    np.testing.assert_array_equal(logits, g["logits"])
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_array_equal(w, g["w"])
    np.testing.assert_array_equal(y, g["y"])


def test_expert_cache_golden(oracle_lib):
    """The oracle's ExpertCache bookkeeping against the reference's counters."""
    import ctypes as C

    with open(os.path.join(GOLDEN, "cache.json")) as f:
        g = json.load(f)
    from oracle.oracle import HERE  # noqa: F401

    class Cache(C.Structure):
        _fields_ = [("budget_bytes", C.c_uint64), ("resident_bytes", C.c_uint64), ("loads", C.c_uint64),
                    ("hits", C.c_uint64), ("evictions", C.c_uint64), ("bytes_streamed", C.c_uint64),
                    ("count", C.c_int64), ("keys", C.c_uint64 * 4096), ("bytes", C.c_uint64 * 4096)]

    lib = oracle_lib.lib
    lib.orc_cache_make_key.restype = C.c_uint64
    lib.orc_cache_make_key.argtypes = [C.c_uint64, C.c_uint64]
    c = Cache()
    lib.orc_cache_configure(C.byref(c), C.c_uint64(g["budget_blocks"] * g["block_bytes"]))
    for (layer, expert), want in zip(g["touches"], g["stats"]):
        lib.orc_cache_touch(C.byref(c), C.c_uint64(lib.orc_cache_make_key(layer, expert)),
                            C.c_uint64(g["block_bytes"]))
        assert [c.resident_bytes, c.count, c.loads, c.hits, c.evictions, c.bytes_streamed] == want
    lib.orc_cache_clear(C.byref(c))
    assert [c.resident_bytes, c.count, c.loads, c.hits, c.evictions, c.bytes_streamed] == g["after_clear"]


def test_sampled_parity_checker_accepts_the_oracle_and_rejects_a_perturbation():
    """The bench's parity leg (tests/parity.py) on CPU: the oracle's own output passes,
    an output with one expert's contribution dropped does not."""
    import numpy as np

    from litemind_b200 import synthetic as syn
    from oracle.oracle import Oracle, RouterConfig
    from tests.parity import sampled_oracle_parity

    shape = syn.MoeShape(hidden=256, inter=128, n_routed_experts=16, n_shared_experts=2, top_k=6)
    W = syn.layer_weights(shape, seed=3, std=0.05)
    xb = syn.tokens(shape, 12, seed=5)
    y, idx, w, _ = Oracle().moe_layer(syn.bf16_to_f32(xb).reshape(12, -1), W, RouterConfig(16, 6), 2)
    ok = sampled_oracle_parity(y, xb, W, [0, 3, 11])
    assert ok["pass"] and ok["max_rel"] == 0.0 and ok["tokens"] == 3
    bad = y.copy()
    bad[3] *= 1.05
    assert not sampled_oracle_parity(bad, xb, W, [0, 3, 11])["pass"]
