"""The oracle against the live reference build (oracle/_ref), bit for bit.

Random inputs beyond the committed golden vectors: every shape and routing
configuration here must give identical bits from the C restatement and from the
reference's own compiled sources.  Skipped where the reference build is absent.
"""
import numpy as np
import pytest

from litemind_b200 import synthetic as syn
from oracle.oracle import RouterConfig


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 3), (67, 253), (33, 40), (5, 2047), (16, 2048), (9, 1408)])
def test_kernels_bit_exact(oracle_lib, reference_lib, rows, cols):
    rng = np.random.default_rng(rows * 10007 + cols)
    w = syn.bf16_round(rng.uniform(-1, 1, rows * cols).astype(np.float32)).reshape(rows, cols)
    wf = rng.standard_normal((rows, cols)).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    acc = rng.standard_normal(rows).astype(np.float32)
    np.testing.assert_array_equal(oracle_lib.matvec_bf16(w, x), reference_lib.matvec_bf16(w, x))
    np.testing.assert_array_equal(oracle_lib.matvec_bf16_accumulate(w, x, acc, 0.3),
                                  reference_lib.matvec_bf16_accumulate(w, x, acc, 0.3))
    np.testing.assert_array_equal(oracle_lib.matvec_f32(wf, x), reference_lib.matvec_f32(wf, x))
    v = (rng.standard_normal(cols) * 3).astype(np.float32)
    np.testing.assert_array_equal(oracle_lib.softmax(v), reference_lib.softmax(v))
    np.testing.assert_array_equal(oracle_lib.silu_multiply(v, x), reference_lib.silu_multiply(v, x))
    np.testing.assert_array_equal(oracle_lib.rms_norm(v, x, 1e-6), reference_lib.rms_norm(v, x, 1e-6))
    np.testing.assert_array_equal(oracle_lib.axpy(0.7, v, x), reference_lib.axpy(0.7, v, x))


def test_router_bit_exact(oracle_lib, reference_lib):
    rng = np.random.default_rng(3)
    for case in range(3000):
        E = int(rng.choice([1, 2, 5, 8, 16, 64, 6, 12, 160]))
        K = int(rng.integers(0, E + 2))  # includes 0 and > E: empty / clipped selections
        cfg = RouterConfig(E, K, int(rng.choice([1, 2, 3, 4, 8])), int(rng.integers(0, 4)),
                           bool(rng.integers(0, 2)), bool(rng.integers(0, 2)), float(rng.choice([1.0, 2.0, 0.5])))
        n = E if case % 5 else int(rng.integers(0, E + 3))  # wrong logit counts give empty selections
        logits = (rng.standard_normal(n) * 2).astype(np.float32)
        if case % 3 == 0:
            logits = np.round(logits)
        a, b = oracle_lib.router_select(logits, cfg), reference_lib.router_select(logits, cfg)
        np.testing.assert_array_equal(a[0], b[0], err_msg=f"case {case}")
        np.testing.assert_array_equal(a[1], b[1], err_msg=f"case {case}")


def test_select_top_k_errors_match(oracle_lib, reference_lib):
    lg = np.array([0, 5, 1, 4, 2, 3, -1, -2], np.float32)
    for args in [(8, 3, True), (8, 0, False), (8, 9, False), (4, 2, True), (0, 1, False)]:
        outs = []
        for lib in (oracle_lib, reference_lib):
            try:
                outs.append(lib.select_top_k(lg, *args))
            except ValueError:
                outs.append("throws")
        if isinstance(outs[0], str) or isinstance(outs[1], str):
            assert outs[0] == outs[1]
        else:
            np.testing.assert_array_equal(outs[0][0], outs[1][0])
            np.testing.assert_array_equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("T,bias", [(1, False), (13, True), (40, False)])
def test_moe_layer_bit_exact(oracle_lib, reference_lib, T, bias):
    shape = syn.MoeShape(hidden=256, inter=128, n_routed_experts=16, n_shared_experts=2, top_k=4)
    W = syn.layer_weights(shape, seed=T, std=0.05)
    x = syn.bf16_to_f32(syn.tokens(shape, T, seed=T)).reshape(T, -1)
    b = syn.zipf_bias(shape, seed=T) if bias else None
    for cfg in (RouterConfig(16, 4), RouterConfig(16, 4, 4, 2, True, True, 1.0), RouterConfig(16, 4, 1, 1, False,
                                                                                                False, 2.5)):
        o = oracle_lib.moe_layer(x, W, cfg, 2, bias=b, threads=4)
        r = reference_lib.moe_layer(x, W, cfg, 2, bias=b, threads=4)
        for a, c in zip(o, r):
            np.testing.assert_array_equal(a, c)


def test_bf16_rounding_matches_oracle(oracle_lib):
    import ctypes as C

    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                           np.array([0.0, -0.0, 1e-40, -1e-40, 3.4e38, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9],
                                    np.float32)])
    ours = syn.bf16_round(vals)
    f = oracle_lib.lib.orc_f32_to_bf16
    theirs = np.array([f(C.c_float(float(v))) for v in vals], np.uint16)
    np.testing.assert_array_equal(ours, theirs)
