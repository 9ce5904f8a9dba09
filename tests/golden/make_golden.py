"""Generates the golden vectors in this directory from the reference's own code.

    python tests/golden/make_golden.py

Runs in a container that has the reference checkout: oracle/Makefile compiles the
reference's sources into oracle/_ref/libref_litemind.so, and every expected output
below comes from that library (the reference's gemm::, MoeRouter and ExpertCache,
driven through oracle/ref_harness.cpp).  The fixtures are small and committed, so
the CPU tests can pin the oracle on machines without the reference.

Files:
  kernels.npz   tests/KernelTest.cpp's seeded 67x253 matvec inputs and the reference's
                matvec / accumulate / serial outputs, plus softmax, silu, rms_norm and
                axpy cases
  router.npz    400 routing cases (random, tied and all-equal logits; greedy and
                group-limited; normalised and scaled) with the reference's selections
  moe_small.npz MoE blocks at small shapes (the reference's tools/make_test_model.py
                architecture: hidden 32, 4 experts of 16, top-2, 1 shared; and a
                group-limited normalised 16-expert shape) with inputs and weights
  moe_v2lite.npz  DeepSeek-V2-Lite layer outputs for 3 tokens; the weights and tokens
                are regenerated from litemind_b200.synthetic (seed 0 / tokens seed 1)
  cache.json    an ExpertCache touch sequence with the reference's counters
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from litemind_b200 import synthetic as syn  # noqa: E402
from oracle import oracle as orc  # noqa: E402

ROUTER_CASES = 400


def kernels(ref: orc.Reference) -> None:
    w32, w16, x = ref.kerneltest_inputs()
    rng = np.random.default_rng(7)
    acc0 = np.ones(67, np.float32)
    sm = [np.array([1.0, 2.0, 3.0], np.float32), np.array([1000.0, 1001.0], np.float32),
          (rng.standard_normal(64) * 3).astype(np.float32)]
    gate = (rng.standard_normal(97) * 4).astype(np.float32)
    up = rng.standard_normal(97).astype(np.float32)
    rms_v = rng.standard_normal(2048).astype(np.float32)
    rms_w = rng.standard_normal(2048).astype(np.float32)
    wf = rng.standard_normal((8, 2048)).astype(np.float32) * np.float32(0.02)
    xf = rng.standard_normal(2048).astype(np.float32)
    np.savez_compressed(
        os.path.join(HERE, "kernels.npz"),
        kt_w_f32=w32, kt_w_bf16=w16, kt_x=x,
        kt_matvec=ref.matvec_bf16(w16, x), kt_serial=ref.matvec_bf16_serial(w16, x),
        kt_accumulate=ref.matvec_bf16_accumulate(w16, x, acc0, 0.5),
        kt_expected=(w32.astype(np.float64) @ x.astype(np.float64)),
        softmax_in_0=sm[0], softmax_out_0=ref.softmax(sm[0]), softmax_in_1=sm[1], softmax_out_1=ref.softmax(sm[1]),
        softmax_in_2=sm[2], softmax_out_2=ref.softmax(sm[2]),
        silu_gate=gate, silu_up=up, silu_out=ref.silu_multiply(gate, up),
        rms_in=rms_v, rms_w=rms_w, rms_out=ref.rms_norm(rms_v, rms_w, 1e-6),
        rms_known_in=np.array([1, 2, 3, 4], np.float32), rms_known_out=ref.rms_norm(
            np.array([1, 2, 3, 4], np.float32), np.full(4, 2.0, np.float32), 1e-6),
        axpy_src=gate, axpy_dst=up, axpy_out=ref.axpy(0.37, gate, up),
        router_w=wf, router_x=xf, router_logits=ref.matvec_f32(wf, xf),
    )


def router(ref: orc.Reference) -> None:
    rng = np.random.default_rng(11)
    rows = []
    for case in range(ROUTER_CASES):
        E = int(rng.choice([4, 6, 8, 12, 16, 64, 160]))
        K = int(rng.integers(1, min(E, 8) + 1))
        n_group = int(rng.choice([1, 2, 4, 8, 3]))
        topk_group = int(rng.integers(1, 4))
        group_limited = bool(rng.integers(0, 2))
        norm = bool(rng.integers(0, 2))
        scale = float(rng.choice([1.0, 1.0, 2.5, 0.5]))
        logits = (rng.standard_normal(E) * 2).astype(np.float32)
        if case % 4 == 1:
            logits = np.round(logits)  # exact ties
        elif case % 4 == 2:
            logits[:] = 0.25  # all equal
        cfg = orc.RouterConfig(E, K, n_group, topk_group, group_limited, norm, scale)
        idx, w = ref.router_select(logits, cfg)
        rows.append((E, K, n_group, topk_group, int(group_limited), int(norm), scale, logits, idx, w))
    E_max, K_max = 160, 8
    np.savez_compressed(
        os.path.join(HERE, "router.npz"),
        params=np.array([r[:6] for r in rows], np.int64),
        scale=np.array([r[6] for r in rows], np.float32),
        logits=np.stack([np.pad(r[7], (0, E_max - r[7].size)) for r in rows]),
        idx=np.stack([np.pad(r[8], (0, K_max - r[8].size), constant_values=-1) for r in rows]),
        w=np.stack([np.pad(r[9], (0, K_max - r[9].size)) for r in rows]),
        count=np.array([r[8].size for r in rows], np.int64),
    )


def moe_small(ref: orc.Reference) -> None:
    cases = {}
    shapes = [
        ("testmodel", syn.MoeShape(hidden=32, inter=16, n_routed_experts=4, n_shared_experts=1, top_k=2),
         orc.RouterConfig(4, 2), 6, None),
        ("grouped", syn.MoeShape(hidden=64, inter=48, n_routed_experts=16, n_shared_experts=2, top_k=4),
         orc.RouterConfig(16, 4, 4, 2, True, True, 2.0), 9, None),
        ("biased", syn.MoeShape(hidden=96, inter=32, n_routed_experts=8, n_shared_experts=1, top_k=3),
         orc.RouterConfig(8, 3, 1, 1, False, False, 1.5), 7, "bias"),
    ]
    for name, shape, cfg, T, bias_kind in shapes:
        W = syn.layer_weights(shape, seed=21, std=0.08)
        x = syn.bf16_to_f32(syn.tokens(shape, T, seed=21)).reshape(T, shape.hidden)
        bias = syn.zipf_bias(shape, seed=21) if bias_kind else None
        y, idx, w, logits = ref.moe_layer(x, W, cfg, shape.n_shared_experts, bias=bias, threads=2)
        for k, v in W.items():
            cases[f"{name}_{k}"] = v
        cases[f"{name}_x"] = x
        if bias is not None:
            cases[f"{name}_bias"] = bias
        cases[f"{name}_y"] = y
        cases[f"{name}_idx"] = idx
        cases[f"{name}_w"] = w
        cases[f"{name}_logits"] = logits
        cases[f"{name}_shape"] = np.array([shape.hidden, shape.inter, shape.n_routed_experts,
                                           shape.n_shared_experts, shape.top_k], np.int64)
        cases[f"{name}_routing"] = np.array([cfg.n_group, cfg.topk_group, int(cfg.group_limited),
                                            int(cfg.norm_topk_prob)], np.int64)
        cases[f"{name}_scale"] = np.float32(cfg.routed_scaling_factor)
    np.savez_compressed(os.path.join(HERE, "moe_small.npz"), **cases)


def moe_v2lite(ref: orc.Reference) -> None:
    W = syn.layer_weights(syn.V2_LITE, seed=0)
    xb = syn.tokens(syn.V2_LITE, 3, seed=1)
    x = syn.bf16_to_f32(xb).reshape(3, -1)
    y, idx, w, logits = ref.moe_layer(x, W, orc.RouterConfig(), 2, threads=0)
    # A fingerprint of the regenerated weights guards against generator drift.
    fp = np.array([int(W[k].astype(np.uint64).sum()) for k in ("gate", "up", "down", "shared_gate",
                                                                 "shared_up", "shared_down")], np.uint64)
    np.savez_compressed(os.path.join(HERE, "moe_v2lite.npz"), x_bits=xb, y=y, idx=idx, w=w, logits=logits,
                        weight_fingerprint=fp, router_sum=np.float64(W["router"].astype(np.float64).sum()))


def cache(ref: orc.Reference) -> None:
    rng = np.random.default_rng(5)
    expert_elems = 1408 * 2048
    block = 3 * expert_elems * 2
    lib = ref.lib
    h = lib.ref_cache_new()
    lib.ref_cache_configure(h, 10 * block)
    touches, stats = [], []
    for step in range(300):
        layer, expert = int(rng.integers(0, 3)), int(rng.integers(0, 12))
        key = int(lib.ref_cache_make_key(layer, expert))
        lib.ref_cache_touch(h, key, expert_elems, expert_elems, expert_elems)
        s = np.zeros(6, np.uint64)
        lib.ref_cache_stats(h, s)
        touches.append([layer, expert])
        stats.append([int(v) for v in s])
    lib.ref_cache_clear(h)
    s = np.zeros(6, np.uint64)
    lib.ref_cache_stats(h, s)
    lib.ref_cache_free(h)
    with open(os.path.join(HERE, "cache.json"), "w") as f:
        json.dump({"budget_blocks": 10, "block_bytes": block, "touches": touches, "stats": stats,
                   "after_clear": [int(v) for v in s],
                   "stats_fields": ["resident_bytes", "resident_experts", "loads", "hits", "evictions",
                                    "bytes_streamed"]}, f)


def main() -> None:
    orc.build()
    ref = orc.Reference()
    kernels(ref)
    router(ref)
    moe_small(ref)
    moe_v2lite(ref)
    cache(ref)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
