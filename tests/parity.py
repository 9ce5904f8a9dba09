"""Parity criteria shared by the GPU tests.

Routing: the top-k expert indices must equal the oracle's, except where the two
experts that trade places have router probabilities within ROUTE_TIE of each other
(the GPU's f32 logits are summed in a different order than the reference's
sequential dot, src/Gemm.cpp:183-189).  Outputs: for every token whose routing
matched, max |y - y_ref| / max |y_ref| <= MAX_REL and cosine(y, y_ref) >= MIN_COS
(f32 accumulation; the expert activations pass through bf16 on the tensor cores).
"""
from __future__ import annotations

import numpy as np

ROUTE_TIE = 1e-6
MAX_REL = 1e-2
MIN_COS = 0.9999
# Routing weights: softmax probabilities of f32 logits.  Large bf16 batches get their
# logits from the tensor cores (the f32 router split exactly into three bf16 parts),
# whose f32 accumulation is coarser than a CUDA-core sum: up to ~2e-5 relative.
WEIGHT_RTOL = 1e-4


def softmax64(logits: np.ndarray) -> np.ndarray:
    z = logits.astype(np.float64)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


def routing_mismatches(idx: np.ndarray, ref_idx: np.ndarray, ref_logits: np.ndarray):
    """Returns (exempt_tokens, bad_tokens): tokens whose selection differs only at
    near-ties, and tokens that differ otherwise."""
    probs = softmax64(ref_logits)
    exempt, bad = [], []
    for t in range(idx.shape[0]):
        if np.array_equal(idx[t], ref_idx[t]):
            continue
        p = probs[t]
        ok = True
        for a, b in zip(idx[t], ref_idx[t]):
            if a != b and abs(p[int(a)] - p[int(b)]) > ROUTE_TIE:
                ok = False
        (exempt if ok else bad).append(t)
    return exempt, bad


def output_errors(y: np.ndarray, ref: np.ndarray):
    """Per-token (max relative error, cosine)."""
    y = y.astype(np.float64)
    ref = ref.astype(np.float64)
    denom = np.maximum(np.abs(ref).max(axis=-1), 1e-30)
    rel = np.abs(y - ref).max(axis=-1) / denom
    cos = (y * ref).sum(-1) / np.maximum(np.linalg.norm(y, axis=-1) * np.linalg.norm(ref, axis=-1), 1e-30)
    return rel, cos


def assert_layer_parity(y, idx, w, ref_y, ref_idx, ref_w, ref_logits, what=""):
    exempt, bad = routing_mismatches(idx, ref_idx, ref_logits)
    assert not bad, f"{what}: routing differs beyond near-ties for tokens {bad[:10]}"
    keep = np.ones(y.shape[0], bool)
    keep[exempt] = False
    assert keep.sum() > 0 or y.shape[0] == 0
    np.testing.assert_allclose(w[keep], ref_w[keep], rtol=WEIGHT_RTOL, atol=1e-7, err_msg=what)
    rel, cos = output_errors(y[keep], ref_y[keep])
    assert rel.max(initial=0.0) <= MAX_REL, f"{what}: max relative error {rel.max():.3e} > {MAX_REL}"
    assert cos.min(initial=1.0) >= MIN_COS, f"{what}: min cosine {cos.min():.7f} < {MIN_COS}"
    return {"exempt": len(exempt), "max_rel": float(rel.max(initial=0.0)), "min_cos": float(cos.min(initial=1.0))}


def sampled_oracle_parity(y, x_bits, W, rows, bias=None) -> dict:
    """Sampled tokens of a V2-Lite-shaped batch against the CPU oracle (the
    reference's MoE block restated in C): per token max |y - y_ref| / max |y_ref| and
    cosine, leaving out tokens whose 6th and 7th router probabilities lie within
    ROUTE_TIE (either expert is a correct choice there).  y: [T, H] f32 output of
    the GPU path; x_bits: [T, H] bf16 bits of its input; W: its weights."""
    from litemind_b200 import synthetic as syn
    from oracle.oracle import Oracle, RouterConfig

    rows = np.asarray(rows)
    xs = syn.bf16_to_f32(x_bits[rows]).reshape(len(rows), -1)
    n_shared = W["shared_gate"].shape[0] // W["gate"].shape[1]
    cfg = RouterConfig(W["router"].shape[0], 6)
    ry, _, _, rlog = Oracle().moe_layer(xs, W, cfg, n_shared, bias=bias)
    p = np.sort(softmax64(rlog), axis=1)[:, ::-1]
    k = cfg.num_experts_per_tok
    tie = (p[:, k - 1] - p[:, k]) <= ROUTE_TIE
    rel, cos = output_errors(y[rows][~tie], ry[~tie])
    return {"tokens": int(len(rows)), "exempt_near_ties": int(tie.sum()),
            "max_rel": float(rel.max(initial=0.0)), "min_cos": float(cos.min(initial=1.0)),
            "pass": bool(rel.max(initial=0.0) <= MAX_REL and cos.min(initial=1.0) >= MIN_COS),
            "criteria": f"max_rel <= {MAX_REL}, cosine >= {MIN_COS} (fp32 accumulate); oracle = the reference's "
                        "MoE block restated in C"}
