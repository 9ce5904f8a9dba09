"""lm_moe_route_static: routing that allocates no device memory.

Some callers cannot allocate: code inside a CUDA graph capture, plugins whose host
application owns every device allocation, paths that must not trigger an
allocation's synchronisation.  lm_moe_route_static serves them with a fixed scratch
array inside the library.  This test calls it through the C ABI and checks, on two calls in
a row (the second call reuses the scratch the first one left behind), that it
routes as the context-based entry point lm_moe_route does and as the CPU oracle
(the reference's gemm::matvec_f32 + MoeRouter::select, restated in C) does, and
that a batch beyond the scratch's capacity is refused.  It lives in its own file, collected
last, and needs nothing from the other tests.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import _lib, synthetic as syn  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor  # noqa: E402
from oracle.oracle import Oracle, RouterConfig  # noqa: E402
from tests.parity import routing_mismatches  # noqa: E402

SHAPE = syn.MoeShape(hidden=512, inter=128, n_routed_experts=64, n_shared_experts=1, top_k=6)
W_RTOL = 1e-4  # routing weights, as in tests/parity.py


def _static_route(lib, router, x, bias, k, norm=False, scale=1.0):
    T, H = x.shape
    E = router.shape[0]
    idx = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    w = torch.zeros((T, k), dtype=torch.float32, device="cuda")
    status = lib.lm_moe_route_static(C.c_void_p(router.data_ptr()), C.c_void_p(x.data_ptr()), T, H, E, k, int(norm),
                                     scale, None if bias is None else C.c_void_p(bias.data_ptr()),
                                     C.c_void_p(idx.data_ptr()), C.c_void_p(w.data_ptr()),
                                     C.c_void_p(torch.cuda.current_stream().cuda_stream))
    return status, idx, w


def test_static_route_matches_context_route():
    lib = _lib.load()
    W = syn.layer_weights(SHAPE, seed=4, std=0.02)
    layer = MoeLayer(MoeConfig.from_shape(SHAPE, max_tokens=2048))
    layer.upload_layer(0, W)
    router = torch.from_numpy(W["router"]).cuda()
    bias = torch.from_numpy(syn.zipf_bias(SHAPE, seed=4)).cuda()
    for call, (T, b) in enumerate([(1000, None), (37, bias)]):  # two calls in a row
        x = bf16_tensor(syn.tokens(SHAPE, T, seed=40 + call))
        status, idx, w = _static_route(lib, router, x, b, SHAPE.top_k)
        assert status == _lib.LM_OK
        ref_idx, ref_w, ref_logits = layer.route(0, x, bias=b)
        torch.cuda.synchronize()
        # The two entry points may sum the logits in different orders (CUDA cores
        # here, tensor cores for large batches there): indices must agree except
        # where two experts' probabilities are within 1e-6, as everywhere else.
        idx, ref_idx, w, ref_w = idx.cpu().numpy(), ref_idx.cpu().numpy(), w.cpu().numpy(), ref_w.cpu().numpy()
        exempt, bad = routing_mismatches(idx, ref_idx, ref_logits.cpu().numpy())
        assert not bad, f"call {call}: routing differs beyond near-ties for tokens {bad[:10]}"
        keep = np.ones(T, bool)
        keep[exempt] = False
        np.testing.assert_allclose(w[keep], ref_w[keep], rtol=W_RTOL, atol=1e-8, err_msg=f"call {call}")
        # The oracle: per token, f32 logits (+ bias), then the reference's selection.
        orc = Oracle()
        xf = syn.bf16_to_f32(x.view(torch.int16).cpu().numpy().view(np.uint16)).reshape(T, -1)
        bias_np = None if b is None else b.cpu().numpy()
        o_logits = np.stack([orc.matvec_f32(W["router"], xf[t]) for t in range(T)])
        if bias_np is not None:
            o_logits = o_logits + bias_np
        cfg = RouterConfig(SHAPE.n_routed_experts, SHAPE.top_k)
        sel = [orc.router_select(o_logits[t], cfg) for t in range(T)]
        o_idx = np.stack([i for i, _ in sel]).astype(np.int32)
        o_w = np.stack([v for _, v in sel])
        exempt, bad = routing_mismatches(idx, o_idx, o_logits)
        assert not bad, f"call {call}: routing differs from the oracle beyond near-ties for tokens {bad[:10]}"
        keep = np.ones(T, bool)
        keep[exempt] = False
        np.testing.assert_allclose(w[keep], o_w[keep], rtol=W_RTOL, atol=1e-8, err_msg=f"call {call} vs oracle")
    layer.close()


def test_static_route_refuses_batches_beyond_its_scratch():
    lib = _lib.load()
    router = torch.zeros((64, 512), dtype=torch.float32, device="cuda")
    x = torch.zeros((2048, 512), dtype=torch.bfloat16, device="cuda")
    status, _, _ = _static_route(lib, router, x, None, 6)
    assert status == _lib.LM_ERR_TOO_MANY_TOKENS
    status, _, _ = _static_route(lib, router, x[:0], None, 6)
    assert status == _lib.LM_OK
