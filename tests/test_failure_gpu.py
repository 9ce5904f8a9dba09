"""Failure detection on the GPU without a GPU fault.

The fused decode kernel waits on grid-wide arrival counters; every such wait is
bounded and, when it runs out, the kernel records a status code in device memory
and returns instead of hanging.  Here the host-side testing knob
(lm_moe_debug_set) makes each wait expect one arrival more than the grid provides
-- a flag that nothing sets -- with a short limit.  The forward must then report
LM_ERR_DEVICE_TIMEOUT within about the limit, and the very next forward (knob
cleared) must succeed and match the oracle: the context stays usable because the
error path re-arms every counter.  Nothing here faults, traps or hangs a GPU.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import _lib, synthetic as syn  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor  # noqa: E402
from oracle.oracle import Oracle, RouterConfig  # noqa: E402
from tests.parity import assert_layer_parity  # noqa: E402

SHAPE = syn.MoeShape(hidden=512, inter=256, n_routed_experts=16, n_shared_experts=2, top_k=4)
LIMIT_NS = 50_000_000  # 50 ms


@pytest.fixture(scope="module")
def setup():
    W = syn.layer_weights(SHAPE, seed=11, std=0.05)
    layer = MoeLayer(MoeConfig.from_shape(SHAPE, max_tokens=64), device=0)
    layer.upload_layer(0, W)
    yield layer, W
    layer.close()


def _oracle(W, xb):
    ry, ridx, rw, rlog = Oracle().moe_layer(syn.bf16_to_f32(xb).reshape(xb.shape), W,
                                            RouterConfig(SHAPE.n_routed_experts, SHAPE.top_k),
                                            SHAPE.n_shared_experts)
    return ry, ridx, rw, rlog


def _check_ok(layer, W, xb, y):
    idx, w, _ = layer.route(0, bf16_tensor(xb))
    layer.sync()
    assert_layer_parity(y, idx.cpu().numpy(), w.cpu().numpy(), *_oracle(W, xb), what="after recovery")


@pytest.mark.parametrize("T", [4, 32])
def test_expired_grid_wait_reports_timeout_and_context_recovers(setup, T):
    layer, W = setup
    xb = syn.tokens(SHAPE, T, seed=12)
    x = bf16_tensor(xb)
    layer.debug_set(_lib.LM_DEBUG_WAIT_LIMIT_NS, LIMIT_NS)
    layer.debug_set(_lib.LM_DEBUG_GRID_EXTRA, 1)
    try:
        t0 = time.perf_counter()
        layer.forward(0, x)
        with pytest.raises(_lib.LiteMindError) as err:
            layer.sync()
        elapsed = time.perf_counter() - t0
    finally:
        layer.debug_set(_lib.LM_DEBUG_GRID_EXTRA, 0)
        layer.debug_set(_lib.LM_DEBUG_WAIT_LIMIT_NS, 0)
    assert err.value.status == _lib.LM_ERR_DEVICE_TIMEOUT
    assert "bounded wait" in str(err.value)
    assert elapsed < 1.5, f"the expired wait took {elapsed:.2f} s (limit {LIMIT_NS / 1e9} s)"
    # A second sync has nothing left to report.
    layer.sync()
    # The counters were re-armed: the next forwards run normally, twice in a row.
    for _ in range(2):
        y = layer.forward(0, x)
        layer.sync()
    _check_ok(layer, W, xb, y.cpu().numpy())


@pytest.mark.parametrize("page_locked", [False, True])
def test_host_entry_reports_timeout_with_one_sync(setup, page_locked):
    """lm_moe_forward_host reads the status word back with y: the same error, no hang.
    Pageable buffers come back by copy-engine transfers; page-locked ones by the push
    kernel, which copies the status word too."""
    layer, W = setup
    xb = syn.tokens(SHAPE, 16, seed=13)

    def call():
        if not page_locked:
            return layer.forward_host(0, xb)
        x_host = torch.from_numpy(np.ascontiguousarray(xb).view(np.int16)).pin_memory()
        y_host = torch.empty((16, SHAPE.hidden), dtype=torch.float32).pin_memory()
        layer.forward_host_ptr(0, x_host.data_ptr(), 16, y_host.data_ptr())
        return y_host.numpy().copy()

    layer.debug_set(_lib.LM_DEBUG_WAIT_LIMIT_NS, LIMIT_NS)
    layer.debug_set(_lib.LM_DEBUG_GRID_EXTRA, 3)
    try:
        with pytest.raises(_lib.LiteMindError) as err:
            call()
    finally:
        layer.debug_set(_lib.LM_DEBUG_GRID_EXTRA, 0)
        layer.debug_set(_lib.LM_DEBUG_WAIT_LIMIT_NS, 0)
    assert err.value.status == _lib.LM_ERR_DEVICE_TIMEOUT
    _check_ok(layer, W, xb, call())


def test_debug_knobs_are_checked(setup):
    layer, _ = setup
    for knob, value in ((_lib.LM_DEBUG_GRID_EXTRA, 5000), (_lib.LM_DEBUG_WAIT_LIMIT_NS, 10 ** 10), (99, 1),
                        (_lib.LM_DEBUG_GRID_EXTRA, -1)):
        with pytest.raises(_lib.LiteMindError) as err:
            layer.debug_set(knob, value)
        assert err.value.status == _lib.LM_ERR_INVALID_ARGUMENT


def test_ep_init_refuses_nccl_copy_engine_mode(monkeypatch):
    """NCCL's copy-engine peer transfers are refused before NCCL is touched."""
    monkeypatch.setenv("NCCL_P2P_USE_CUDA_MEMCPY", "1")
    layer = MoeLayer(MoeConfig.from_shape(SHAPE, max_tokens=16), device=0)
    try:
        with pytest.raises(_lib.LiteMindError) as err:
            layer.ep_init(bytes(128), 0, 1)
        assert err.value.status == _lib.LM_ERR_UNSUPPORTED
        assert "NCCL_P2P_USE_CUDA_MEMCPY" in str(err.value)
    finally:
        layer.close()
