"""The MoE block on the GPU against the oracle (oracle/moe_oracle.c).

Small shapes cover the ragged cases (empty experts, one expert taking every token,
every token-tile width); DeepSeek-V2-Lite shapes cover the benchmark
configurations.  Where T is too large for the CPU oracle to finish in seconds, a
sample of tokens is checked: tokens are independent, so the oracle run on the
sample must reproduce those rows of the GPU output.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import synthetic as syn  # noqa: E402
from litemind_b200._lib import LM_ERR_INVALID_ARGUMENT, LM_ERR_NOT_LOADED, LM_ERR_TOO_MANY_TOKENS, LiteMindError  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor  # noqa: E402
from oracle.oracle import RouterConfig  # noqa: E402
from tests.parity import assert_layer_parity  # noqa: E402

SMALL = syn.MoeShape(hidden=256, inter=128, n_routed_experts=8, n_shared_experts=1, top_k=2)


def run_gpu(layer: MoeLayer, x_bits, bias=None):
    x = bf16_tensor(x_bits)
    b = None if bias is None else torch.from_numpy(bias).cuda()
    y = layer.forward(0, x, bias=b)
    idx, w, logits = layer.route(0, x, bias=b)
    layer.sync()
    return y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), logits.cpu().numpy()


def run_oracle(oracle_lib, shape, W, x_bits, bias=None):
    x = syn.bf16_to_f32(x_bits).reshape(x_bits.shape)
    cfg = RouterConfig(shape.n_routed_experts, shape.top_k)
    return oracle_lib.moe_layer(x, W, cfg, shape.n_shared_experts, bias=bias, threads=0)


@pytest.fixture(scope="module")
def small_layer():
    W = syn.layer_weights(SMALL, seed=11, std=0.1)
    layer = MoeLayer(MoeConfig.from_shape(SMALL, max_tokens=4096))
    layer.upload_layer(0, W)
    yield layer, W
    layer.close()


@pytest.mark.parametrize("T", [1, 2, 5, 37, 64, 65, 300, 1000, 4096])
def test_small_shape_parity(oracle_lib, small_layer, T):
    layer, W = small_layer
    x = syn.tokens(SMALL, T, seed=T)
    y, idx, w, _ = run_gpu(layer, x)
    ry, ridx, rw, rlog = run_oracle(oracle_lib, SMALL, W, x)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"small T={T}")


def test_all_tokens_on_one_expert(oracle_lib, small_layer):
    layer, W = small_layer
    bias = np.full(SMALL.n_routed_experts, -30.0, np.float32)
    bias[5] = 30.0
    bias[2] = 20.0  # second choice for everyone; six experts get nothing
    x = syn.tokens(SMALL, 333, seed=5)
    y, idx, w, _ = run_gpu(layer, x, bias)
    assert (idx[:, 0] == 5).all() and (idx[:, 1] == 2).all()
    counts = layer.expert_counts()
    assert counts[5] == 333 and counts[2] == 333 and counts.sum() == 666
    ry, ridx, rw, rlog = run_oracle(oracle_lib, SMALL, W, x, bias)
    assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what="one expert")


def test_zero_tokens_and_errors(small_layer):
    layer, _ = small_layer
    x = bf16_tensor(syn.tokens(SMALL, 1, seed=1))
    y = torch.full((1, SMALL.hidden), 7.0, device="cuda")
    layer.forward(0, x[:0], y=y[:0])  # T = 0 is a no-op
    layer.sync()
    assert float(y[0, 0]) == 7.0
    with pytest.raises(LiteMindError) as e:
        layer.forward(1, x)
    assert e.value.status == LM_ERR_INVALID_ARGUMENT
    big = torch.zeros((4097, SMALL.hidden), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(LiteMindError) as e:
        layer.forward(0, big)
    assert e.value.status == LM_ERR_TOO_MANY_TOKENS
    fresh = MoeLayer(MoeConfig.from_shape(SMALL, max_tokens=16))
    with pytest.raises(LiteMindError) as e:
        fresh.forward(0, x)
    assert e.value.status == LM_ERR_NOT_LOADED
    fresh.close()


def test_accumulate_adds_to_output(small_layer):
    layer, _ = small_layer
    x = bf16_tensor(syn.tokens(SMALL, 50, seed=9))
    y0 = layer.forward(0, x)
    y1 = torch.ones_like(y0)
    layer.forward(0, x, y=y1, accumulate=True)
    layer.sync()
    torch.testing.assert_close(y1 - 1.0, y0, rtol=1e-5, atol=1e-5)


def test_forward_host_matches_device(small_layer):
    layer, _ = small_layer
    xb = syn.tokens(SMALL, 77, seed=3)
    y_dev = layer.forward(0, bf16_tensor(xb))
    layer.sync()
    y_host = layer.forward_host(0, xb)
    np.testing.assert_allclose(y_host, y_dev.cpu().numpy(), rtol=1e-5, atol=1e-6)


def _page_locked(nbytes: int):
    """A zeroed page-locked host buffer with 64 spare bytes (room for a misaligned start)."""
    return torch.zeros(nbytes + 64, dtype=torch.uint8).pin_memory()


def _read_f32(buf, offset: int, shape):
    return np.frombuffer(buf.numpy().tobytes()[offset:offset + 4 * int(np.prod(shape))], np.float32).reshape(shape)


@pytest.mark.parametrize("T,offset,with_bias", [(77, 0, False), (77, 2, False), (1, 0, True), (16, 0, True),
                                                (16, 4, True), (300, 0, False), (1000, 0, True)])
def test_forward_host_page_locked_buffers(small_layer, T, offset, with_bias):
    """Page-locked buffers: 16-byte aligned ones move by SM loads and stores over mapped
    memory, misaligned ones (offset 2 or 4) by copy-engine transfers; both must give the
    device-buffer forward's result, on two calls in a row.  Up to 256 tokens the fused
    kernel runs between the pull and push kernels; 300 and 1000 tokens take the grouped
    launches (1000: tensor-core router logits), whose first kernel must wait for the pull."""
    layer, _ = small_layer
    xb = syn.tokens(SMALL, T, seed=T + 3)
    bias = np.linspace(-1.0, 1.0, SMALL.n_routed_experts).astype(np.float32) if with_bias else None
    y_dev = layer.forward(0, bf16_tensor(xb), bias=None if bias is None else torch.from_numpy(bias).cuda())
    layer.sync()
    x_buf = _page_locked(xb.nbytes)
    x_buf.numpy()[offset:offset + xb.nbytes] = np.ascontiguousarray(xb).view(np.uint8).reshape(-1)
    b_ptr = None
    if bias is not None:
        b_buf = _page_locked(bias.nbytes)
        b_buf.numpy()[offset:offset + bias.nbytes] = bias.view(np.uint8)
        b_ptr = b_buf.data_ptr() + offset
    y_buf = _page_locked(T * SMALL.hidden * 4)
    for call in range(2):
        layer.forward_host_ptr(0, x_buf.data_ptr() + offset, T, y_buf.data_ptr() + offset, b_ptr)
        y = _read_f32(y_buf, offset, (T, SMALL.hidden))
        np.testing.assert_allclose(y, y_dev.cpu().numpy(), rtol=1e-5, atol=1e-6, err_msg=f"call {call}")


# ── DeepSeek-V2-Lite shapes ────────────────────────────────────────────────

@pytest.fixture(scope="module")
def v2_layer(v2lite_weights):
    layer = MoeLayer(MoeConfig(max_tokens=16384))
    layer.upload_layer(0, v2lite_weights)
    yield layer
    layer.close()


@pytest.mark.parametrize("T,seed", [(1, 1), (8, 1), (32, 1), (128, 0), (256, 1)])
def test_v2lite_decode_parity(oracle_lib, v2lite_weights, v2_layer, T, seed):
    """The V2-Lite layer at T=128 (token seed 0) and at decode sizes T in 1/8/32/256 (token seed 1)."""
    x = syn.tokens(syn.V2_LITE, T, seed=seed)
    y, idx, w, _ = run_gpu(v2_layer, x)
    ry, ridx, rw, rlog = run_oracle(oracle_lib, syn.V2_LITE, v2lite_weights, x)
    stats = assert_layer_parity(y, idx, w, ry, ridx, rw, rlog, what=f"V2-Lite T={T}")
    print(f"T={T}: {stats}")


@pytest.mark.parametrize("T", [1, 32, 128])
def test_v2lite_forward_host_page_locked(v2lite_weights, v2_layer, T):
    """The host entry with page-locked buffers (the e2e measurement's form) at decode sizes,
    where the fused kernel runs between the pull and push kernels."""
    xb = syn.tokens(syn.V2_LITE, T, seed=T)
    y_dev = v2_layer.forward(0, bf16_tensor(xb))
    v2_layer.sync()
    x_host = torch.from_numpy(np.ascontiguousarray(xb).view(np.int16)).pin_memory()
    y_host = torch.empty((T, syn.V2_LITE.hidden), dtype=torch.float32).pin_memory()
    for _ in range(2):
        v2_layer.forward_host_ptr(0, x_host.data_ptr(), T, y_host.data_ptr())
        np.testing.assert_allclose(y_host.numpy(), y_dev.cpu().numpy(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("T,zipf", [(2048, False), (4096, False), (16384, True)])
def test_v2lite_prefill_sampled_parity(oracle_lib, v2lite_weights, v2_layer, T, zipf):
    """Prefill: T=16384 with a Zipf(1.2) expert load, and 2048- and 4096-token batches
    (about 384 rows per expert at 4096: each expert's last token block runs narrow)."""
    x = syn.tokens(syn.V2_LITE, T, seed=2)
    bias = syn.zipf_bias(syn.V2_LITE, seed=2) if zipf else None
    y, idx, w, _ = run_gpu(v2_layer, x, bias)
    counts = v2_layer.expert_counts()
    assert counts.sum() == T * 6
    np.testing.assert_array_equal(np.bincount(idx.reshape(-1), minlength=64), counts)
    sample = np.random.default_rng(T).choice(T, 48, replace=False)
    sample.sort()
    ry, ridx, rw, rlog = run_oracle(oracle_lib, syn.V2_LITE, v2lite_weights, x[sample], bias)
    assert_layer_parity(y[sample], idx[sample], w[sample], ry, ridx, rw, rlog, what=f"V2-Lite T={T}")
