"""Dense feed-forward layers (lm_ffn_*) against the oracle's restatement of
Impl::feed_forward (src/DeepSeekRunner.cpp:228-240): gate and up matvecs, SiLU,
the down matvec accumulated with scale 1.  DeepSeek-V2-Lite's layer 0 is dense with
intermediate 10944 (include/Config.hpp:59); smaller shapes cover token counts."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import synthetic as syn  # noqa: E402
from litemind_b200._lib import LM_ERR_NOT_LOADED, LM_ERR_UNSUPPORTED, LiteMindError  # noqa: E402
from litemind_b200.checkpoint import write_safetensors  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor  # noqa: E402
from tests.parity import MAX_REL, MIN_COS, output_errors  # noqa: E402


def _weights(hidden, inter, seed, std):
    rng = np.random.default_rng(seed)
    g = syn.bf16_round(rng.normal(0, std, (inter, hidden)).astype(np.float32))
    u = syn.bf16_round(rng.normal(0, std, (inter, hidden)).astype(np.float32))
    d = syn.bf16_round(rng.normal(0, std, (hidden, inter)).astype(np.float32))
    return g, u, d


def _oracle_ffn(oracle_lib, g, u, d, x_f32):
    out = np.zeros((x_f32.shape[0], d.shape[0]), np.float32)
    for t, x in enumerate(x_f32):
        h = oracle_lib.silu_multiply(oracle_lib.matvec_bf16(g, x), oracle_lib.matvec_bf16(u, x))
        out[t] = oracle_lib.matvec_bf16_accumulate(d, h, out[t], 1.0)
    return out


def _check(y, ref, what):
    rel, cos = output_errors(y, ref)
    assert rel.max() <= MAX_REL, f"{what}: max relative error {rel.max():.3e}"
    assert cos.min() >= MIN_COS, f"{what}: min cosine {cos.min():.7f}"


@pytest.mark.parametrize("T", [1, 7, 64, 300])
def test_dense_ffn_small(oracle_lib, T):
    H, D = 512, 1024
    g, u, d = _weights(H, D, 1, 0.05)
    layer = MoeLayer(MoeConfig(hidden_size=H, moe_intermediate_size=256, n_routed_experts=8, num_experts_per_tok=2,
                               max_tokens=512))
    layer.ffn_upload(0, g, u, d)
    x = syn.tokens(syn.MoeShape(hidden=H, inter=256, n_routed_experts=8, n_shared_experts=2, top_k=2), T, seed=T)
    y = layer.ffn_forward(0, bf16_tensor(x))
    layer.sync()
    _check(y.cpu().numpy(), _oracle_ffn(oracle_lib, g, u, d, syn.bf16_to_f32(x).reshape(T, H)), f"dense T={T}")
    y2 = torch.ones_like(y)
    layer.ffn_forward(0, bf16_tensor(x), y=y2, accumulate=True)
    layer.sync()
    torch.testing.assert_close(y2 - 1.0, y, rtol=1e-5, atol=1e-5)
    layer.close()


def test_dense_ffn_v2lite_layer0(oracle_lib):
    H, D = 2048, 10944
    g, u, d = _weights(H, D, 2, 0.02)
    layer = MoeLayer(MoeConfig(max_tokens=64))
    layer.ffn_upload(0, g, u, d)
    for T in (3, 40):
        x = syn.tokens(syn.V2_LITE, T, seed=10 + T)
        y = layer.ffn_forward(0, bf16_tensor(x))
        layer.sync()
        rows = np.arange(T) if T <= 4 else np.array([0, T // 2, T - 1])
        ref = _oracle_ffn(oracle_lib, g, u, d, syn.bf16_to_f32(x).reshape(T, H)[rows])
        _check(y.cpu().numpy()[rows], ref, f"V2-Lite dense T={T}")
    layer.close()


def test_dense_block_and_safetensors(tmp_path, oracle_lib):
    H, D = 512, 768
    g, u, d = _weights(H, D, 3, 0.05)
    norm = np.linspace(0.5, 1.5, H).astype(np.float32)
    write_safetensors(tmp_path / "dense.safetensors", {
        "model.layers.0.mlp.gate_proj.weight": ("BF16", g), "model.layers.0.mlp.up_proj.weight": ("BF16", u),
        "model.layers.0.mlp.down_proj.weight": ("BF16", d), "model.layers.0.post_attention_layernorm.weight": ("F32", norm)})
    layer = MoeLayer(MoeConfig(hidden_size=H, moe_intermediate_size=256, n_routed_experts=8, num_experts_per_tok=2,
                               max_tokens=64))
    layer.ffn_load_safetensors(1, [tmp_path / "dense.safetensors"], intermediate=D, checkpoint_layer=0)
    T = 9
    hidden0 = np.random.default_rng(4).standard_normal((T, H)).astype(np.float32)
    hidden = torch.from_numpy(hidden0.copy()).cuda()
    layer.ffn_block_forward(1, hidden)
    layer.sync()
    xn = np.stack([oracle_lib.rms_norm(r, norm, 1e-6) for r in hidden0])
    ref = _oracle_ffn(oracle_lib, g, u, d, xn)
    _check(hidden.cpu().numpy() - hidden0, ref, "dense block")
    with pytest.raises(LiteMindError) as err:
        layer.ffn_forward(0, bf16_tensor(syn.bf16_round(hidden0)))
    assert err.value.status == LM_ERR_NOT_LOADED
    with pytest.raises(LiteMindError) as err:
        layer.ffn_upload(2, g[:100], u[:100], d[:, :100])
    assert err.value.status == LM_ERR_UNSUPPORTED
    layer.close()
