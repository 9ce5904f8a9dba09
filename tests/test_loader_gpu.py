"""lm_moe_load_safetensors: a MoE layer uploaded straight from SafeTensors shards
must run exactly as the same weights uploaded from host arrays, and a checkpoint
that does not fit the config must fail with the reference's messages."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import synthetic as syn  # noqa: E402
from litemind_b200._lib import LiteMindError  # noqa: E402
from litemind_b200.checkpoint import layer_tensors, write_safetensors  # noqa: E402
from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor  # noqa: E402

SHAPE = syn.MoeShape(hidden=512, inter=256, n_routed_experts=16, n_shared_experts=2, top_k=4)


def _split_write(tmp_path, tensors, n_shards=3):
    """Spread the tensors over several shards, round robin."""
    names = sorted(tensors)
    paths = []
    for k in range(n_shards):
        part = {n: tensors[n] for n in names[k::n_shards]}
        p = tmp_path / f"model-{k + 1:05d}-of-{n_shards:05d}.safetensors"
        write_safetensors(p, part, metadata={"format": "pt"})
        paths.append(p)
    return paths


@pytest.mark.parametrize("router_dtype", ["F32", "BF16"])
def test_loaded_layer_runs_like_uploaded_layer(tmp_path, router_dtype):
    weights = [syn.layer_weights(SHAPE, seed=3, layer=l, std=0.05) for l in range(2)]
    norm = np.linspace(0.8, 1.2, SHAPE.hidden).astype(np.float32)
    tensors = {}
    for l in range(2):
        tensors.update(layer_tensors(weights[l], l, SHAPE.n_shared_experts, norm, router_dtype=router_dtype))
    paths = _split_write(tmp_path, tensors)

    from_file = MoeLayer(MoeConfig.from_shape(SHAPE, max_tokens=64))
    from_file.load_safetensors(0, paths, checkpoint_layer=1)
    w = dict(weights[1])
    if router_dtype == "BF16":
        w["router"] = syn.bf16_to_f32(syn.bf16_round(w["router"])).reshape(w["router"].shape)
    from_host = MoeLayer(MoeConfig.from_shape(SHAPE, max_tokens=64))
    from_host.upload_layer(0, w, norm_weight=norm)
    for T in (5, 48):  # the fused decode path and the grouped path
        x = bf16_tensor(syn.tokens(SHAPE, T, seed=T))
        a = from_file.forward(0, x)
        b = from_host.forward(0, x)
        from_file.sync()
        from_host.sync()
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
        hidden = torch.randn(T, SHAPE.hidden, device="cuda")
        h1, h2 = hidden.clone(), hidden.clone()
        from_file.block_forward(0, h1)
        from_host.block_forward(0, h2)
        torch.testing.assert_close(h1, h2, rtol=1e-5, atol=1e-6)
    from_file.close()
    from_host.close()


def test_checkpoint_that_does_not_fit_the_config(tmp_path):
    weights = syn.layer_weights(SHAPE, seed=3, std=0.05)
    tensors = layer_tensors(weights, 0, SHAPE.n_shared_experts)
    paths = _split_write(tmp_path, tensors, n_shards=1)
    wrong = MoeLayer(MoeConfig.from_shape(syn.MoeShape(hidden=512, inter=128, n_routed_experts=16,
                                                       n_shared_experts=2, top_k=4), max_tokens=8))
    with pytest.raises(LiteMindError, match="has shape"):
        wrong.load_safetensors(0, paths)
    missing = dict(tensors)
    del missing["model.layers.0.mlp.experts.9.down_proj.weight"]
    (tmp_path / "missing").mkdir()
    paths2 = _split_write(tmp_path / "missing", missing, n_shards=1)
    right = MoeLayer(MoeConfig.from_shape(SHAPE, max_tokens=8))
    with pytest.raises(LiteMindError, match="has no tensor named 'model.layers.0.mlp.experts.9.down_proj.weight'"):
        right.load_safetensors(0, paths2)
    with pytest.raises(LiteMindError, match="has no tensor named"):
        right.load_safetensors(0, paths, checkpoint_layer=5)
    wrong.close()
    right.close()
