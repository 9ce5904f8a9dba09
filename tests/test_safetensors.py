"""SafeTensors shards: the library's header parser (lm_safetensors_info, the front of
lm_moe_load_safetensors) against the reference's own SafeTensor::open/find
(src/SafeTensor.cpp:87-157, compiled into oracle/_ref) and against the `safetensors`
package, on well-formed and malformed shards.  No GPU needed.
"""
import json
import struct

import numpy as np
import pytest

from litemind_b200 import _lib
from litemind_b200 import synthetic as syn
from litemind_b200.checkpoint import layer_tensors, safetensors_info, write_safetensors

DT = {"BF16": _lib.LM_DTYPE_BF16, "F16": _lib.LM_DTYPE_F16, "F32": _lib.LM_DTYPE_F32}


def _tensors():
    rng = np.random.default_rng(5)
    return {
        "model.layers.3.mlp.experts.0.gate_proj.weight": ("BF16", syn.bf16_round(rng.standard_normal((6, 8)))),
        "model.layers.3.mlp.gate.weight": ("F32", rng.standard_normal((4, 8)).astype(np.float32)),
        "scale": ("F16", rng.standard_normal(5).astype(np.float16)),
        "empty": ("F32", np.zeros((0, 3), np.float32)),
    }


def test_writer_output_reads_back_with_the_safetensors_package(tmp_path):
    torch = pytest.importorskip("torch")
    st = pytest.importorskip("safetensors")
    path = tmp_path / "shard.safetensors"
    tensors = _tensors()
    write_safetensors(path, tensors, metadata={"format": "pt"})
    with st.safe_open(str(path), framework="pt") as f:
        assert set(f.keys()) == set(tensors)
        for name, (dtype, array) in tensors.items():
            got = f.get_tensor(name)
            if dtype == "BF16":
                np.testing.assert_array_equal(got.view(torch.int16).numpy().view(np.uint16), array)
            else:
                np.testing.assert_array_equal(got.numpy(), array)


def test_info_matches_reference_parser_and_payload(tmp_path, reference_lib):
    path = tmp_path / "shard.safetensors"
    tensors = _tensors()
    write_safetensors(path, tensors)
    raw = path.read_bytes()
    for name, (dtype, array) in tensors.items():
        info = safetensors_info(path, name)
        rc, rdtype, rshape, roffset, rnbytes, _ = reference_lib.safetensor_info(str(path), name)
        assert rc == 0
        assert (info["dtype"], info["shape"], info["offset"], info["nbytes"]) == (rdtype, rshape, roffset, rnbytes)
        assert info["dtype"] == DT[dtype] and info["shape"] == list(array.shape)
        assert raw[info["offset"]: info["offset"] + info["nbytes"]] == np.ascontiguousarray(array).tobytes()


def test_shards_written_by_the_safetensors_package(tmp_path, reference_lib):
    stn = pytest.importorskip("safetensors.numpy")
    path = tmp_path / "pkg.safetensors"
    arrays = {"a": np.arange(12, dtype=np.float32).reshape(3, 4), "b": np.ones(7, np.float16)}
    stn.save_file(arrays, str(path))
    for name, a in arrays.items():
        info = safetensors_info(path, name)
        assert info["shape"] == list(a.shape)
        assert reference_lib.safetensor_info(str(path), name)[1:5] == (info["dtype"], info["shape"], info["offset"],
                                                                         info["nbytes"])


def _shard(header_obj=None, header_bytes=None, payload=b"", length=None):
    body = header_bytes if header_bytes is not None else json.dumps(header_obj).encode()
    n = len(body) if length is None else length
    return struct.pack("<Q", n) + body + payload


MALFORMED = {
    "too short": b"\x01\x02\x03",
    "zero header": struct.pack("<Q", 0) + b"{}",
    "header past the end": _shard({"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}, length=10 ** 6),
    "not an object": _shard([1, 2, 3]),
    "bad json": _shard(header_bytes=b'{"a": {"dtype": "F32", '),
    "unknown dtype": _shard({"a": {"dtype": "Q8", "shape": [1], "data_offsets": [0, 1]}}, payload=b"\0"),
    "no shape": _shard({"a": {"dtype": "F32", "data_offsets": [0, 4]}}, payload=b"\0" * 4),
    "negative dim": _shard({"a": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, payload=b"\0" * 4),
    "descending offsets": _shard({"a": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}, payload=b"\0" * 4),
    "size mismatch": _shard({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}, payload=b"\0" * 4),
    "past the end": _shard({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, payload=b"\0" * 4),
    "no tensors": _shard({"__metadata__": {"k": "v"}}),
}


@pytest.mark.parametrize("case", sorted(MALFORMED))
def test_malformed_shards_are_rejected_as_the_reference_rejects_them(tmp_path, reference_lib, case):
    path = tmp_path / "bad.safetensors"
    path.write_bytes(MALFORMED[case])
    with pytest.raises(_lib.LiteMindError) as err:
        safetensors_info(path, "a")
    assert err.value.status == _lib.LM_ERR_INVALID_ARGUMENT
    rc, *_, ref_error = reference_lib.safetensor_info(str(path), "a")
    assert rc == 1, f"the reference accepted '{case}'"
    assert str(path) in ref_error and str(path) in str(err.value)


# Numbers the JSON header can hold but no shard can: rejected before any cast or
# product could wrap (a negative or fractional offset, an offset far past the end,
# a shape whose element count overflows 64 bits).
OUT_OF_RANGE = {
    "negative offset": _shard({"a": {"dtype": "F32", "shape": [1], "data_offsets": [-4, 0]}}, payload=b"\0" * 4),
    "fractional offset": _shard({"a": {"dtype": "F32", "shape": [1], "data_offsets": [0.5, 4.5]}},
                                payload=b"\0" * 8),
    "offset wraps": _shard({"a": {"dtype": "F32", "shape": [1], "data_offsets": [2 ** 64 - 2, 2 ** 64 + 2]}},
                           payload=b"\0" * 4),
    "shape overflows": _shard({"a": {"dtype": "F32", "shape": [2 ** 32, 2 ** 32, 4], "data_offsets": [0, 0]}},
                              payload=b"\0" * 4),
}


@pytest.mark.parametrize("case", sorted(OUT_OF_RANGE))
def test_out_of_range_numbers_are_rejected(tmp_path, case):
    path = tmp_path / "bad.safetensors"
    path.write_bytes(OUT_OF_RANGE[case])
    with pytest.raises(_lib.LiteMindError) as err:
        safetensors_info(path, "a")
    assert err.value.status == _lib.LM_ERR_INVALID_ARGUMENT
    assert str(path) in str(err.value)


def test_missing_tensor(tmp_path, reference_lib):
    path = tmp_path / "shard.safetensors"
    write_safetensors(path, _tensors())
    with pytest.raises(_lib.LiteMindError) as err:
        safetensors_info(path, "nope")
    assert err.value.status == _lib.LM_ERR_NOT_LOADED
    assert reference_lib.safetensor_info(str(path), "nope")[0] == 2


def test_layer_tensor_names_follow_the_deepseek_checkpoint():
    shape = syn.MoeShape(hidden=128, inter=64, n_routed_experts=4, n_shared_experts=2, top_k=2)
    names = set(layer_tensors(syn.layer_weights(shape, seed=1), 7, shape.n_shared_experts))
    assert "model.layers.7.mlp.gate.weight" in names
    assert "model.layers.7.post_attention_layernorm.weight" in names
    assert {f"model.layers.7.mlp.experts.3.{p}_proj.weight" for p in ("gate", "up", "down")} <= names
    assert "model.layers.7.mlp.shared_experts.down_proj.weight" in names
    assert len(names) == 2 + 3 * 4 + 3
