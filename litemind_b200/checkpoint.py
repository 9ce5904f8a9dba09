"""SafeTensors checkpoints of MoE layers: a writer (for synthetic checkpoints and
tests) and a header lookup through the library (lm_safetensors_info).

Tensor names follow DeepSeek checkpoints as DeepSeekRunner::Impl::resolve_layer
reads them (src/DeepSeekRunner.cpp:157-224 of the reference).  The writer lays a
shard out as the format prescribes: an 8-byte little-endian header length, the JSON
header (padded with spaces so the payload starts 8-byte aligned), then each tensor's
bytes in header order.  BF16 tensors are given as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct

import numpy as np

from . import _lib

_DTYPES = {"BF16": (np.uint16, 2), "F16": (np.float16, 2), "F32": (np.float32, 4)}


def write_safetensors(path: str | os.PathLike, tensors: dict, metadata: dict | None = None) -> None:
    """tensors: name -> (dtype, array) with dtype 'BF16' (uint16 bits), 'F16' or 'F32'."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs, offset = [], 0
    for name, (dtype, array) in tensors.items():
        np_type, _ = _DTYPES[dtype]
        data = np.ascontiguousarray(array, dtype=np_type).tobytes()
        header[name] = {"dtype": dtype, "shape": list(np.shape(array)), "data_offsets": [offset, offset + len(data)]}
        blobs.append(data)
        offset += len(data)
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * ((-(8 + len(text))) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for b in blobs:
            f.write(b)


def layer_tensors(weights: dict, layer: int, n_shared: int, norm_weight: np.ndarray | None = None,
                  router_dtype: str = "F32") -> dict:
    """The checkpoint tensors of one MoE layer from a litemind_b200.synthetic weight dict."""
    p = f"model.layers.{layer}."
    E, I, H = weights["gate"].shape
    router = weights["router"]
    if router_dtype == "BF16":
        from .synthetic import bf16_round
        router = bf16_round(router)
    elif router_dtype == "F16":
        router = router.astype(np.float16)
    out = {p + "mlp.gate.weight": (router_dtype, router)}
    norm = np.ones(H, np.float32) if norm_weight is None else norm_weight
    out[p + "post_attention_layernorm.weight"] = ("F32", norm)
    for e in range(E):
        q = f"{p}mlp.experts.{e}."
        out[q + "gate_proj.weight"] = ("BF16", weights["gate"][e])
        out[q + "up_proj.weight"] = ("BF16", weights["up"][e])
        out[q + "down_proj.weight"] = ("BF16", weights["down"][e])
    if n_shared > 0:
        q = p + "mlp.shared_experts."
        out[q + "gate_proj.weight"] = ("BF16", weights["shared_gate"])
        out[q + "up_proj.weight"] = ("BF16", weights["shared_up"])
        out[q + "down_proj.weight"] = ("BF16", weights["shared_down"])
    return out


def safetensors_info(path: str | os.PathLike, name: str) -> dict:
    """lm_safetensors_info: one tensor's header entry, or LiteMindError with the reason."""
    lib = _lib.load()
    dtype, ndim = C.c_int32(0), C.c_int32(0)
    shape = (C.c_int64 * _lib.LM_SAFETENSORS_MAX_DIMS)()
    offset, nbytes = C.c_uint64(0), C.c_uint64(0)
    err = C.create_string_buffer(1024)
    rc = lib.lm_safetensors_info(str(path).encode(), name.encode(), C.byref(dtype), C.byref(ndim), shape,
                                 C.byref(offset), C.byref(nbytes), err, len(err))
    if rc != _lib.LM_OK:
        raise _lib.LiteMindError(rc, err.value.decode())
    return {"dtype": dtype.value, "shape": list(shape[: ndim.value]), "offset": offset.value, "nbytes": nbytes.value}
