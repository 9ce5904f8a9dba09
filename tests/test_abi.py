"""The C ABI library without a GPU: it loads, exports every entry point that
include/*.h declares, validates arguments before touching the device, and fails
loudly (LM_ERR_CUDA) instead of computing on the CPU when no GPU is present."""
import ctypes as C
import glob
import os
import re

import pytest

from litemind_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(lm_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from litemind_b200 import build

    if not os.path.exists(_lib.LIB_PATH):
        build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_default_config_is_deepseek_v2_lite(lib):
    c = _lib.LmMoeConfig()
    lib.lm_moe_config_default(C.byref(c))
    assert (c.hidden_size, c.moe_intermediate_size, c.n_routed_experts, c.n_shared_experts,
            c.num_experts_per_tok, c.norm_topk_prob, c.topk_method) == (2048, 1408, 64, 2, 6, 0, 0)
    assert c.routed_scaling_factor == 1.0 and abs(c.rms_norm_eps - 1e-6) < 1e-12


def _create(lib, **kw):
    c = _lib.LmMoeConfig()
    lib.lm_moe_config_default(C.byref(c))
    for k, v in kw.items():
        setattr(c, k, v)
    h = C.c_void_p()
    return lib.lm_moe_create(C.byref(c), 0, C.byref(h)), h


def test_create_validates_config_first(lib):
    # Config::validate (src/Config.cpp:172-175): top-k may not exceed the experts.
    assert _create(lib, num_experts_per_tok=65)[0] == _lib.LM_ERR_INVALID_ARGUMENT
    assert _create(lib, hidden_size=0)[0] == _lib.LM_ERR_INVALID_ARGUMENT
    assert _create(lib, topk_method=7)[0] == _lib.LM_ERR_INVALID_ARGUMENT
    assert _create(lib, hidden_size=2000)[0] == _lib.LM_ERR_UNSUPPORTED  # tiles need multiples of 128
    assert _create(lib, n_routed_experts=300, num_experts_per_tok=6)[0] == _lib.LM_ERR_UNSUPPORTED
    assert lib.lm_moe_create(None, 0, None) == _lib.LM_ERR_INVALID_ARGUMENT


def test_no_gpu_is_an_error_not_a_fallback(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    status, handle = _create(lib)
    assert status == _lib.LM_ERR_CUDA and not handle.value


def test_null_context_and_arguments(lib):
    assert lib.lm_moe_forward(None, 0, None, 1, None, None, 0, None) == _lib.LM_ERR_INVALID_ARGUMENT
    assert lib.lm_moe_destroy(None) == _lib.LM_OK
    assert lib.lm_moe_sync(None, None) == _lib.LM_ERR_INVALID_ARGUMENT
    assert lib.lm_gemm_matvec_bf16(None, None, None, -1, 4, None) == _lib.LM_ERR_INVALID_ARGUMENT
    assert lib.lm_gemm_matvec_bf16(None, None, None, 0, 4, None) == _lib.LM_OK  # empty: nothing to do
    assert lib.lm_gemm_softmax(None, 3, 0, None) == _lib.LM_OK  # src/Gemm.cpp:210-212
    assert lib.lm_gemm_axpy(1.0, None, None, 5, None) == _lib.LM_ERR_INVALID_ARGUMENT


def test_new_entry_points_check_their_arguments(lib):
    assert lib.lm_moe_debug_set(None, _lib.LM_DEBUG_GRID_EXTRA, 0) == _lib.LM_ERR_INVALID_ARGUMENT
    assert lib.lm_moe_expert_counts(None, None, 64) == _lib.LM_ERR_INVALID_ARGUMENT
    buf = C.create_string_buffer(128)
    assert lib.lm_moe_ep_init(None, buf, 0, 1) == _lib.LM_ERR_INVALID_ARGUMENT


def test_kernel_description_names_the_b200_kernels(lib):
    text = lib.lm_kernel_description().decode()
    assert "sm_100a" in text and "tcgen05" in text


def test_status_strings(lib):
    for code in range(8):
        assert lib.lm_status_string(code)
    assert lib.lm_status_string(99) == b"unknown status"


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError):
        _lib.load(str(tmp_path / "absent.so"))
