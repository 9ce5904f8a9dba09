"""The gemm:: kernels on device memory (lm_gemm_*, include/litemind_b200/Gemm.hpp)
against the reference's own known-answer tests.

Inputs and expected values come from tests/golden/kernels.npz: the seeded 67 x 253
matvec of the reference's tests/KernelTest.cpp:28-79 (widths deliberately not a
multiple of any vector width), its accumulate case (1 + 0.5 W x), the softmax
stability case at logits 1000/1001 and the SiLU and RMSNorm cases (:81-110), each
with the reference's own outputs recorded by tests/golden/make_golden.py.
Tolerances are KernelTest's: 1e-3 against the double-precision matvec, 1e-6 for
softmax sums and SiLU, 1e-5 for RMSNorm.  Larger aligned shapes check the
vectorised path against a float64 product.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from litemind_b200 import _lib  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kernels.npz")


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    return torch.from_numpy(a).cuda()


def p(t):
    return C.c_void_p(t.data_ptr())


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def run(status):
    assert status == _lib.LM_OK
    torch.cuda.synchronize()


def test_matvec_bf16_kerneltest_case(lib, g):
    rows, cols = g["kt_w_bf16"].shape
    w, x = dev(g["kt_w_bf16"]), dev(g["kt_x"])
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    run(lib.lm_gemm_matvec_bf16(p(w), p(x), p(out), rows, cols, stream()))
    y = out.cpu().numpy()
    np.testing.assert_allclose(y, g["kt_expected"], rtol=0, atol=1e-3)  # tests/KernelTest.cpp:62-64
    np.testing.assert_allclose(y, g["kt_matvec"], rtol=0, atol=1e-4)   # the reference's own result
    np.testing.assert_allclose(y, g["kt_serial"], rtol=0, atol=1e-4)


def test_matvec_bf16_accumulate_kerneltest_case(lib, g):
    rows, cols = g["kt_w_bf16"].shape
    w, x = dev(g["kt_w_bf16"]), dev(g["kt_x"])
    out = torch.ones(rows, dtype=torch.float32, device="cuda")
    run(lib.lm_gemm_matvec_bf16_accumulate(p(w), p(x), p(out), rows, cols, 0.5, stream()))
    y = out.cpu().numpy()
    np.testing.assert_allclose(y, 1.0 + 0.5 * g["kt_expected"], rtol=0, atol=1e-3)  # :74-78
    np.testing.assert_allclose(y, g["kt_accumulate"], rtol=0, atol=1e-4)


@pytest.mark.parametrize("rows,cols", [(2048, 2048), (1408, 2048), (2048, 1408), (37, 10944), (5, 8)])
def test_matvec_bf16_aligned_shapes(lib, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    wf = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    wb = (wf.view(np.uint32) >> 16).astype(np.uint16)  # truncated to bf16 bits
    wref = (wb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    x = rng.standard_normal(cols).astype(np.float32)
    expected = wref @ x.astype(np.float64)
    w, xd = dev(wb), dev(x)
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    run(lib.lm_gemm_matvec_bf16(p(w), p(xd), p(out), rows, cols, stream()))
    scale = np.abs(wref) @ np.abs(x.astype(np.float64))  # bound of the f32 rounding error per row
    err = np.abs(out.cpu().numpy() - expected)
    assert (err <= 1e-5 * scale + 1e-6).all(), f"max error {err.max():.3e}"
    acc = torch.full((rows,), 2.0, dtype=torch.float32, device="cuda")
    run(lib.lm_gemm_matvec_bf16_accumulate(p(w), p(xd), p(acc), rows, cols, -1.5, stream()))
    err = np.abs(acc.cpu().numpy() - (2.0 - 1.5 * expected))
    assert (err <= 1.5e-5 * scale + 1e-5).all(), f"max error {err.max():.3e}"


def test_matvec_f32_router_case(lib, g):
    w, x = dev(g["router_w"]), dev(g["router_x"])
    rows, cols = g["router_w"].shape
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    run(lib.lm_gemm_matvec_f32(p(w), p(x), p(out), rows, cols, stream()))
    expected = g["router_w"].astype(np.float64) @ g["router_x"].astype(np.float64)
    np.testing.assert_allclose(out.cpu().numpy(), expected, rtol=0, atol=1e-5)
    np.testing.assert_allclose(out.cpu().numpy(), g["router_logits"], rtol=0, atol=1e-5)  # reference's sequential sum


def test_softmax_cases(lib, g):
    for i in range(3):
        v = dev(g[f"softmax_in_{i}"].astype(np.float32))
        run(lib.lm_gemm_softmax(p(v), 1, v.numel(), stream()))
        r = v.cpu().numpy()
        assert np.isfinite(r).all(), "softmax is stable at large logits"  # tests/KernelTest.cpp:98-101
        assert abs(float(r.astype(np.float64).sum()) - 1.0) <= 1e-6
        np.testing.assert_allclose(r, g[f"softmax_out_{i}"], rtol=1e-6, atol=1e-7)
    # Several rows in one call, each normalised on its own.
    rows = np.stack([g["softmax_in_2"], g["softmax_in_2"] + 5.0, -g["softmax_in_2"]]).astype(np.float32)
    v = dev(rows)
    run(lib.lm_gemm_softmax(p(v), 3, rows.shape[1], stream()))
    r = v.cpu().numpy()
    np.testing.assert_allclose(r[0], g["softmax_out_2"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(r[1], g["softmax_out_2"], rtol=1e-5, atol=1e-7)  # shift-invariant
    np.testing.assert_allclose(r.sum(axis=1), 1.0, atol=1e-6)


def test_silu_multiply_cases(lib, g):
    gate, up = dev(g["silu_gate"]), dev(g["silu_up"])
    out = torch.zeros_like(gate)
    run(lib.lm_gemm_silu_multiply(p(gate), p(up), p(out), gate.numel(), stream()))
    np.testing.assert_allclose(out.cpu().numpy(), g["silu_out"], rtol=1e-6, atol=1e-6)
    # tests/KernelTest.cpp:104-110: silu(0) * 3 = 0 and silu(1) * 2.
    gate2, up2 = dev(np.array([0.0, 1.0], np.float32)), dev(np.array([3.0, 2.0], np.float32))
    out2 = torch.zeros(2, dtype=torch.float32, device="cuda")
    run(lib.lm_gemm_silu_multiply(p(gate2), p(up2), p(out2), 2, stream()))
    r = out2.cpu().numpy()
    assert abs(r[0]) <= 1e-6 and abs(r[1] - 2.0 / (1.0 + np.exp(-1.0))) <= 1e-6


def test_rms_norm_cases(lib, g):
    v, w = dev(g["rms_in"]), dev(g["rms_w"])
    run(lib.lm_gemm_rms_norm(p(v), p(w), 1, v.numel(), 1e-6, stream()))
    np.testing.assert_allclose(v.cpu().numpy(), g["rms_out"], rtol=1e-5, atol=1e-6)
    k = dev(g["rms_known_in"])
    two = dev(np.full(4, 2.0, np.float32))
    run(lib.lm_gemm_rms_norm(p(k), p(two), 1, 4, 1e-6, stream()))
    scale = 2.0 / np.sqrt(7.5 + 1e-6)  # tests/KernelTest.cpp:82-88
    np.testing.assert_allclose(k.cpu().numpy(), np.arange(1, 5) * scale, rtol=0, atol=1e-5)
    np.testing.assert_allclose(k.cpu().numpy(), g["rms_known_out"], rtol=0, atol=1e-6)


def test_axpy_case(lib, g):
    src, dst = dev(g["axpy_src"]), dev(g["axpy_dst"])
    run(lib.lm_gemm_axpy(0.37, p(src), p(dst), src.numel(), stream()))
    # The reference's `dst += scale * src` compiles to one fused multiply-add, as here.
    np.testing.assert_array_equal(dst.cpu().numpy(), g["axpy_out"])
