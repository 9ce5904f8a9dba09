"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Two libraries sit behind the same numpy-level functions:

* ``Oracle`` -- ``oracle/_build/libmoe_oracle.so``, the C restatement of the
  reference's MoE path (``oracle/moe_oracle.c``);
* ``Reference`` -- ``oracle/_ref/libref_litemind.so``, the reference's own sources
  (src/Gemm.cpp, src/MoeRouter.cpp, src/ExpertCache.cpp, ...) compiled by
  ``oracle/Makefile`` with ``oracle/ref_harness.cpp``.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module; it is the checker, never the thing measured or shipped.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libmoe_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_litemind.so")
# The reference checkout: LITEMIND_REFERENCE_DIR, else a directory named `reference`
# beside this repository's root.
REFERENCE_DIR = os.environ.get("LITEMIND_REFERENCE_DIR") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")


def build(reference_dir: str | None = None) -> None:
    """Builds both checkers (the reference one only when its sources exist)."""
    ref = reference_dir or REFERENCE_DIR
    cmd = ["make", "-s", "-C", HERE, f"REF={ref}"]
    subprocess.run(cmd, check=True)


@dataclass
class RouterConfig:
    """The routing fields of the reference's Config (include/Config.hpp:59-71)."""

    n_routed_experts: int = 64
    num_experts_per_tok: int = 6
    n_group: int = 1
    topk_group: int = 1
    group_limited: bool = False
    norm_topk_prob: bool = False
    routed_scaling_factor: float = 1.0


class _OrcRouter(C.Structure):
    _fields_ = [("expert_count", C.c_int64), ("top_k", C.c_int64), ("n_group", C.c_int64),
                ("topk_group", C.c_int64), ("group_limited", C.c_int32), ("normalize", C.c_int32),
                ("routed_scaling_factor", C.c_float)]


class _OrcShape(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("inter", C.c_int64), ("n_shared", C.c_int64),
                ("router", _OrcRouter)]


def _opt(arr):
    return None if arr is None else arr.ctypes.data_as(C.c_void_p)


class _Base:
    prefix = ""

    def __init__(self, path: str):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built; run `make -C oracle`")
        self.lib = C.CDLL(path)

    # --- kernels ---------------------------------------------------------
    def matvec_bf16(self, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        rows, cols = w.shape
        out = np.zeros(rows, np.float32)
        self._matvec_bf16(np.ascontiguousarray(w, np.uint16), np.ascontiguousarray(x, np.float32),
                          out, rows, cols)
        return out

    def matvec_bf16_accumulate(self, w, x, out, scale):
        rows, cols = w.shape
        out = np.ascontiguousarray(out, np.float32).copy()
        self._matvec_bf16_acc(np.ascontiguousarray(w, np.uint16), np.ascontiguousarray(x, np.float32),
                              out, rows, cols, scale)
        return out

    def matvec_f32(self, w, x):
        rows, cols = w.shape
        out = np.zeros(rows, np.float32)
        fn = getattr(self.lib, self.prefix + "matvec_f32")
        fn.argtypes = [_f32p, _f32p, _f32p, C.c_int64 if self.prefix == "ref_" else C.c_size_t,
                       C.c_int64 if self.prefix == "ref_" else C.c_size_t]
        fn(np.ascontiguousarray(w, np.float32), np.ascontiguousarray(x, np.float32), out, rows, cols)
        return out

    def softmax(self, v):
        v = np.ascontiguousarray(v, np.float32).copy()
        fn = getattr(self.lib, self.prefix + "softmax")
        fn.argtypes = [_f32p, C.c_int64 if self.prefix == "ref_" else C.c_size_t]
        fn(v, v.size)
        return v

    def silu_multiply(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        d = np.zeros_like(g)
        fn = getattr(self.lib, self.prefix + "silu_multiply")
        fn.argtypes = [_f32p, _f32p, _f32p, C.c_int64 if self.prefix == "ref_" else C.c_size_t]
        fn(g, u, d, g.size)
        return d

    def rms_norm(self, v, w, eps):
        v = np.ascontiguousarray(v, np.float32).copy()
        fn = getattr(self.lib, self.prefix + "rms_norm")
        fn.argtypes = [_f32p, _f32p, C.c_int64 if self.prefix == "ref_" else C.c_size_t, C.c_float]
        fn(v, np.ascontiguousarray(w, np.float32), v.size, eps)
        return v

    def axpy(self, scale, src, dst):
        dst = np.ascontiguousarray(dst, np.float32).copy()
        fn = getattr(self.lib, self.prefix + "axpy")
        fn.argtypes = [C.c_float, _f32p, _f32p, C.c_int64 if self.prefix == "ref_" else C.c_size_t]
        fn(scale, np.ascontiguousarray(src, np.float32), dst, dst.size)
        return dst


class Oracle(_Base):
    """The C restatement (oracle/moe_oracle.c)."""

    prefix = "orc_"

    def __init__(self, path: str = ORACLE_SO):
        super().__init__(path)
        L = self.lib
        L.orc_matvec_bf16.argtypes = [_u16p, _f32p, _f32p, C.c_size_t, C.c_size_t]
        L.orc_matvec_bf16_accumulate.argtypes = [_u16p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_float]
        L.orc_router_init.argtypes = [C.POINTER(_OrcRouter), C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                      C.c_int32, C.c_int32, C.c_float]
        L.orc_router_select.argtypes = [C.POINTER(_OrcRouter), _f32p, C.c_int64, _i64p, _f32p]
        L.orc_router_select.restype = C.c_int64
        L.orc_select_top_k.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int32, _i64p, _f32p]
        L.orc_select_top_k.restype = C.c_int64
        L.orc_moe_layer.argtypes = [C.POINTER(_OrcShape), C.c_int64, _f32p, _f32p, C.c_void_p,
                                    _u16p, _u16p, _u16p, _u16p, _u16p, _u16p, _f32p, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_int]
        L.orc_moe_layer.restype = C.c_int
        L.orc_f32_to_bf16.argtypes = [C.c_float]
        L.orc_f32_to_bf16.restype = C.c_uint16
        self._matvec_bf16 = L.orc_matvec_bf16
        self._matvec_bf16_acc = L.orc_matvec_bf16_accumulate

    def _router(self, cfg: RouterConfig) -> _OrcRouter:
        r = _OrcRouter()
        self.lib.orc_router_init(C.byref(r), cfg.n_routed_experts, cfg.num_experts_per_tok, cfg.n_group,
                                 cfg.topk_group, int(cfg.group_limited), int(cfg.norm_topk_prob),
                                 cfg.routed_scaling_factor)
        return r

    def router_select(self, logits: np.ndarray, cfg: RouterConfig):
        logits = np.ascontiguousarray(logits, np.float32)
        k = max(cfg.num_experts_per_tok, 1)
        idx = np.zeros(max(k, logits.size), np.int64)
        w = np.zeros(max(k, logits.size), np.float32)
        n = self.lib.orc_router_select(C.byref(self._router(cfg)), logits, logits.size, idx, w)
        return idx[:n].copy(), w[:n].copy()

    def select_top_k(self, logits, expert_count, top_k, normalize):
        logits = np.ascontiguousarray(logits, np.float32)
        idx = np.zeros(max(top_k, 1), np.int64)
        w = np.zeros(max(top_k, 1), np.float32)
        n = self.lib.orc_select_top_k(logits, logits.size, expert_count, top_k, int(normalize), idx, w)
        if n < 0:
            raise ValueError("MoE routing requires one logit per expert and a valid top-k value.")
        return idx[:n].copy(), w[:n].copy()

    def moe_layer(self, x, weights, cfg: RouterConfig, n_shared: int, bias=None, threads: int = 0):
        """x: [T, H] f32.  weights: dict from litemind_b200.synthetic (gate/up/down/...)."""
        T, H = x.shape
        I = weights["gate"].shape[1]
        shape = _OrcShape(H, I, n_shared, self._router(cfg))
        E, K = cfg.n_routed_experts, cfg.num_experts_per_tok
        y = np.zeros((T, H), np.float32)
        idx = np.zeros((T, K), np.int64)
        w = np.zeros((T, K), np.float32)
        logits = np.zeros((T, E), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        rc = self.lib.orc_moe_layer(
            C.byref(shape), T, np.ascontiguousarray(x, np.float32), weights["router"], _opt(b),
            weights["gate"], weights["up"], weights["down"], weights["shared_gate"],
            weights["shared_up"], weights["shared_down"], y, _opt(idx), _opt(w), _opt(logits),
            threads)
        if rc != 0:
            raise RuntimeError(f"orc_moe_layer failed ({rc})")
        return y, idx, w, logits


class Reference(_Base):
    """The reference's own code (oracle/_ref/libref_litemind.so)."""

    prefix = "ref_"

    def __init__(self, path: str = REF_SO):
        super().__init__(path)
        L = self.lib
        L.ref_hardware_threads.restype = C.c_int64
        L.ref_kernel_description.restype = C.c_char_p
        L.ref_matvec_bf16.argtypes = [_u16p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int]
        L.ref_matvec_bf16_serial.argtypes = [_u16p, _f32p, _f32p, C.c_int64, C.c_int64]
        L.ref_matvec_bf16_accumulate.argtypes = [_u16p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_float,
                                                 C.c_int]
        L.ref_router_select.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                        C.c_int32, C.c_int32, C.c_float, _i64p, _f32p]
        L.ref_router_select.restype = C.c_int64
        L.ref_select_top_k.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int32, _i64p, _f32p]
        L.ref_select_top_k.restype = C.c_int64
        L.ref_moe_layer.argtypes = [C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                    C.c_int64, C.c_int32, C.c_int32, C.c_float, C.c_int64, _f32p, _f32p,
                                    C.c_void_p, _u16p, _u16p, _u16p, _u16p, _u16p, _u16p, _f32p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.ref_moe_layer.restype = C.c_int
        L.ref_kerneltest_inputs.argtypes = [_f32p, _u16p, _f32p]
        L.ref_cache_new.restype = C.c_void_p
        L.ref_cache_free.argtypes = [C.c_void_p]
        L.ref_cache_configure.argtypes = [C.c_void_p, C.c_uint64]
        L.ref_cache_touch.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64]
        L.ref_cache_clear.argtypes = [C.c_void_p]
        L.ref_cache_stats.argtypes = [C.c_void_p, _u64p]
        L.ref_cache_make_key.argtypes = [C.c_uint64, C.c_uint64]
        L.ref_cache_make_key.restype = C.c_uint64
        L.ref_safetensor_info.argtypes = [C.c_char_p, C.c_char_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_char_p, C.c_int32]
        L.ref_safetensor_info.restype = C.c_int
        self.threads = 0
        self._matvec_bf16 = lambda w, x, out, r, c: L.ref_matvec_bf16(w, x, out, r, c, self.threads)
        self._matvec_bf16_acc = lambda w, x, out, r, c, s: L.ref_matvec_bf16_accumulate(
            w, x, out, r, c, s, self.threads)

    def safetensor_info(self, path: str, name: str):
        """SafeTensor::open + find on one shard: (status, dtype, shape, offset, nbytes, error);
        status 0 found, 1 shard rejected, 2 no such tensor."""
        dtype, ndim = C.c_int32(0), C.c_int32(0)
        shape = (C.c_int64 * 8)()
        offset, nbytes = C.c_uint64(0), C.c_uint64(0)
        err = C.create_string_buffer(1024)
        rc = self.lib.ref_safetensor_info(path.encode(), name.encode(), C.byref(dtype), C.byref(ndim), shape,
                                          C.byref(offset), C.byref(nbytes), err, len(err))
        return rc, dtype.value, list(shape[: ndim.value]), offset.value, nbytes.value, err.value.decode()

    def kerneltest_inputs(self):
        """tests/KernelTest.cpp's seeded 67x253 inputs: (w_f32, w_bf16, x)."""
        w32 = np.zeros(67 * 253, np.float32)
        w16 = np.zeros(67 * 253, np.uint16)
        x = np.zeros(253, np.float32)
        self.lib.ref_kerneltest_inputs(w32, w16, x)
        return w32.reshape(67, 253), w16.reshape(67, 253), x

    def hardware_threads(self) -> int:
        return int(self.lib.ref_hardware_threads())

    def kernel_description(self) -> str:
        return self.lib.ref_kernel_description().decode()

    def matvec_bf16_serial(self, w, x):
        rows, cols = w.shape
        out = np.zeros(rows, np.float32)
        self.lib.ref_matvec_bf16_serial(np.ascontiguousarray(w, np.uint16),
                                        np.ascontiguousarray(x, np.float32), out, rows, cols)
        return out

    def router_select(self, logits, cfg: RouterConfig):
        logits = np.ascontiguousarray(logits, np.float32)
        k = max(cfg.num_experts_per_tok, 1)
        idx = np.zeros(max(k, logits.size), np.int64)
        w = np.zeros(max(k, logits.size), np.float32)
        n = self.lib.ref_router_select(logits, logits.size, cfg.n_routed_experts, cfg.num_experts_per_tok,
                                       cfg.n_group, cfg.topk_group, int(cfg.group_limited),
                                       int(cfg.norm_topk_prob), cfg.routed_scaling_factor, idx, w)
        return idx[:n].copy(), w[:n].copy()

    def select_top_k(self, logits, expert_count, top_k, normalize):
        logits = np.ascontiguousarray(logits, np.float32)
        idx = np.zeros(max(top_k, 1), np.int64)
        w = np.zeros(max(top_k, 1), np.float32)
        n = self.lib.ref_select_top_k(logits, logits.size, expert_count, top_k, int(normalize), idx, w)
        if n < 0:
            raise ValueError("MoE routing requires one logit per expert and a valid top-k value.")
        return idx[:n].copy(), w[:n].copy()

    def moe_layer(self, x, weights, cfg: RouterConfig, n_shared: int, bias=None, threads: int = 0):
        T, H = x.shape
        I = weights["gate"].shape[1]
        E, K = cfg.n_routed_experts, cfg.num_experts_per_tok
        y = np.zeros((T, H), np.float32)
        idx = np.zeros((T, K), np.int64)
        w = np.zeros((T, K), np.float32)
        logits = np.zeros((T, E), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        rc = self.lib.ref_moe_layer(
            H, I, n_shared, E, K, cfg.n_group, cfg.topk_group, int(cfg.group_limited),
            int(cfg.norm_topk_prob), cfg.routed_scaling_factor, T, np.ascontiguousarray(x, np.float32),
            weights["router"], _opt(b), weights["gate"], weights["up"], weights["down"],
            weights["shared_gate"], weights["shared_up"], weights["shared_down"], y, _opt(idx), _opt(w),
            _opt(logits), threads)
        if rc != 0:
            raise RuntimeError(f"ref_moe_layer failed ({rc})")
        return y, idx, w, logits


def oracle() -> Oracle:
    return Oracle()


def reference_available() -> bool:
    return os.path.exists(REF_SO)


def reference() -> Reference:
    return Reference()
