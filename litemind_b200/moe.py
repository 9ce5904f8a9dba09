"""Host-side mirror of the reference's MoE interfaces over the C ABI.

``MoeRouter`` keeps the reference's ``MoeRouter`` semantics (include/MoeRouter.hpp:27-55):
``select(logits)`` returns ``ExpertSelection`` entries in descending weight with the
lower index first on ties, an empty list when the logit count is wrong
(src/MoeRouter.cpp:57-59), and ``select_top_k`` raises ``ValueError`` where the
reference throws ``std::invalid_argument`` (src/MoeRouter.cpp:119-121).
``MoeLayer`` is the batched MoE block (src/DeepSeekRunner.cpp:264-290) with HBM
residency.  Device memory, streams and tensors are PyTorch plumbing; all
arithmetic runs in liblitemind_b200.so on the GPU.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import LmMoeConfig, check, load
from .synthetic import MoeShape

try:  # torch is the device-memory plumbing for Python callers
    import torch
except ImportError:  # pragma: no cover
    torch = None


@dataclass
class MoeConfig:
    """The Config fields of the MoE path (include/Config.hpp:59-71)."""

    hidden_size: int = 2048
    moe_intermediate_size: int = 1408
    n_routed_experts: int = 64
    n_shared_experts: int = 2
    num_experts_per_tok: int = 6
    norm_topk_prob: bool = False
    routed_scaling_factor: float = 1.0
    topk_method: str = "greedy"
    n_group: int = 1
    topk_group: int = 1
    rms_norm_eps: float = 1e-6
    num_layers: int = 1
    max_tokens: int = 16384

    @classmethod
    def from_shape(cls, shape: MoeShape, **kw) -> "MoeConfig":
        return cls(hidden_size=shape.hidden, moe_intermediate_size=shape.inter,
                   n_routed_experts=shape.n_routed_experts, n_shared_experts=shape.n_shared_experts,
                   num_experts_per_tok=shape.top_k, **kw)

    def to_c(self) -> LmMoeConfig:
        if self.topk_method not in ("greedy", "group_limited_greedy"):
            raise ValueError(f"unsupported topk_method '{self.topk_method}'")
        return LmMoeConfig(self.hidden_size, self.moe_intermediate_size, self.n_routed_experts,
                           self.n_shared_experts, self.num_experts_per_tok, int(self.norm_topk_prob),
                           float(self.routed_scaling_factor),
                           _lib.LM_TOPK_GROUP_LIMITED_GREEDY if self.topk_method == "group_limited_greedy"
                           else _lib.LM_TOPK_GREEDY,
                           self.n_group, self.topk_group, float(self.rms_norm_eps), self.num_layers,
                           self.max_tokens)


@dataclass
class ExpertSelection:
    """One routed-expert decision (include/MoeRouter.hpp:12-15)."""

    expert_index: int
    weight: float


def ep_plan(nranks: int, send_expert_counts, recv_expert_counts, chunks: int = 1, chunk: int = 0) -> dict:
    """lm_moe_ep_plan (chunks = 1) or lm_moe_ep_chunk_plan: send/recv row counts and
    offsets of one expert-parallel forward, or of one chunk of its local experts."""
    s = np.ascontiguousarray(send_expert_counts, np.int32)
    r = np.ascontiguousarray(recv_expert_counts, np.int32)
    plan = _lib.LmEpPlan()
    if chunks == 1 and chunk == 0:
        check(load().lm_moe_ep_plan(nranks, s.size, C.c_void_p(s.ctypes.data), C.c_void_p(r.ctypes.data),
                                    C.byref(plan)))
    else:
        check(load().lm_moe_ep_chunk_plan(nranks, s.size, chunks, chunk, C.c_void_p(s.ctypes.data),
                                          C.c_void_p(r.ctypes.data), C.byref(plan)))
    return {"send_count": list(plan.send_count[:nranks]), "send_offset": list(plan.send_offset[:nranks]),
            "recv_count": list(plan.recv_count[:nranks]), "recv_offset": list(plan.recv_offset[:nranks]),
            "n_send": plan.n_send, "n_recv": plan.n_recv}


def _ptr(t) -> C.c_void_p | None:
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return C.c_void_p(t.ctypes.data)
    return C.c_void_p(t.data_ptr())


def _stream_ptr(stream) -> C.c_void_p | None:
    if stream is None:
        return C.c_void_p(torch.cuda.current_stream().cuda_stream) if torch is not None else None
    return C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def bf16_tensor(bits: np.ndarray, device="cuda"):
    """uint16 bf16 bits (numpy) -> torch.bfloat16 tensor on `device`."""
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t.to(device) if device is not None else t


class MoeLayer:
    """The MoE block on one B200: weights resident, T tokens per call."""

    def __init__(self, config: MoeConfig, device: int = 0):
        self.lib = load()
        self.config = config
        self.device = device
        self._cfg = config.to_c()
        handle = C.c_void_p()
        status = self.lib.lm_moe_create(C.byref(self._cfg), device, C.byref(handle))
        check(status)
        self.ctx = handle

    # --- lifetime ----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "ctx", None):
            self.lib.lm_moe_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, status: int) -> None:
        check(status, self.ctx)

    # --- residency ---------------------------------------------------------
    def upload_layer(self, layer: int, weights: dict, norm_weight: np.ndarray | None = None) -> None:
        w = {k: np.ascontiguousarray(v) for k, v in weights.items()}
        norm = None if norm_weight is None else np.ascontiguousarray(norm_weight, np.float32)
        self._check(self.lib.lm_moe_upload_layer(
            self.ctx, layer, _ptr(w["router"]), _ptr(w["gate"]), _ptr(w["up"]), _ptr(w["down"]),
            _ptr(w["shared_gate"]), _ptr(w["shared_up"]), _ptr(w["shared_down"]), _ptr(norm)))

    def load_safetensors(self, layer: int, shard_paths, checkpoint_layer: int | None = None) -> None:
        """lm_moe_load_safetensors: this context's layer slot from a SafeTensors checkpoint."""
        paths = [str(p).encode() for p in shard_paths]
        arr = (C.c_char_p * len(paths))(*paths)
        self._check(self.lib.lm_moe_load_safetensors(self.ctx, layer, layer if checkpoint_layer is None
                                                     else checkpoint_layer, arr, len(paths)))

    # ── dense feed-forward layers (their own index space) ──
    def ffn_upload(self, layer: int, gate, up, down, norm_weight: np.ndarray | None = None) -> None:
        """gate/up [inter, hidden], down [hidden, inter] as bf16 bits (numpy uint16)."""
        g, u, d = (np.ascontiguousarray(a, np.uint16) for a in (gate, up, down))
        n = None if norm_weight is None else np.ascontiguousarray(norm_weight, np.float32)
        self._check(self.lib.lm_ffn_upload(self.ctx, layer, g.shape[0], _ptr(g), _ptr(u), _ptr(d), _ptr(n)))

    def ffn_load_safetensors(self, layer: int, shard_paths, intermediate: int, checkpoint_layer: int | None = None):
        paths = [str(p).encode() for p in shard_paths]
        arr = (C.c_char_p * len(paths))(*paths)
        self._check(self.lib.lm_ffn_load_safetensors(self.ctx, layer, layer if checkpoint_layer is None
                                                     else checkpoint_layer, intermediate, arr, len(paths)))

    def ffn_forward(self, layer: int, x, y=None, accumulate: bool = False, stream=None):
        T = x.shape[0]
        if y is None:
            y = torch.empty((T, self.config.hidden_size), dtype=torch.float32, device=x.device)
        self._check(self.lib.lm_ffn_forward(self.ctx, layer, _ptr(x) if T else None, T, _ptr(y) if T else None,
                                            int(accumulate), _stream_ptr(stream)))
        return y

    def ffn_block_forward(self, layer: int, hidden, stream=None):
        self._check(self.lib.lm_ffn_block_forward(self.ctx, layer, _ptr(hidden), hidden.shape[0],
                                                  _stream_ptr(stream)))

    def upload_expert(self, layer: int, expert: int, gate, up, down) -> None:
        g, u, d = (np.ascontiguousarray(a) for a in (gate, up, down))
        self._check(self.lib.lm_moe_upload_expert(self.ctx, layer, expert, _ptr(g), _ptr(u), _ptr(d)))

    # --- expert parallelism --------------------------------------------------
    @staticmethod
    def ep_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(load().lm_moe_ep_unique_id(buf))
        return buf.raw

    def ep_init(self, unique_id: bytes, rank: int, nranks: int) -> None:
        """Joins the expert-parallel group; call before uploading weights."""
        buf = C.create_string_buffer(bytes(unique_id), 128)
        self._check(self.lib.lm_moe_ep_init(self.ctx, buf, rank, nranks))

    def memory(self) -> tuple[int, int]:
        r, u = C.c_uint64(), C.c_uint64()
        self._check(self.lib.lm_moe_memory(self.ctx, C.byref(r), C.byref(u)))
        return r.value, u.value

    # --- compute -----------------------------------------------------------
    def forward(self, layer: int, x, bias=None, y=None, accumulate: bool = False, stream=None):
        """x: cuda bf16 [T, hidden] -> y: cuda f32 [T, hidden]."""
        T = x.shape[0]
        if y is None:
            y = torch.empty((T, self.config.hidden_size), dtype=torch.float32, device=x.device)
        xp = _ptr(x) if T > 0 else None
        yp = _ptr(y) if T > 0 else None
        self._check(self.lib.lm_moe_forward(self.ctx, layer, xp, T, _ptr(bias), yp, int(accumulate),
                                            _stream_ptr(stream)))
        return y

    def forward_host(self, layer: int, x_bits: np.ndarray, bias: np.ndarray | None = None,
                     out: np.ndarray | None = None) -> np.ndarray:
        """Host bf16 bits [T, hidden] -> host f32 [T, hidden]; copies inside the call."""
        x_bits = np.ascontiguousarray(x_bits)
        T = x_bits.shape[0]
        if out is None:
            out = np.empty((T, self.config.hidden_size), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self._check(self.lib.lm_moe_forward_host(self.ctx, layer, _ptr(x_bits), T, _ptr(b), _ptr(out)))
        return out

    def forward_host_ptr(self, layer: int, x_ptr: int, T: int, y_ptr: int, bias_ptr: int | None = None) -> None:
        """lm_moe_forward_host on raw host pointers (pinned buffers in the bench)."""
        self._check(self.lib.lm_moe_forward_host(self.ctx, layer, C.c_void_p(x_ptr), T,
                                                 None if bias_ptr is None else C.c_void_p(bias_ptr),
                                                 C.c_void_p(y_ptr)))

    def route(self, layer: int, x, bias=None, stream=None):
        T = x.shape[0]
        K, E = self.config.num_experts_per_tok, self.config.n_routed_experts
        idx = torch.empty((T, K), dtype=torch.int32, device=x.device)
        w = torch.empty((T, K), dtype=torch.float32, device=x.device)
        logits = torch.empty((T, E), dtype=torch.float32, device=x.device)
        self._check(self.lib.lm_moe_route(self.ctx, layer, _ptr(x), T, _ptr(bias), _ptr(idx), _ptr(w),
                                          _ptr(logits), _stream_ptr(stream)))
        return idx, w, logits

    def select(self, logits, stream=None):
        T = logits.shape[0]
        K = self.config.num_experts_per_tok
        idx = torch.empty((T, K), dtype=torch.int32, device=logits.device)
        w = torch.empty((T, K), dtype=torch.float32, device=logits.device)
        self._check(self.lib.lm_moe_select(self.ctx, _ptr(logits), T, _ptr(idx), _ptr(w), _stream_ptr(stream)))
        return idx, w

    def block_forward(self, layer: int, hidden, stream=None):
        self._check(self.lib.lm_moe_block_forward(self.ctx, layer, _ptr(hidden), hidden.shape[0],
                                                  _stream_ptr(stream)))
        return hidden

    def sync(self, stream=None) -> None:
        self._check(self.lib.lm_moe_sync(self.ctx, _stream_ptr(stream)))

    def debug_set(self, knob: int, value: int) -> None:
        """Testing hooks of the failure-detection path (lm_moe_debug_set)."""
        self._check(self.lib.lm_moe_debug_set(self.ctx, knob, value))

    def profile(self, enable: bool) -> None:
        self._check(self.lib.lm_moe_profile_enable(self.ctx, int(enable)))

    def profile_read(self, reset: bool = True) -> dict:
        ms = np.zeros(_lib.LM_PROFILE_SLOTS, np.float64)
        n = np.zeros(_lib.LM_PROFILE_SLOTS, np.int64)
        self._check(self.lib.lm_moe_profile_read(self.ctx, _ptr(ms), _ptr(n), int(reset)))
        return {name: (float(ms[i]), int(n[i])) for i, name in enumerate(_lib.PROFILE_SLOT_NAMES) if n[i] > 0}

    def profile_trace(self) -> np.ndarray:
        """Per-CTA phase stamps (ns) of the last profiled fused decode launch, [ctas, slots]."""
        cap = 1024
        out = np.zeros((cap, _lib.LM_DECODE_TRACE_SLOTS), np.uint64)
        n = C.c_int32(0)
        self._check(self.lib.lm_moe_profile_trace(self.ctx, _ptr(out), cap, C.byref(n)))
        return out[: min(n.value, cap)]

    def profile_ep_timeline(self) -> dict | None:
        """Step times (ms) of the last profiled chunked expert-parallel forward, or None."""
        cap = 40
        out = np.zeros(cap, np.float32)
        n = C.c_int32(0)
        self._check(self.lib.lm_moe_profile_ep_timeline(self.ctx, _ptr(out), cap, C.byref(n)))
        k = n.value
        if k == 0:
            return None
        v = [round(float(t), 4) for t in out[:4 * k + 2]]
        return {"dispatched": v[:k], "shared_done": v[k], "gemm_start": v[k + 1:2 * k + 1],
                "gemm_done": v[2 * k + 1:3 * k + 1], "returned": v[3 * k + 1:4 * k + 1], "combined": v[4 * k + 1]}

    def expert_counts(self) -> np.ndarray:
        out = np.zeros(self.config.n_routed_experts, np.int32)
        self._check(self.lib.lm_moe_expert_counts(self.ctx, _ptr(out), out.size))
        return out


class MoeRouter:
    """litemind::MoeRouter on the GPU (include/MoeRouter.hpp:27-55)."""

    def __init__(self, config: MoeConfig | None = None, device: int = 0):
        cfg = config or MoeConfig()
        # The router needs no expert weights: a one-layer context with no experts
        # resident is enough for lm_moe_select.
        self.config = MoeConfig(**{**cfg.__dict__, "max_tokens": max(cfg.max_tokens, 1), "num_layers": 1,
                                   "hidden_size": 128, "moe_intermediate_size": 64, "n_shared_experts": 0})
        self._layer = MoeLayer(self.config, device)

    def select(self, gate_logits) -> list[ExpertSelection]:
        logits = np.ascontiguousarray(gate_logits, np.float32).reshape(-1)
        if logits.size != self.config.n_routed_experts:
            return []  # src/MoeRouter.cpp:57-59
        t = torch.from_numpy(logits.reshape(1, -1)).cuda()
        idx, w = self._layer.select(t)
        torch.cuda.synchronize()
        return [ExpertSelection(int(i), float(v)) for i, v in zip(idx[0].tolist(), w[0].tolist())]

    def select_batch(self, logits):
        """[T, E] device logits -> ([T, k] int32, [T, k] f32) device tensors."""
        return self._layer.select(logits)

    @staticmethod
    def select_top_k(gate_logits, expert_count: int, top_k: int,
                     normalize_selected_weights: bool) -> list[ExpertSelection]:
        logits = np.ascontiguousarray(gate_logits, np.float32).reshape(-1)
        if expert_count == 0 or top_k == 0 or top_k > expert_count or logits.size != expert_count:
            raise ValueError("MoE routing requires one logit per expert and a valid top-k value.")
        cfg = MoeConfig(n_routed_experts=expert_count, num_experts_per_tok=top_k,
                        norm_topk_prob=normalize_selected_weights, routed_scaling_factor=1.0,
                        topk_method="greedy", n_group=1, topk_group=1, max_tokens=1)
        return MoeRouter(cfg).select(logits)
