"""Python face of the C++ Qwen3 decode engine (include/fire_b200_qwen3.h).

Mirrors Fire's ``Model`` contract (include/Fire/model/model.h:22-52): ``prepare``,
``forward(token_id, pos, logits)``, ``reset``, plus the greedy loops. Weights come
from a ``.fire`` file (``Qwen3Engine.open``) or from named arrays / CUDA tensors
(``Qwen3Engine(profile, tensors)``), e.g. a synthetic checkpoint from
``fire_b200.synth``.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, Optional, Sequence

import numpy as np

from . import _engine_sigs as E
from . import _native as N
from .profiles import Qwen3Profile


def _profile(p: Qwen3Profile) -> E.Profile:
    return E.Profile(p.vocab_size, p.max_seq_len, p.hidden_size, p.intermediate_size, p.num_layers,
                     p.num_attention_heads, p.num_kv_heads, p.head_dim, p.rms_norm_eps, p.rope_theta)


def _options(tp_rank, tp_size, nccl_id, use_graph, pdl, deadline_ms, keep) -> E.Options:
    idp = None
    if nccl_id is not None:
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        keep.append(buf)
        idp = C.cast(buf, C.c_void_p)
    return E.Options(tp_rank, tp_size, idp, 1 if use_graph else 0, 1 if pdl else 0, int(deadline_ms))


def _descriptor(name: str, a, keep) -> E.Tensor:
    try:
        import torch
    except ImportError:  # pragma: no cover
        torch = None
    if torch is not None and isinstance(a, torch.Tensor):
        a = a.contiguous()
        keep.append(a)
        dt = {torch.float32: N.F32, torch.bfloat16: N.BF16, torch.int16: N.BF16, torch.uint8: 2}[a.dtype]
        shape = tuple(a.shape)
        ptr, dev = a.data_ptr(), 1 if a.is_cuda else 0
    else:
        a = np.ascontiguousarray(a)
        keep.append(a)
        dt = {np.dtype(np.float32): N.F32, np.dtype(np.uint16): N.BF16, np.dtype(np.uint8): 2}[a.dtype]
        shape = a.shape
        ptr, dev = a.ctypes.data, 0
    nm = name.encode("ascii")
    keep.append(nm)
    s = (C.c_int64 * 2)(shape[0], shape[1] if len(shape) == 2 else 0)
    return E.Tensor(nm, dt, len(shape), s, ptr, dev)


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    N.check(N.lib().fire_b200_nccl_unique_id(C.cast(buf, C.c_void_p)), "nccl unique id")
    return buf.raw


class Qwen3Engine:
    def __init__(self, profile: Qwen3Profile, tensors: Optional[Dict[str, object]] = None, *, path: str = None,
                 tp_rank: int = 0, tp_size: int = 1, nccl_id: Optional[bytes] = None, use_graph: bool = True,
                 pdl: bool = True, deadline_ms: int = 0):
        L = N.lib()
        self.profile = profile
        self.tp_rank, self.tp_size = tp_rank, tp_size
        keep: list = []
        prof = _profile(profile)
        opts = _options(tp_rank, tp_size, nccl_id, use_graph, pdl, deadline_ms, keep)
        h = C.c_void_p()
        if path is not None:
            rc = L.fire_b200_qwen3_open(path.encode(), C.byref(prof), C.byref(opts), C.byref(h))
        else:
            descs = [_descriptor(n, a, keep) for n, a in tensors.items()]
            if any(d.on_device for d in descs):
                import torch

                torch.cuda.synchronize()  # the engine copies on its own stream
            arr = (E.Tensor * len(descs))(*descs)
            rc = L.fire_b200_qwen3_create(C.byref(prof), arr, len(descs), C.byref(opts), C.byref(h))
        if rc != N.OK:
            raise N.FireB200Error(rc, "qwen3 create: " + L.fire_b200_qwen3_last_error().decode())
        self._h = h
        self._L = L

    @classmethod
    def open(cls, path: str, profile: Qwen3Profile, **kw) -> "Qwen3Engine":
        return cls(profile, path=path, **kw)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.fire_b200_qwen3_destroy(self._h)
            self._h = None

    __del__ = close

    def prepare(self, capacity: int) -> None:
        N.check(self._L.fire_b200_qwen3_prepare(self._h, capacity), "prepare")

    def forward(self, token: int, pos: int, logits=None, stream=None) -> None:
        """Model::forward; `logits` (CUDA float32 [vocab]) receives a copy when given."""
        ptr = None if logits is None else logits.data_ptr()
        N.check(self._L.fire_b200_qwen3_forward(self._h, int(token), int(pos), ptr, N.stream_handle(stream)),
                "forward")

    def generate(self, first_token: int, steps: int, out=None, stream=None):
        """Device-side greedy loop; returns a CUDA int32 tensor [steps] (asynchronous)."""
        import torch

        if out is None:
            out = torch.empty(steps, dtype=torch.int32, device="cuda")
        N.check(self._L.fire_b200_qwen3_generate(self._h, int(first_token), int(steps), out.data_ptr(),
                                                 N.stream_handle(stream)), "generate")
        return out

    def generate_host(self, prompt: Sequence[int], steps: int, stream=None) -> np.ndarray:
        """The reference's host loop: per token H2D + step + D2H + synchronise."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(steps, np.int32)
        N.check(self._L.fire_b200_qwen3_generate_host(self._h, p.ctypes.data, p.size, int(steps), out.ctypes.data,
                                                      N.stream_handle(stream)), "generate_host")
        return out

    def reset(self) -> None:
        N.check(self._L.fire_b200_qwen3_reset(self._h), "reset")

    def truncate(self, length: int) -> None:
        N.check(self._L.fire_b200_qwen3_truncate(self._h, int(length)), "truncate")

    def status(self) -> int:
        """Waits for the enqueued steps; returns the device error code (0 = ok) or raises
        FireB200Error(ERR_TIMEOUT) when the tensor-parallel deadline ran out."""
        code = C.c_int(0)
        rc = self._L.fire_b200_qwen3_status(self._h, C.byref(code))
        if rc not in (N.OK, N.ERR_DEVICE):
            raise N.FireB200Error(rc, "status")
        return int(code.value)

    def abort(self) -> None:
        """Leave the tensor-parallel group (ncclCommAbort); the engine is then only fit for close()."""
        N.check(self._L.fire_b200_qwen3_abort(self._h), "abort")

    def kv_export(self, length: int):
        """(key, value) numpy FP32 [layers, length, kv_heads_local, 128] of positions < length."""
        p = self.profile
        shape = (p.num_layers, int(length), p.num_kv_heads // self.tp_size, p.head_dim)
        k, v = np.empty(shape, np.float32), np.empty(shape, np.float32)
        N.check(self._L.fire_b200_qwen3_kv_export(self._h, int(length), k.ctypes.data, v.ctypes.data, None),
                "kv_export")
        return k, v

    def kv_import(self, key, value) -> None:
        """Load a KV prefix ([layers, length, kv_heads_local, 128] FP32) as the current sequence."""
        k = np.ascontiguousarray(key, np.float32)
        v = np.ascontiguousarray(value, np.float32)
        p = self.profile
        want = (p.num_layers, k.shape[1], p.num_kv_heads // self.tp_size, p.head_dim)
        if k.shape != want or v.shape != want:
            raise ValueError(f"KV prefix must be {want}")
        N.check(self._L.fire_b200_qwen3_kv_import(self._h, int(k.shape[1]), k.ctypes.data, v.ctypes.data, None),
                "kv_import")

    @property
    def length(self) -> int:
        return self._L.fire_b200_qwen3_length(self._h)

    def logits_ptr(self) -> int:
        return self._L.fire_b200_qwen3_logits(self._h)

    @property
    def kernels_per_step(self) -> int:
        return self._L.fire_b200_qwen3_kernels_per_step(self._h)

    def prefill(self, tokens: Sequence[int], logits=None, stream=None) -> None:
        """Consume the prompt tokens at positions length.. in one batched pass (see
        fire_b200_qwen3_prefill); logits of the last token into `logits` if given."""
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        ptr = logits.data_ptr() if logits is not None else None
        N.check(self._L.fire_b200_qwen3_prefill(self._h, ids.ctypes.data, len(ids), ptr, N.stream_handle(stream)),
                "prefill")

    def time_layer_stack(self, reps: int = 5, stream=None) -> float:
        """Average device milliseconds of one launch of the layer-stack kernel alone."""
        ms = C.c_float(0.0)
        N.check(self._L.fire_b200_qwen3_time_layer_stack(self._h, int(reps), C.byref(ms), N.stream_handle(stream)),
                "time_layer_stack")
        return float(ms.value)

    def stack_trace(self) -> np.ndarray:
        """Per-phase timeline of the last layer-stack launch, [CTAs, layers, 5, 13] values
        (empty unless FIRE_B200_STACK_TRACE=1 was set when the engine was created)."""
        n = int(self._L.fire_b200_qwen3_stack_trace(self._h, None, 0))
        if n <= 0:
            return np.zeros((0,), np.uint64)
        out = np.zeros(n, np.uint64)
        got = int(self._L.fire_b200_qwen3_stack_trace(self._h, out.ctypes.data, n))
        if got < 0:
            raise N.FireB200Error(got, "stack trace read failed")
        return out.reshape(-1, self.profile.num_layers, 5, 13)

    @property
    def step_weight_bytes(self) -> int:
        return int(self._L.fire_b200_qwen3_step_weight_bytes(self._h))
