"""TEST INFRASTRUCTURE ONLY - numpy/ctypes front end of the parity oracle.

Loads ``oracle/libfire_oracle.so`` (the C restatement of Fire's CPU decode path,
``oracle/fire_oracle.c``) and, when built, ``oracle/_ref/libfire_ref.so`` (the
reference's own kernels compiled from its sources by ``oracle/Makefile``). Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import
this module; the fire_b200 product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfire_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libfire_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64

_lib: Optional[C.CDLL] = None


def build() -> None:
    """Compile the C restatement (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.fo_set_threads.argtypes = [C.c_int]
        L.fo_get_threads.restype = C.c_int
        L.fo_dequant_int4.argtypes = [_u8p, _f32p, _u8p, _f32p, _i64, _i64, C.c_int]
        L.fo_linear_f32.argtypes = [_f32p, _f32p, C.c_float, _f32p, _i64, _i64, _i64]
        L.fo_linear_bf16.argtypes = [_f32p, _u16p, C.c_float, _f32p, _i64, _i64, _i64]
        L.fo_linear_int4.argtypes = [_f32p, _u8p, _f32p, _u8p, _f32p, _i64, _i64, _i64, C.c_int]
        L.fo_linear_int4_f64.argtypes = [_f32p, _u8p, _f32p, _u8p, _f64p, _i64, _i64, _i64,
                                         C.c_int]
        L.fo_rmsnorm.argtypes = [_f32p, _f32p, _f32p, _i64, C.c_float]
        L.fo_rmsnorm_rows.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, C.c_float]
        L.fo_rope_cache.argtypes = [C.c_int, C.c_int, C.c_float, _f32p, _f32p]
        L.fo_rope.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.fo_softmax.argtypes = [_f32p, _i64]
        L.fo_mha.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p] + [C.c_int] * 6
        L.fo_swiglu.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.fo_add.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.fo_embedding.argtypes = [_i32p, _i64, C.c_void_p, C.c_int, _i64, _f32p]
        L.fo_argmax.argtypes = [_f32p, _i64]
        L.fo_argmax.restype = _i64
        L.fo_qwen3_scratch_floats.argtypes = [C.c_void_p, C.c_int]
        L.fo_qwen3_scratch_floats.restype = _i64
        L.fo_qwen3_prepare.argtypes = [C.c_void_p, C.c_void_p]
        L.fo_qwen3_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, _f32p]
        L.fo_qwen3_forward.restype = C.c_int
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().fo_set_threads(int(n))


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------ kernels ----

def dequant_int4(qw, scales, zeros, group: int) -> np.ndarray:
    qw, scales, zeros = _c(qw, np.uint8), _c(scales, np.float32), _c(zeros, np.uint8)
    n, k = qw.shape[0], qw.shape[1] * 2
    w = np.empty((n, k), np.float32)
    lib().fo_dequant_int4(qw, scales, zeros, w, n, k, group)
    return w


def linear_int4(x, qw, scales, zeros, group: int = 128) -> np.ndarray:
    """Dequantise-then-FP32 Linear (tools/quant.py:249-255 + cpu/matmul_kernel.cpp:95-106)."""
    x = _c(x, np.float32)
    qw, scales, zeros = _c(qw, np.uint8), _c(scales, np.float32), _c(zeros, np.uint8)
    rows = 1 if x.ndim == 1 else x.shape[0]
    n, k = qw.shape[0], qw.shape[1] * 2
    y = np.empty((rows, n), np.float32)
    lib().fo_linear_int4(x, qw, scales, zeros, y, rows, n, k, group)
    return y[0] if x.ndim == 1 else y


def linear_int4_f64(x, qw, scales, zeros, group: int = 128) -> np.ndarray:
    x = _c(x, np.float32)
    qw, scales, zeros = _c(qw, np.uint8), _c(scales, np.float32), _c(zeros, np.uint8)
    rows = 1 if x.ndim == 1 else x.shape[0]
    n, k = qw.shape[0], qw.shape[1] * 2
    y = np.empty((rows, n), np.float64)
    lib().fo_linear_int4_f64(x, qw, scales, zeros, y, rows, n, k, group)
    return y[0] if x.ndim == 1 else y


def linear_f32(x, w, scale: float = 1.0) -> np.ndarray:
    x, w = _c(x, np.float32), _c(w, np.float32)
    rows = 1 if x.ndim == 1 else x.shape[0]
    y = np.empty((rows, w.shape[0]), np.float32)
    lib().fo_linear_f32(x, w, scale, y, rows, w.shape[0], w.shape[1])
    return y[0] if x.ndim == 1 else y


def linear_bf16(x, w_bits, scale: float = 1.0) -> np.ndarray:
    x, w = _c(x, np.float32), _c(w_bits, np.uint16)
    rows = 1 if x.ndim == 1 else x.shape[0]
    y = np.empty((rows, w.shape[0]), np.float32)
    lib().fo_linear_bf16(x, w, scale, y, rows, w.shape[0], w.shape[1])
    return y[0] if x.ndim == 1 else y


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x, w = _c(x, np.float32), _c(w, np.float32)
    y = np.empty_like(x)
    lib().fo_rmsnorm(x.reshape(-1), w.reshape(-1), y.reshape(-1), x.size, eps)
    return y


def rmsnorm_rows(x, w, eps: float) -> np.ndarray:
    x, w = _c(x, np.float32), _c(w, np.float32)
    width = x.shape[-1]
    y = np.empty_like(x)
    lib().fo_rmsnorm_rows(x.reshape(-1), w, y.reshape(-1), x.size // width, width, eps)
    return y


def rope_cache(head: int, max_seq: int, theta: float):
    s = np.empty((max_seq, head // 2), np.float32)
    c = np.empty((max_seq, head // 2), np.float32)
    lib().fo_rope_cache(head, max_seq, theta, s, c)
    return s, c


def rope(q, k, cos, sin, pos: int):
    q, k = _c(q, np.float32).copy(), _c(k, np.float32).copy()
    lib().fo_rope(q.reshape(-1), k.reshape(-1), _c(cos, np.float32).reshape(-1),
                  _c(sin, np.float32).reshape(-1), q.shape[0], k.shape[0], q.shape[1], pos)
    return q, k


def softmax(x) -> np.ndarray:
    x = _c(x, np.float32).copy()
    lib().fo_softmax(x, x.size)
    return x


def mha(q, key_cache, value_cache, layer: int, pos: int, score=None):
    q, kc, vc = _c(q, np.float32), _c(key_cache, np.float32), _c(value_cache, np.float32)
    layers, cap, kvh, hd = kc.shape
    qh = q.shape[0]
    score = np.full((qh, cap), -777.0, np.float32) if score is None else _c(score, np.float32)
    out = np.empty((qh, hd), np.float32)
    lib().fo_mha(q.reshape(-1), kc.reshape(-1), vc.reshape(-1), score.reshape(-1),
                 out.reshape(-1), qh, kvh, hd, cap, layer, pos)
    return out, score


def swiglu(g, u) -> np.ndarray:
    g, u = _c(g, np.float32), _c(u, np.float32)
    o = np.empty_like(g)
    lib().fo_swiglu(g.reshape(-1), u.reshape(-1), o.reshape(-1), g.size)
    return o


def add(a, b) -> np.ndarray:
    a, b = _c(a, np.float32), _c(b, np.float32)
    o = np.empty_like(a)
    lib().fo_add(a.reshape(-1), b.reshape(-1), o.reshape(-1), a.size)
    return o


def embedding(tokens, table) -> np.ndarray:
    tokens = _c(tokens, np.int32).reshape(-1)
    table = np.ascontiguousarray(table)
    dtype = 1 if table.dtype == np.uint16 else 0
    if dtype == 0:
        table = _c(table, np.float32)
    out = np.empty((tokens.size, table.shape[1]), np.float32)
    lib().fo_embedding(tokens, tokens.size, table.ctypes.data, dtype, table.shape[1], out)
    return out


def argmax(x) -> int:
    x = _c(x, np.float32).reshape(-1)
    return int(lib().fo_argmax(x, x.size))


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


# -------------------------------------------------------------------- model ----

class _Linear(C.Structure):
    _fields_ = [("kind", C.c_int), ("n", C.c_int64), ("k", C.c_int64), ("group", C.c_int),
                ("w", C.c_void_p), ("scales", C.c_void_p), ("zeros", C.c_void_p)]


class _Layer(C.Structure):
    _fields_ = [("attention_norm", C.c_void_p), ("wq", _Linear), ("wk", _Linear),
                ("wv", _Linear), ("wo", _Linear), ("q_norm", C.c_void_p),
                ("k_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("w1", _Linear),
                ("w2", _Linear), ("w3", _Linear)]


class _Model(C.Structure):
    _fields_ = [("hidden", C.c_int), ("intermediate", C.c_int), ("layers", C.c_int),
                ("q_heads", C.c_int), ("kv_heads", C.c_int), ("head_dim", C.c_int),
                ("vocab", C.c_int64), ("eps", C.c_float), ("theta", C.c_float),
                ("emb_dtype", C.c_int), ("embedding", C.c_void_p), ("layer", C.c_void_p),
                ("final_norm", C.c_void_p), ("output", _Linear)]


class _State(C.Structure):
    _fields_ = [("capacity", C.c_int), ("max_seq", C.c_int), ("key_cache", C.c_void_p),
                ("value_cache", C.c_void_p), ("rope_sin", C.c_void_p), ("rope_cos", C.c_void_p),
                ("scratch", C.c_void_p)]


def _ptr(a: Optional[np.ndarray]) -> Optional[int]:
    return None if a is None else a.ctypes.data


class Qwen3Oracle:
    """CPU restatement of Qwen3Model (src/model/qwen.cpp:155-303) over numpy weights.

    ``weights`` is a mapping from Fire tensor names (``tools/export_qwen3.py:268-365``
    naming: ``layers.{i}.attention.wq.qweight`` ...) to numpy arrays, as produced by
    ``fire_b200.synth`` or read from a ``.fire`` file. INT4 projections are a
    qweight/scales/zero_points triplet; plain projections are FP32 or BF16 (uint16 bits).
    """

    def __init__(self, profile, weights, capacity: int, max_seq: Optional[int] = None):
        self.p = profile
        self.keep = []  # keeps every array referenced by the C structs alive
        L = lib()

        def arr(name, dtype):
            a = np.ascontiguousarray(weights[name], dtype=dtype)
            self.keep.append(a)
            return a

        def linear(base: str, n: int, k: int) -> _Linear:
            if base + ".qweight" in weights:
                q = arr(base + ".qweight", np.uint8)
                s = arr(base + ".scales", np.float32)
                z = arr(base + ".zero_points", np.uint8)
                return _Linear(2, n, k, k // s.shape[1], _ptr(q), _ptr(s), _ptr(z))
            w = weights[base + ".weight"]
            if w.dtype == np.uint16:
                w = arr(base + ".weight", np.uint16)
                return _Linear(1, n, k, 0, _ptr(w), None, None)
            w = arr(base + ".weight", np.float32)
            return _Linear(0, n, k, 0, _ptr(w), None, None)

        p = profile
        H, Fd, Q, KV = p.hidden_size, p.intermediate_size, p.q_dim, p.kv_dim
        layers = (_Layer * p.num_layers)()
        for i in range(p.num_layers):
            pre = f"layers.{i}"
            layers[i].attention_norm = _ptr(arr(pre + ".attention_norm.weight", np.float32))
            layers[i].wq = linear(pre + ".attention.wq", Q, H)
            layers[i].wk = linear(pre + ".attention.wk", KV, H)
            layers[i].wv = linear(pre + ".attention.wv", KV, H)
            layers[i].wo = linear(pre + ".attention.wo", H, Q)
            layers[i].q_norm = _ptr(arr(pre + ".attention.q_norm.weight", np.float32))
            layers[i].k_norm = _ptr(arr(pre + ".attention.k_norm.weight", np.float32))
            layers[i].ffn_norm = _ptr(arr(pre + ".ffn_norm.weight", np.float32))
            layers[i].w1 = linear(pre + ".feed_forward.w1", Fd, H)
            layers[i].w2 = linear(pre + ".feed_forward.w2", H, Fd)
            layers[i].w3 = linear(pre + ".feed_forward.w3", Fd, H)
        self.keep.append(layers)
        emb = weights["tok_embeddings.weight"]
        emb_dtype = 1 if emb.dtype == np.uint16 else 0
        emb = arr("tok_embeddings.weight", np.uint16 if emb_dtype else np.float32)
        m = _Model(H, Fd, p.num_layers, p.num_attention_heads, p.num_kv_heads, p.head_dim,
                   p.vocab_size, p.rms_norm_eps, p.rope_theta, emb_dtype, _ptr(emb),
                   C.cast(layers, C.c_void_p), _ptr(arr("norm.weight", np.float32)),
                   linear("output", p.vocab_size, H))
        self.model = m
        max_seq = max_seq or capacity
        self.capacity = capacity
        self.kc = np.zeros((p.num_layers, capacity, p.num_kv_heads, p.head_dim), np.float32)
        self.vc = np.zeros_like(self.kc)
        self.sin = np.empty((max_seq, p.head_dim // 2), np.float32)
        self.cos = np.empty_like(self.sin)
        self.scratch = np.empty(L.fo_qwen3_scratch_floats(C.byref(m), capacity), np.float32)
        self.state = _State(capacity, max_seq, _ptr(self.kc), _ptr(self.vc), _ptr(self.sin),
                            _ptr(self.cos), _ptr(self.scratch))
        L.fo_qwen3_prepare(C.byref(self.model), C.byref(self.state))
        self.length = 0

    def forward(self, token: int, pos: int) -> np.ndarray:
        if pos != self.length:
            raise ValueError("position does not match the current sequence length")
        logits = np.empty(self.p.vocab_size, np.float32)
        rc = lib().fo_qwen3_forward(C.byref(self.model), C.byref(self.state), int(token),
                                    int(pos), logits)
        if rc != 0:
            raise ValueError(f"oracle forward rejected token/pos ({rc})")
        self.length += 1
        return logits

    def reset(self) -> None:
        self.length = 0


# ------------------------------------------------------- reference library ----

_ref: Optional[C.CDLL] = None


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref() -> C.CDLL:
    """The reference's own kernels, built from its sources (oracle/Makefile ``ref``)."""
    global _ref
    if _ref is None:
        R = C.CDLL(REF_PATH)
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        R.ref_matmul_quant_cu.argtypes = [vp] * 5 + [i] * 4 + [vp]
        R.ref_matmul_cu.argtypes = [vp, vp, i, f, vp, i, i, i, vp]
        R.ref_rmsnorm_cu.argtypes = [vp, vp, vp, i, i, i, f, vp]
        R.ref_rope_cache_cu.argtypes = [i, i, f, vp, vp, vp]
        R.ref_rope_cu.argtypes = [vp, vp, vp, vp, i, i, i, i, i, vp]
        R.ref_mha_cu.argtypes = [vp] * 5 + [i] * 7 + [vp]
        R.ref_embedding_cu.argtypes = [vp, i, vp, i, i, i, vp, vp]
        R.ref_swiglu_cu.argtypes = [vp, vp, vp, i, vp]
        R.ref_add_cu.argtypes = [vp, vp, vp, i, vp]
        R.ref_argmax_cu.argtypes = [vp, C.c_int64, vp]
        R.ref_argmax_cu.restype = C.c_int64
        R.ref_rmsnorm_cpu.argtypes = [_f32p, _f32p, _f32p, i, i, i, f]
        R.ref_rope_cache_cpu.argtypes = [i, i, f, _f32p, _f32p]
        R.ref_rope_cpu.argtypes = [_f32p, _f32p, _f32p, _f32p, i, i, i, i, i]
        R.ref_mha_cpu.argtypes = [_f32p] * 5 + [i] * 7
        R.ref_softmax_cpu.argtypes = [_f32p, i]
        _ref = R
    return _ref
