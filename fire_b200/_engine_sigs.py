"""ctypes signatures of the engine-level entry points (include/fire_b200_qwen3.h)."""
from __future__ import annotations

import ctypes as C


class Profile(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("max_seq_len", C.c_int), ("hidden_size", C.c_int),
                ("intermediate_size", C.c_int), ("num_layers", C.c_int), ("num_attention_heads", C.c_int),
                ("num_kv_heads", C.c_int), ("head_dim", C.c_int), ("rms_norm_eps", C.c_float),
                ("rope_theta", C.c_float)]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("ndim", C.c_int), ("shape", C.c_int64 * 2),
                ("data", C.c_void_p), ("on_device", C.c_int)]


class Options(C.Structure):
    _fields_ = [("tp_rank", C.c_int), ("tp_size", C.c_int), ("nccl_id", C.c_void_p), ("use_graph", C.c_int),
                ("pdl", C.c_int), ("deadline_ms", C.c_int)]


_vp, _i = C.c_void_p, C.c_int
SIGNATURES: dict = {
    "fire_b200_nccl_unique_id": (_i, [_vp]),
    "fire_b200_qwen3_create": (_i, [C.POINTER(Profile), C.POINTER(Tensor), _i, C.POINTER(Options), C.POINTER(_vp)]),
    "fire_b200_qwen3_open": (_i, [C.c_char_p, C.POINTER(Profile), C.POINTER(Options), C.POINTER(_vp)]),
    "fire_b200_qwen3_last_error": (C.c_char_p, []),
    "fire_b200_qwen3_prepare": (_i, [_vp, _i]),
    "fire_b200_qwen3_forward": (_i, [_vp, _i, _i, _vp, _vp]),
    "fire_b200_qwen3_generate": (_i, [_vp, _i, _i, _vp, _vp]),
    "fire_b200_qwen3_generate_host": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "fire_b200_qwen3_reset": (_i, [_vp]),
    "fire_b200_qwen3_status": (_i, [_vp, C.POINTER(C.c_int)]),
    "fire_b200_qwen3_abort": (_i, [_vp]),
    "fire_b200_qwen3_kv_export": (_i, [_vp, _i, _vp, _vp, _vp]),
    "fire_b200_qwen3_kv_import": (_i, [_vp, _i, _vp, _vp, _vp]),
    "fire_b200_qwen3_truncate": (_i, [_vp, _i]),
    "fire_b200_qwen3_length": (_i, [_vp]),
    "fire_b200_qwen3_logits": (_vp, [_vp]),
    "fire_b200_qwen3_kernels_per_step": (_i, [_vp]),
    "fire_b200_qwen3_stack_trace": (C.c_int64, [_vp, _vp, C.c_int64]),
    "fire_b200_qwen3_time_layer_stack": (_i, [_vp, _i, C.POINTER(C.c_float), _vp]),
    "fire_b200_qwen3_prefill": (_i, [_vp, _vp, _i, _vp, _vp]),
    "fire_b200_qwen3_step_weight_bytes": (C.c_uint64, [_vp]),
    "fire_b200_qwen3_destroy": (None, [_vp]),
}


def bind(L: C.CDLL) -> None:
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args
