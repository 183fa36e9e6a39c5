"""ctypes binding of ``fire_b200/libfire_b200.so`` (the C ABI in ``include/fire_b200.h``).

The library is the product: there is no CPU or pure-PyTorch fallback. If the
library is missing, or a call runs without a CUDA device, the call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from typing import Dict, List

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "libfire_b200.so")
HEADER = os.path.join(ROOT, "include", "fire_b200.h")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_NO_DEVICE, ERR_STATE, ERR_IO, ERR_NOMEM = 0, -1, -2, -3, -4, -5, -6
ERR_DEVICE, ERR_TIMEOUT = -7, -8
F32, BF16 = 0, 1


class FireB200Error(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status})" if what else status_string(status))


_lib = None

_vp, _i, _f, _i64, _sz = C.c_void_p, C.c_int, C.c_float, C.c_int64, C.c_size_t

# name -> (restype, argtypes)
SIGNATURES: Dict[str, tuple] = {
    "fire_b200_abi_version": (_i, []),
    "fire_b200_status_string": (C.c_char_p, [_i]),
    "fire_b200_linear_w4": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "fire_b200_linear_w4_prefill_workspace_bytes": (C.c_size_t, [_i, _i, _i]),
    "fire_b200_linear_w4_prefill": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, C.c_size_t, _vp, _vp]),
    "fire_b200_linear_dense": (_i, [_vp, _vp, _i, _f, _vp, _i, _i, _i, _vp]),
    "fire_b200_rmsnorm": (_i, [_vp, _vp, _vp, _i, _f, _vp]),
    "fire_b200_rmsnorm_rows": (_i, [_vp, _vp, _vp, _i, _i, _f, _vp]),
    "fire_b200_rope_cache": (_i, [_i, _i, _f, _vp, _vp, _vp]),
    "fire_b200_rope": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "fire_b200_mha_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "fire_b200_mha_decode": (_i, [_vp, _vp, _vp, _vp, _vp] + [_i] * 7 + [_vp, _sz, _vp]),
    "fire_b200_embedding": (_i, [_vp, _i, _vp, _i, _i, _i, _vp, _vp]),
    "fire_b200_swiglu": (_i, [_vp, _vp, _vp, _i, _vp]),
    "fire_b200_add": (_i, [_vp, _vp, _vp, _i, _vp]),
    "fire_b200_argmax_workspace_bytes": (_sz, []),
    "fire_b200_argmax": (_i, [_vp, _i64, _vp, _vp, _sz, _vp]),
    # include/fire_b200_alloc.h
    "fire_b200_device_alloc": (_i, [_sz, C.POINTER(_vp)]),
    "fire_b200_device_release": (_i, [_vp]),
    "fire_b200_device_memset_zero": (_i, [_vp, _sz, _vp, _i]),
    "fire_b200_device_memcpy": (_i, [_vp, _vp, _sz, _i, _vp, _i]),
    "fire_b200_device_pool_stats": (_i, [_i, C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_sz)]),
    "fire_b200_device_pool_trim": (_i, [_i]),
}
CPU2GPU, CPU2CPU, GPU2CPU, GPU2GPU = 0, 1, 2, 3


def declared_symbols() -> List[str]:
    """Every function name declared in include/*.h (the exported C ABI)."""
    names: List[str] = []
    inc = os.path.join(ROOT, "include")
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            text = open(os.path.join(inc, fn)).read()
            names += re.findall(r"\b(fire_b200_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FireB200Error(ERR_UNSUPPORTED, f"{LIB_PATH} is not built (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        from . import _engine_sigs  # engine entry points (same library)

        _engine_sigs.bind(L)
        _lib = L
    return _lib


def status_string(status: int) -> str:
    try:
        return lib().fire_b200_status_string(int(status)).decode()
    except Exception:  # noqa: BLE001 - library itself missing
        return f"status {status}"


def check(status: int, what: str) -> None:
    if status != OK:
        raise FireB200Error(status, what)


def stream_handle(stream) -> int:
    """cudaStream_t of a torch.cuda.Stream (or None -> torch's current stream)."""
    import torch

    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream
