"""ctypes signatures of the engine-level entry points (bound by _native.lib())."""
from __future__ import annotations

import ctypes as C

SIGNATURES: dict = {}


def bind(L: C.CDLL) -> None:
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args
