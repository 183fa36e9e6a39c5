"""fire_b200: Fire's single-token Qwen3 INT4 decode path, rebuilt for NVIDIA B200 (sm_100a).

The compute lives in ``libfire_b200.so`` (hand-written CUDA kernels behind the C ABI
in ``include/fire_b200.h``); this package is the host-side mirror of Fire's operator
and model interface plus data tools (``.fire`` format, RTN INT4, synthetic checkpoints).
"""
from .profiles import QWEN3_0_6B, QWEN3_8B, TINY, Qwen3Profile  # noqa: F401

__all__ = ["Qwen3Profile", "QWEN3_0_6B", "QWEN3_8B", "TINY"]
