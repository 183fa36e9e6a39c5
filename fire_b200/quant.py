"""Fire's group-wise UInt4 weight layout: quantise, pack, unpack, dequantise.

The layout contract is Fire's ``tools/quant.py``: asymmetric round-to-nearest
(NumPy ties-to-even) with values in [0, 15], ``w ~= s * (q - z)``, groups along
the input dimension, an all-zero group encoded as q=0, s=1, z=0, and two values
per byte with the even column in the low nibble. AutoAWQ GEMM checkpoints pack
eight values per int32 in the order [0, 2, 4, 6, 1, 3, 5, 7]
(``tools/export_qwen3.py:800-850``); :func:`unpack_awq_gemm` undoes it.

These are data-preparation helpers (synthetic checkpoints, exporters); the
decode path itself only ever reads the packed bytes on the GPU.
"""
from __future__ import annotations

import numpy as np

GROUP_SIZE = 128


def quantize_int4_groupwise(weights: np.ndarray, group_size: int = GROUP_SIZE):
    """RTN INT4 of a FP32 [out, in] matrix -> (q u8 [out,in], scales f32 [out,in/g], zeros u8).

    Follows tools/quant.py:14-101: range widened to include 0, s = (max-min)/15
    (1 for an all-zero group), z = clip(rint(-min/s), 0, 15),
    q = clip(rint(w/s + z), 0, 15), all in FP32.
    """
    w = np.asarray(weights)
    if w.dtype != np.float32 or w.ndim != 2:
        raise TypeError("weights must be a 2-D float32 array")
    if group_size <= 0 or w.shape[1] % group_size:
        raise ValueError("group_size must be positive and divide in_features")
    if not np.all(np.isfinite(w)):
        raise ValueError("weights must contain only finite values")
    out_f, in_f = w.shape
    g = w.reshape(out_f, in_f // group_size, group_size)
    lo = np.minimum(g.min(axis=2), np.float32(0))
    hi = np.maximum(g.max(axis=2), np.float32(0))
    s = ((hi - lo) / np.float32(15)).astype(np.float32)
    empty = s == 0
    s[empty] = np.float32(1)
    z = np.clip(np.rint(-lo / s), 0, 15).astype(np.uint8)
    q = np.clip(np.rint(g / s[..., None] + z[..., None]), 0, 15).astype(np.uint8)
    if empty.any():
        q[empty] = 0
        z[empty] = 0
    return (np.ascontiguousarray(q.reshape(out_f, in_f)), np.ascontiguousarray(s),
            np.ascontiguousarray(z))


def pack_uint4(values: np.ndarray) -> np.ndarray:
    """[out, in] values in [0,15] -> [out, in/2] bytes, even column in the low nibble."""
    v = np.asarray(values)
    if v.dtype != np.uint8 or v.ndim != 2 or v.shape[1] % 2:
        raise ValueError("values must be 2-D uint8 with an even last dimension")
    if np.any(v > 15):
        raise ValueError("UInt4 values must be in [0, 15]")
    return np.ascontiguousarray(v[:, 0::2] | (v[:, 1::2] << 4))


def unpack_uint4(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, np.uint8)
    out = np.empty((p.shape[0], p.shape[1] * 2), np.uint8)
    out[:, 0::2] = p & 0x0F
    out[:, 1::2] = p >> 4
    return out


def dequantize_int4_groupwise(packed, scales, zeros, group_size: int = GROUP_SIZE):
    """w[o, k] = s[o, k//g] * (q[o, k] - z[o, k//g]) in FP32 (tools/quant.py:141-261)."""
    q = unpack_uint4(packed).astype(np.float32)
    s = np.asarray(scales, np.float32)
    z = np.asarray(zeros, np.uint8).astype(np.float32)
    o, k = q.shape
    qg = q.reshape(o, k // group_size, group_size)
    return np.ascontiguousarray((s[..., None] * (qg - z[..., None])).reshape(o, k),
                                dtype=np.float32)


AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
_AWQ_INVERSE = tuple(AWQ_ORDER.index(i) for i in range(8))


def unpack_awq_gemm(words: np.ndarray) -> np.ndarray:
    """AutoAWQ GEMM int32 [in, out/8] -> UInt4 values [out, in] (export_qwen3.py:800-807)."""
    w = np.ascontiguousarray(words).view(np.uint32)
    shifts = np.arange(0, 32, 4, dtype=np.uint32)
    vals = ((w[:, :, None] >> shifts) & 15).astype(np.uint8)      # [in, out/8, slot]
    vals = vals[:, :, list(_AWQ_INVERSE)]                         # slot -> output channel
    return np.ascontiguousarray(vals.reshape(w.shape[0], -1).T)


def quantize_torch(weights, group_size: int = GROUP_SIZE):
    """The same RTN rule on a torch FP32 tensor (any device); used to make large
    synthetic checkpoints directly on the GPU. Returns (packed u8, scales f32, zeros u8)."""
    import torch

    out_f, in_f = weights.shape
    g = weights.reshape(out_f, in_f // group_size, group_size)
    zero = torch.zeros((), dtype=torch.float32, device=weights.device)
    lo = torch.minimum(g.amin(dim=2), zero)
    hi = torch.maximum(g.amax(dim=2), zero)
    s = (hi - lo) / 15.0
    empty = s == 0
    s = torch.where(empty, torch.ones_like(s), s)
    z = torch.clamp(torch.round(-lo / s), 0, 15)
    q = torch.clamp(torch.round(g / s[..., None] + z[..., None]), 0, 15)
    q = torch.where(empty[..., None], torch.zeros_like(q), q).to(torch.uint8)
    z = torch.where(empty, torch.zeros_like(z), z).to(torch.uint8)
    q = q.reshape(out_f, in_f)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()
    return packed, s.contiguous(), z.contiguous()
