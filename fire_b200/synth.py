"""Seeded synthetic Qwen3 checkpoints in Fire's tensor naming and layouts.

There is no real checkpoint here; every weight is drawn from a seeded normal
distribution and quantised with the reference RTN rule, which is how the
workloads this project is measured on are defined:

* tensor names and order follow Fire's exporter descriptor
  (``tools/export_qwen3.py:268-365``): embedding, then per layer attention_norm,
  wq, wk, wv, wo, q_norm, k_norm, ffn_norm, w1 (gate), w2 (down), w3 (up), then
  norm and output;
* layout ``"int4"`` is the RTN export (``_build_int4_entries``, :638-693): every
  linear, the LM head included, becomes a qweight/scales/zero_points triplet and the
  embedding stays FP32;
* layout ``"mixed"`` is the AWQ import (``_build_awq_patterns``, :368-395): the seven
  projections are INT4 triplets, embedding and LM head are BF16, norms FP32. Scales
  are rounded to FP16 values (stored FP32), as AWQ checkpoints carry them.

Linear weights ~ N(0, 0.02) before quantisation; norm weights are 1.0.
"""
from __future__ import annotations

from typing import Dict, Iterator, List, Tuple

import numpy as np

from .profiles import Qwen3Profile
from .quant import GROUP_SIZE, pack_uint4, quantize_int4_groupwise

PROJECTIONS = ("attention.wq", "attention.wk", "attention.wv", "attention.wo",
               "feed_forward.w1", "feed_forward.w2", "feed_forward.w3")


def descriptor(p: Qwen3Profile) -> List[Tuple[str, Tuple[int, ...]]]:
    """(fire base name, logical shape) in exporter order."""
    H, F, Q, KV, D = p.hidden_size, p.intermediate_size, p.q_dim, p.kv_dim, p.head_dim
    out = [("tok_embeddings.weight", (p.vocab_size, H))]
    for i in range(p.num_layers):
        pre = f"layers.{i}."
        out += [(pre + "attention_norm.weight", (H,)), (pre + "attention.wq.weight", (Q, H)),
                (pre + "attention.wk.weight", (KV, H)), (pre + "attention.wv.weight", (KV, H)),
                (pre + "attention.wo.weight", (H, Q)), (pre + "attention.q_norm.weight", (D,)),
                (pre + "attention.k_norm.weight", (D,)), (pre + "ffn_norm.weight", (H,)),
                (pre + "feed_forward.w1.weight", (F, H)), (pre + "feed_forward.w2.weight", (H, F)),
                (pre + "feed_forward.w3.weight", (F, H))]
    out += [("norm.weight", (H,)), ("output.weight", (p.vocab_size, H))]
    return out


def _is_projection(name: str) -> bool:
    return any(name.endswith(s + ".weight") for s in PROJECTIONS)


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even FP32 -> BF16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def generate(p: Qwen3Profile, layout: str = "int4", seed: int = 0,
             std: float = 0.02) -> Dict[str, np.ndarray]:
    """All tensors of a synthetic checkpoint as numpy arrays, in container order.

    Every tensor is drawn in descriptor order from one ``default_rng(seed)``.
    Returns {fire name: array} (INT4 triplets as ``.qweight/.scales/.zero_points``).
    """
    if layout not in ("int4", "mixed"):
        raise ValueError("layout must be 'int4' or 'mixed'")
    rng = np.random.default_rng(seed)
    out: Dict[str, np.ndarray] = {}
    for name, shape in descriptor(p):
        if len(shape) == 1:
            out[name] = np.ones(shape, np.float32)
            continue
        w = rng.normal(0.0, std, shape).astype(np.float32)
        quantised = _is_projection(name) or (layout == "int4" and name == "output.weight")
        if quantised:
            q, s, z = quantize_int4_groupwise(w, GROUP_SIZE)
            if layout == "mixed":
                s = s.astype(np.float16).astype(np.float32)
            base = name[: -len(".weight")]
            out[base + ".qweight"] = pack_uint4(q)
            out[base + ".scales"] = s
            out[base + ".zero_points"] = z
        elif layout == "mixed":
            out[name] = _bf16_bits(w)
        else:
            out[name] = w
    return out


def container_entries(weights: Dict[str, np.ndarray]) -> List[Tuple[str, np.ndarray, int]]:
    """(name, array, group) entries for :func:`fire_b200.fire_format.write`."""
    return [(n, a, GROUP_SIZE if n.endswith(".qweight") else 0) for n, a in weights.items()]


def generate_torch(p: Qwen3Profile, layout: str = "mixed", seed: int = 0, std: float = 0.02,
                   device="cuda") -> Dict[str, "object"]:
    """The same construction drawn with a seeded torch generator on ``device``.

    Used for the large (8B) workloads, which would take minutes to draw with numpy.
    Same names, dtypes, shapes, distribution and quantisation rule as
    :func:`generate` (a different random stream). BF16 tensors are returned as
    uint16-viewable int16 bit patterns.
    """
    import torch

    from .quant import quantize_torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out: Dict[str, object] = {}
    for name, shape in descriptor(p):
        if len(shape) == 1:
            out[name] = torch.ones(shape, dtype=torch.float32, device=device)
            continue
        quantised = _is_projection(name) or (layout == "int4" and name == "output.weight")
        if quantised:
            w = torch.empty(shape, dtype=torch.float32, device=device).normal_(0.0, std,
                                                                             generator=gen)
            q, s, z = quantize_torch(w, GROUP_SIZE)
            del w
            if layout == "mixed":
                s = s.to(torch.float16).to(torch.float32)
            base = name[: -len(".weight")]
            out[base + ".qweight"], out[base + ".scales"], out[base + ".zero_points"] = q, s, z
        else:
            # Draw row blocks so a [151936, 4096] FP32 intermediate never exists at once.
            dt = torch.bfloat16 if layout == "mixed" else torch.float32
            t = torch.empty(shape, dtype=dt, device=device)
            step = 16384
            for r in range(0, shape[0], step):
                blk = torch.empty((min(step, shape[0] - r), shape[1]), dtype=torch.float32,
                                  device=device).normal_(0.0, std, generator=gen)
                t[r:r + blk.shape[0]] = blk.to(dt)
            out[name] = t.view(torch.int16) if dt == torch.bfloat16 else t
    return out
