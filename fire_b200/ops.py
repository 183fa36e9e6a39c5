"""Fire's operator interface on top of the fire_b200 C ABI (GPU only).

Mirrors ``include/Fire/op/*.h`` / ``src/op/*.cpp``: the same operator names,
``forward`` signatures (input/output tensors + an ``OpContext``), the same
argument checks and the same ``Status`` results (``InvalidArgument`` with a message
instead of a launch), so Fire's op tests read the same here. Tensors are CUDA
``torch.Tensor`` views (torch provides device memory and streams only); every
computation is a call into ``libfire_b200.so``. There is no CPU path: a CPU
context is rejected, as Fire rejects INT4 on CPU (``src/op/linear.cpp:68-74``).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch

from . import _native as N


class StatusCode(enum.IntEnum):
    """include/Fire/base/base.h:41-49."""
    Success = 0
    FunctionUnImplement = 1
    PathNotValid = 2
    ModelParseError = 3
    InternalError = 5
    KeyValueHasExist = 6
    InvalidArgument = 7


@dataclass
class Status:
    code: StatusCode = StatusCode.Success
    message: str = ""

    def ok(self) -> bool:
        return self.code == StatusCode.Success

    __bool__ = ok


def Success() -> Status:
    return Status()


def InvalidArgument(msg: str) -> Status:
    return Status(StatusCode.InvalidArgument, msg)


def InternalError(msg: str) -> Status:
    return Status(StatusCode.InternalError, msg)


class DeviceType(enum.IntEnum):
    Unknown = 0
    GPU = 1
    CPU = 2


class DataType(enum.IntEnum):
    Unknown = 0
    Fp32 = 1
    Int8 = 2
    Int32 = 3
    UInt8 = 4
    Bf16 = 5


class QuantType(enum.IntEnum):
    """include/Fire/op/operator.h:25-31."""
    None_ = 0
    Int8GroupWise = 1
    Int8PerTensor = 2
    Int8PerChannel = 3
    Int4GroupWise = 4


@dataclass
class QuantConfig:
    quant_type: QuantType = QuantType.None_
    group_size: int = 0
    symmetric: bool = True


@dataclass
class Parameter:
    """include/Fire/op/operator.h:43-69: data + optional INT4 metadata."""
    data: Optional[torch.Tensor] = None
    quant_config: QuantConfig = field(default_factory=QuantConfig)
    scales: Optional[torch.Tensor] = None
    zero_points: Optional[torch.Tensor] = None

    def is_quantized(self) -> bool:
        return self.quant_config.quant_type != QuantType.None_


@dataclass
class OpContext:
    """include/Fire/op/operator.h:78-85 (the stream is a torch.cuda.Stream or None)."""
    device_type: DeviceType = DeviceType.Unknown
    stream: Optional[torch.cuda.Stream] = None
    workspace: Optional[torch.Tensor] = None


_DT = {torch.float32: DataType.Fp32, torch.int8: DataType.Int8, torch.int32: DataType.Int32,
       torch.uint8: DataType.UInt8, torch.bfloat16: DataType.Bf16}


def data_type(t: torch.Tensor) -> DataType:
    return _DT.get(t.dtype, DataType.Unknown)


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _check_tensor(t: Optional[torch.Tensor], device: DeviceType, dtype: DataType) -> Status:
    """Operator::_check_tensor (src/op/operator.cpp): allocated, right device and dtype."""
    if t is None or t.numel() == 0:
        return InvalidArgument("tensor is empty")
    if device == DeviceType.GPU and not t.is_cuda:
        return InvalidArgument("tensor device does not match the context")
    if device == DeviceType.CPU and t.is_cuda:
        return InvalidArgument("tensor device does not match the context")
    if data_type(t) != dtype:
        return InvalidArgument("tensor data type mismatch")
    if not t.is_contiguous():
        return InvalidArgument("tensor must be contiguous")
    return Success()


def _gpu_only(ctx: OpContext, what: str) -> Status:
    if ctx.device_type not in (DeviceType.CPU, DeviceType.GPU):
        return InvalidArgument(f"{what} requires a CPU or GPU device")
    if ctx.device_type != DeviceType.GPU:
        return InvalidArgument(f"{what}: fire_b200 runs on the GPU only")
    return Success()


def _launch(status: int, what: str) -> Status:
    return Success() if status == N.OK else InternalError(f"{what}: {N.status_string(status)}")


class _ParamOperator:
    def __init__(self) -> None:
        self.params: List[Parameter] = []

    def reset_param_size(self, n: int) -> None:
        self.params = [Parameter() for _ in range(n)]

    def get_param(self, i: int) -> Parameter:
        return self.params[i]

    def set_param(self, i: int, p) -> None:
        self.params[i] = p if isinstance(p, Parameter) else Parameter(data=p)


class LinearOp(_ParamOperator):
    """src/op/linear.cpp:11-159. INT4 group-wise or FP32/BF16 weights (+ optional bias)."""

    def __init__(self, matmul_scale: float = 1.0) -> None:
        super().__init__()
        self.matmul_scale = matmul_scale

    def forward(self, x: torch.Tensor, y: torch.Tensor, ctx: OpContext) -> Status:
        st = self._check(x, y, ctx)
        if not st:
            return st
        p = self.params[0]
        rows = 1 if x.dim() == 1 else x.shape[0]
        k = x.shape[-1]
        s = N.stream_handle(ctx.stream)
        if p.is_quantized():
            rc = N.lib().fire_b200_linear_w4(_ptr(x), _ptr(p.data), _ptr(p.scales), _ptr(p.zero_points),
                                             _ptr(y), rows, p.data.shape[0], k, p.quant_config.group_size, s)
            return _launch(rc, "linear int4")
        w = p.data
        dt = N.BF16 if w.dtype == torch.bfloat16 else N.F32
        rc = N.lib().fire_b200_linear_dense(_ptr(x), _ptr(w), dt, self.matmul_scale, _ptr(y), rows,
                                            w.shape[0], k, s)
        if rc == N.OK and len(self.params) == 2:
            rc = N.lib().fire_b200_add(_ptr(y), _ptr(self.params[1].data), _ptr(y), y.numel(), s)
        return _launch(rc, "linear dense")

    def _check(self, x, y, ctx) -> Status:
        st = _gpu_only(ctx, "linear")
        if not st:
            return st
        if not self.params or len(self.params) > 2:
            return InvalidArgument("linear requires a weight and an optional bias")
        for t in (x, y):
            st = _check_tensor(t, ctx.device_type, DataType.Fp32)
            if not st:
                return st
        if x.dim() not in (1, 2):
            return InvalidArgument("linear only supports one- or two-dimensional input")
        if y.dim() != x.dim():
            return InvalidArgument("linear input and output rank mismatch")
        p = self.params[0]
        k = x.shape[-1]
        if p.is_quantized():
            if len(self.params) != 1:
                return InvalidArgument("quantized linear does not support bias")
            if p.quant_config.quant_type != QuantType.Int4GroupWise:
                return InvalidArgument("linear only supports group-wise int4 weights")
            st = _check_tensor(p.data, ctx.device_type, DataType.UInt8)
            if not st:
                return st
            if p.data.dim() != 2:
                return InvalidArgument("quantized linear weight must be two-dimensional")
            n = p.data.shape[0]
            if k % 2 or p.data.shape[1] != k // 2:
                return InvalidArgument("linear input feature dimension does not match packed int4 weight")
            g = p.quant_config.group_size
            if g <= 0 or k % g:
                return InvalidArgument("quantized linear group size must be positive and divide input features")
            meta = (n, k // g)
            st = _check_tensor(p.scales, ctx.device_type, DataType.Fp32)
            if not st:
                return st
            if tuple(p.scales.shape) != meta:
                return InvalidArgument("quantized linear scales shape mismatch")
            st = _check_tensor(p.zero_points, ctx.device_type, DataType.UInt8)
            if not st:
                return st
            if tuple(p.zero_points.shape) != meta:
                return InvalidArgument("quantized linear zero points shape mismatch")
        else:
            if p.data is None or data_type(p.data) not in (DataType.Fp32, DataType.Bf16):
                return InvalidArgument("linear weight must be FP32 or BF16")
            st = _check_tensor(p.data, ctx.device_type, data_type(p.data))
            if not st:
                return st
            if p.data.dim() != 2:
                return InvalidArgument("linear weight must be two-dimensional")
            n = p.data.shape[0]
            if p.data.shape[1] != k:
                return InvalidArgument("linear input feature dimension does not match weight")
            if len(self.params) == 2:
                st = _check_tensor(self.params[1].data, ctx.device_type, DataType.Fp32)
                if not st:
                    return st
                if self.params[1].data.numel() != y.numel():
                    return InvalidArgument("linear bias size must match the output size")
        if y.shape[-1] != n:
            return InvalidArgument("linear output feature dimension does not match weight")
        if x.dim() == 2 and x.shape[0] != y.shape[0]:
            return InvalidArgument("linear input and output row count mismatch")
        return Success()


class RmsNormOp(_ParamOperator):
    """src/op/rmsnorm.cpp:11-57: 1-D input -> whole-vector norm, else per-row norm."""

    def __init__(self, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps

    def forward(self, x: torch.Tensor, y: torch.Tensor, ctx: OpContext) -> Status:
        dim = x.shape[-1] if x is not None and x.dim() > 0 else 0
        if dim <= 0:
            return InvalidArgument("rmsnorm dimension must be positive")
        st = _gpu_only(ctx, "rmsnorm")
        if not st:
            return st
        if len(self.params) != 1:
            return InvalidArgument("rmsnorm requires exactly one weight parameter")
        if self.params[0].is_quantized():
            return InvalidArgument("rmsnorm does not support quantized weights")
        for t in (x, y, self.params[0].data):
            st = _check_tensor(t, ctx.device_type, DataType.Fp32)
            if not st:
                return st
        if tuple(x.shape) != tuple(y.shape):
            return InvalidArgument("rmsnorm input and output shape mismatch")
        w = self.params[0].data
        if tuple(w.shape) != (dim,):
            return InvalidArgument("rmsnorm weight shape mismatch")
        s = N.stream_handle(ctx.stream)
        if x.dim() != 1:
            rc = N.lib().fire_b200_rmsnorm_rows(_ptr(x), _ptr(w), _ptr(y), x.numel() // dim, dim, self.eps, s)
        else:
            rc = N.lib().fire_b200_rmsnorm(_ptr(x), _ptr(w), _ptr(y), dim, self.eps, s)
        return _launch(rc, "rmsnorm")


class RoPEOp:
    """src/op/rope.cpp: q [heads, hs], k [kv_heads, hs], caches [max_seq, hs/2]."""

    def forward(self, q, k, cos, sin, pos: int, ctx: OpContext) -> Status:
        st = _gpu_only(ctx, "rope")
        if not st:
            return st
        for t in (q, k, cos, sin):
            st = _check_tensor(t, ctx.device_type, DataType.Fp32)
            if not st:
                return st
        if q.dim() != 2 or k.dim() != 2 or cos.dim() != 2 or sin.dim() != 2:
            return InvalidArgument("rope tensors must be two-dimensional")
        hs = q.shape[1]
        if hs % 2 or k.shape[1] != hs:
            return InvalidArgument("rope head size must be even and match between q and k")
        if k.shape[0] > q.shape[0]:
            return InvalidArgument("rope key heads exceed query heads")
        if tuple(cos.shape) != tuple(sin.shape) or cos.shape[1] != hs // 2:
            return InvalidArgument("rope cache shape must be [max_seq, head_size/2]")
        if pos < 0 or pos >= cos.shape[0]:
            return InvalidArgument("rope position is outside the cache")
        rc = N.lib().fire_b200_rope(_ptr(q), _ptr(k), _ptr(cos), _ptr(sin), q.shape[0], k.shape[0], hs,
                                    cos.shape[0], pos, N.stream_handle(ctx.stream))
        return _launch(rc, "rope")


def rope_cache(head_size: int, max_seq: int, theta: float, sin: torch.Tensor, cos: torch.Tensor,
               stream=None) -> None:
    """RoPECacheKernel (kernels_interface.h:33-35)."""
    N.check(N.lib().fire_b200_rope_cache(head_size, max_seq, theta, _ptr(sin), _ptr(cos),
                                         N.stream_handle(stream)), "rope cache")


class MultiHeadAttentionOp:
    """src/op/mha.cpp:15-90 (score [q_heads, capacity] receives the probabilities)."""

    def forward(self, q, key_cache, value_cache, score, out, layer: int, pos: int, ctx: OpContext) -> Status:
        st = _gpu_only(ctx, "mha")
        if not st:
            return st
        for t in (q, key_cache, value_cache, score, out):
            st = _check_tensor(t, ctx.device_type, DataType.Fp32)
            if not st:
                return st
        if q.dim() != 2:
            return InvalidArgument("mha query must be two-dimensional")
        if key_cache.dim() != 4 or value_cache.dim() != 4:
            return InvalidArgument("mha key and value caches must be four-dimensional")
        if score.dim() != 2 or out.dim() != 2:
            return InvalidArgument("mha score and output must be two-dimensional")
        if tuple(key_cache.shape) != tuple(value_cache.shape):
            return InvalidArgument("mha key and value cache shapes must match")
        qh, hd = q.shape
        layers, cap, kvh, khd = key_cache.shape
        if layer < 0 or layer >= layers:
            return InvalidArgument("mha layer index is outside the cache")
        if pos < 0 or pos >= cap:
            return InvalidArgument("mha position is outside the cache capacity")
        if hd != khd:
            return InvalidArgument("mha query and cache head dimensions must match")
        if kvh > qh or qh % kvh:
            return InvalidArgument("mha query head count must be divisible by the KV head count")
        if tuple(score.shape) != (qh, cap):
            return InvalidArgument("mha score shape must be [query heads, capacity]")
        if tuple(out.shape) != (qh, hd):
            return InvalidArgument("mha output shape must match the query shape")
        need = N.lib().fire_b200_mha_workspace_bytes(qh, kvh, hd, cap)
        ws = ctx.workspace
        if ws is None or ws.numel() * ws.element_size() < need:
            ws = torch.zeros(need, dtype=torch.uint8, device=q.device)
            ctx.workspace = ws
        rc = N.lib().fire_b200_mha_decode(_ptr(q), _ptr(key_cache), _ptr(value_cache), _ptr(score), _ptr(out),
                                          layers, cap, qh, kvh, hd, layer, pos, _ptr(ws),
                                          ws.numel() * ws.element_size(), N.stream_handle(ctx.stream))
        return _launch(rc, "mha")


class EmbeddingOp(_ParamOperator):
    """src/op/embedding.cpp: int32 tokens [n] -> [n, dim] (or [dim] for one token)."""

    def forward(self, tokens, out, ctx: OpContext) -> Status:
        st = _gpu_only(ctx, "embedding")
        if not st:
            return st
        if len(self.params) != 1:
            return InvalidArgument("embedding requires exactly one weight parameter")
        w = self.params[0].data
        st = _check_tensor(tokens, ctx.device_type, DataType.Int32)
        if not st:
            return st
        if w is None or w.dim() != 2 or data_type(w) not in (DataType.Fp32, DataType.Bf16):
            return InvalidArgument("embedding weight must be a FP32 or BF16 matrix")
        st = _check_tensor(out, ctx.device_type, DataType.Fp32)
        if not st:
            return st
        if out.numel() != tokens.numel() * w.shape[1]:
            return InvalidArgument("embedding output shape mismatch")
        dt = N.BF16 if w.dtype == torch.bfloat16 else N.F32
        rc = N.lib().fire_b200_embedding(_ptr(tokens), tokens.numel(), _ptr(w), dt, w.shape[0], w.shape[1],
                                         _ptr(out), N.stream_handle(ctx.stream))
        return _launch(rc, "embedding")


class _Binary:
    name = ""

    def forward(self, a, b, out, ctx: OpContext) -> Status:
        st = _gpu_only(ctx, self.name)
        if not st:
            return st
        for t in (a, b, out):
            st = _check_tensor(t, ctx.device_type, DataType.Fp32)
            if not st:
                return st
        if tuple(a.shape) != tuple(b.shape) or tuple(a.shape) != tuple(out.shape):
            return InvalidArgument(f"{self.name} input and output shapes must match")
        return _launch(self._call(a, b, out, N.stream_handle(ctx.stream)), self.name)


class VecAddOp(_Binary):
    """src/op/add.cpp."""
    name = "add"

    def _call(self, a, b, out, s):
        return N.lib().fire_b200_add(_ptr(a), _ptr(b), _ptr(out), a.numel(), s)


class SwiGLUOp(_Binary):
    """src/op/swiglu.cpp."""
    name = "swiglu"

    def _call(self, a, b, out, s):
        return N.lib().fire_b200_swiglu(_ptr(a), _ptr(b), _ptr(out), a.numel(), s)


def argmax(logits: torch.Tensor, stream=None, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Device-side greedy argmax (first index of the maximum) -> int64 CUDA scalar tensor."""
    L = N.lib()
    need = L.fire_b200_argmax_workspace_bytes()
    if workspace is None or workspace.numel() < need:
        workspace = torch.zeros(need, dtype=torch.uint8, device=logits.device)
    out = torch.empty((), dtype=torch.int64, device=logits.device)
    N.check(L.fire_b200_argmax(_ptr(logits), logits.numel(), _ptr(out), _ptr(workspace), workspace.numel(),
                               N.stream_handle(stream)), "argmax")
    return out
