"""The tensor-core prefill Linear (INT4 group 128 dequantised to BF16, tcgen05 MMA with an
FP32 TMEM accumulator) against FP32 references of the same product.

Bars: rel-L2 <= 2e-3 against the FP32 Linear on the dequantised weights (the reference's
FP32 CPU path, src/op/kernels/cpu/matmul_kernel.cpp:6-52, on the weights of tools/quant.py
dequantize_int4_groupwise), and rel-L2 <= 5e-5 against the same product with the kernel's
own operand rounding applied first (W to BF16, x to bf16(x) + bf16(x - bf16(x))), which
isolates the kernel's arithmetic (the tensor cores' FP32 accumulation, in their order, over
up to 12288 terms).
"""
import numpy as np
import pytest
import torch

from fire_b200 import _native as N
from fire_b200 import quant

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_round(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def bf16_split(a):
    hi = bf16_round(a)
    return hi.astype(np.float64) + bf16_round(np.asarray(a, np.float32) - hi).astype(np.float64)


def make(m, n, k, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    q, s, z = quant.quantize_int4_groupwise(w, 128)
    packed = quant.pack_uint4(q)
    x = rng.normal(0.0, 1.0, (m, k)).astype(np.float32)
    wdq = quant.dequantize_int4_groupwise(packed, s, z, 128).astype(np.float32)
    return x, packed, s.astype(np.float32), z.astype(np.uint8), wdq


def run(x, packed, s, z, m, n, k):
    L = N.lib()
    dx, dq, ds, dz = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (x, packed, s, z))
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    wsb = L.fire_b200_linear_w4_prefill_workspace_bytes(m, n, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.fire_b200_linear_w4_prefill(dx.data_ptr(), dq.data_ptr(), ds.data_ptr(), dz.data_ptr(), y.data_ptr(), m,
                                       n, k, 128, ws.data_ptr(), wsb, st.data_ptr(), 0)
    assert rc == N.OK, rc
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    return y.cpu().numpy()


@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (128, 128, 256), (256, 384, 1024),
                                   # the Qwen3-8B projection shapes at M = 512 (q/k/v, o, gate/up, down)
                                   (512, 6144, 4096), (512, 4096, 4096), (512, 24576, 4096), (512, 4096, 12288)])
def test_prefill_tcgen05_vs_fp32(cuda, m, n, k):
    x, packed, s, z, wdq = make(m, n, k, seed=m + n + k)
    y = run(x, packed, s, z, m, n, k)
    ref32 = x.astype(np.float64) @ wdq.astype(np.float64).T
    refbf = bf16_split(x) @ bf16_round(wdq).astype(np.float64).T
    assert np.isfinite(y).all()
    assert rel_l2(y, refbf) <= 5e-5, rel_l2(y, refbf)
    assert rel_l2(y, ref32) <= 2e-3, rel_l2(y, ref32)


def test_prefill_rejects_unsupported_shapes(cuda):
    L = N.lib()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    # rows not a multiple of 128, group not 128, workspace too small, null pointer
    assert L.fire_b200_linear_w4_prefill(p, p, p, p, p, 100, 128, 128, 128, p, 1 << 20, None, 0) == N.ERR_UNSUPPORTED
    assert L.fire_b200_linear_w4_prefill(p, p, p, p, p, 128, 128, 128, 64, p, 1 << 20, None, 0) == N.ERR_UNSUPPORTED
    assert L.fire_b200_linear_w4_prefill(p, p, p, p, p, 128, 128, 4096, 128, p, 1024, None, 0) == N.ERR_INVALID
    assert L.fire_b200_linear_w4_prefill(None, p, p, p, p, 128, 128, 128, 128, p, 1 << 20, None, 0) == N.ERR_INVALID
    assert L.fire_b200_linear_w4_prefill_workspace_bytes(512, 4096, 4096) == 2 * 512 * 4096 * 2 + 4096 * 4096 * 2
