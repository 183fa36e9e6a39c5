"""The drop-in boundary end to end: the reference's own LinearOp::forward
(src/op/linear.cpp:11-36, with its _check validation :38-159 and Fire's Tensor / Parameter /
OpContext types), compiled from its sources, dispatching through the integration shims to the
fire_b200 C ABI (oracle/Makefile `boundary`, oracle/ref_shim/boundary.cpp). Results must match
the oracle as the direct C ABI calls do; arguments Fire's operator rejects never reach a kernel.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from fire_b200 import quant
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(O.__file__), "_ref", "libfire_boundary.so")
SUCCESS, INVALID_ARGUMENT = 0, 7  # base::StatusCode (include/Fire/base/base.h:41-49)
NOT_CALLED = -1000  # kernel_rc when the operator never reached a kernel


@pytest.fixture(scope="module")
def boundary(cuda):
    if not os.path.exists(LIB):
        pytest.skip("reference boundary library not built (oracle/Makefile boundary)")
    L = C.CDLL(LIB)
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    L.boundary_linear_w4.argtypes = [vp] * 5 + [i] * 4 + [vp, C.POINTER(i)]
    L.boundary_linear_dense.argtypes = [vp, vp, i, f, vp, i, i, i, vp, C.POINTER(i)]
    return L


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def run_w4(L, x, p, s, z, rows, n, k, group):
    y = torch.empty((rows, n), device="cuda")
    krc = C.c_int(-99)
    d = [dev(a) for a in (x, p, s, z)]  # kept alive across the call
    st = L.boundary_linear_w4(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), y.data_ptr(),
                              rows, n, k, group, None, C.byref(krc))
    torch.cuda.synchronize()
    return st, krc.value, y.cpu().numpy()


@pytest.mark.parametrize("n,k,seed", [(3072, 1024, 0), (12288, 4096, 1), (4096, 12288, 2)])
def test_fire_linear_op_reaches_fire_b200_int4_gemv(boundary, n, k, seed):
    """Config-1 (3072x1024, N(0,0.02) seed 0, RTN) and two Qwen3-8B shapes through Fire's LinearOp."""
    rng = np.random.default_rng(seed)
    W = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, (1, k)).astype(np.float32)[0]
    q, s, z = quant.quantize_int4_groupwise(W, 128)
    p = quant.pack_uint4(q)
    st, krc, y = run_w4(boundary, x, p, s, z, 1, n, k, 128)
    assert st == SUCCESS and krc == 0
    assert rel_l2(y[0], O.linear_int4(x, p, s, z)) <= 1e-5


def test_fire_linear_op_multi_row_and_odd_group(boundary):
    """Two-dimensional input (rows 17) and group 3 splitting a byte: fire_b200's general path."""
    rng = np.random.default_rng(5)
    n, k = 19, 258
    W = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, (17, k)).astype(np.float32)
    q, s, z = quant.quantize_int4_groupwise(W, 3)
    p = quant.pack_uint4(q)
    st, krc, y = run_w4(boundary, x, p, s, z, 17, n, k, 3)
    assert st == SUCCESS and krc == 0
    want = O.linear_int4(x, p, s, z, 3)
    assert np.all(np.abs(y - want) <= 1e-3)


def test_fire_linear_op_rejects_before_the_kernel(boundary):
    """A group size that does not divide K is refused by LinearOp::_check (src/op/linear.cpp:93-97):
    InvalidArgument, and the fire_b200 kernel is never called."""
    n, k = 16, 256
    p = np.zeros((n, k // 2), np.uint8)
    s = np.ones((n, 2), np.float32)
    z = np.zeros((n, 2), np.uint8)
    st, krc, _ = run_w4(boundary, np.ones(k, np.float32), p, s, z, 1, n, k, 100)
    assert st == INVALID_ARGUMENT and krc == NOT_CALLED


def test_fire_linear_op_bf16_head_with_scale(boundary):
    rng = np.random.default_rng(9)
    n, k = 3000, 4096
    wf = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    wb = (wf.view(np.uint32) >> 16).astype(np.uint16)
    x = rng.normal(0, 1, k).astype(np.float32)
    y = torch.empty(n, device="cuda")
    krc = C.c_int(-99)
    dx, dw = dev(x), dev(wb)
    st = boundary.boundary_linear_dense(dx.data_ptr(), dw.data_ptr(), 1, 0.5, y.data_ptr(), 1, n, k, None,
                                        C.byref(krc))
    torch.cuda.synchronize()
    assert st == SUCCESS and krc.value == 0
    assert rel_l2(y.cpu().numpy(), O.linear_bf16(x, wb, 0.5)) <= 1e-5
