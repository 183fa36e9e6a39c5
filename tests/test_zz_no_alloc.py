"""GPU: the attention entry point that allocates nothing (fire_b200_mha_decode_noalloc).

It exists for callers that cannot allocate device memory or pass a workspace - a plug-in
behind an interface that only hands over its tensors, or a program whose device memory
is fixed at start-up. Its scratch is an array inside the library, so this test checks,
through the C ABI, that it gives the same result as the workspace entry point
(fire_b200_mha_decode) on two calls in a row (the array keeps the previous call's
contents), and that shapes whose scratch would not fit are rejected.

The file is named to run last, so a failure here cannot hide the other tests.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fire_b200 import _native as N

pytestmark = pytest.mark.gpu

_vp, _i = C.c_void_p, C.c_int


def _bind():
    L = N.lib()
    f = L.fire_b200_mha_decode_noalloc
    f.restype = _i
    f.argtypes = [_vp] * 5 + [_i] * 7 + [_vp]
    return L, f


def _vals(size, mul, off, scale):
    i = np.arange(size)
    return ((((i * mul + off) % 31).astype(np.int64) - 15) * scale).astype(np.float32)


@pytest.mark.parametrize("shape,layer,pos", [((2, 257, 4, 2, 5), 1, 256), ((2, 2048, 32, 8, 128), 1, 2047),
                                             ((3, 300, 16, 8, 128), 2, 129)])
def test_noalloc_matches_workspace_entry_point_twice(cuda, shape, layer, pos):
    L, noalloc = _bind()
    layers, cap, qh, kvh, hd = shape
    q = torch.from_numpy(_vals(qh * hd, 7, 3, 0.125).reshape(qh, hd)).cuda()
    kc = torch.from_numpy(_vals(layers * cap * kvh * hd, 11, 5, 0.0625).reshape(layers, cap, kvh, hd)).cuda()
    vc = torch.from_numpy(_vals(layers * cap * kvh * hd, 13, 9, 0.1875).reshape(layers, cap, kvh, hd)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    need = L.fire_b200_mha_workspace_bytes(qh, kvh, hd, cap)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    ref_out = torch.empty((qh, hd), device="cuda")
    ref_score = torch.full((qh, cap), -777.0, device="cuda")
    assert L.fire_b200_mha_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ref_score.data_ptr(),
                                  ref_out.data_ptr(), layers, cap, qh, kvh, hd, layer, pos, ws.data_ptr(), need,
                                  stream) == N.OK
    for call in range(2):
        out = torch.full((qh, hd), float("nan"), device="cuda")
        score = torch.full((qh, cap), -777.0, device="cuda")
        assert noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), score.data_ptr(), out.data_ptr(), layers, cap,
                       qh, kvh, hd, layer, pos, stream) == N.OK, f"call {call}"
        torch.cuda.synchronize()
        # same tolerance as the attention parity tests (test/test_op/test_mha.cpp:204-215)
        assert torch.all(torch.abs(out - ref_out) <= 3e-5), f"call {call}"
        assert torch.all(torch.abs(score[:, :pos + 1] - ref_score[:, :pos + 1]) <= 2e-5), f"call {call}"
        assert torch.all(score[:, pos + 1:] == -777.0)


def test_noalloc_rejects_scratch_beyond_its_fixed_size(cuda):
    L, noalloc = _bind()
    p = C.c_void_p(256)  # never dereferenced: the size check rejects first
    # 32 q heads x dim 128 need more than 4 MiB of scratch beyond capacity 16128
    assert noalloc(p, p, p, None, p, 1, 16128 + 64, 32, 8, 128, 0, 0, None) == N.ERR_UNSUPPORTED
    assert noalloc(None, p, p, None, p, 1, 64, 32, 8, 128, 0, 0, None) == N.ERR_INVALID
