"""The tensor-core prefill Linear (INT4 group 128 dequantised to FP16, each row of x scaled
by a power of two and rounded to FP16, tcgen05 MMA with an FP32 TMEM accumulator) against
FP32 references of the same product.

Bars: rel-L2 <= 1e-3 against the FP32 Linear on the dequantised weights (the reference's
FP32 CPU path, src/op/kernels/cpu/matmul_kernel.cpp:6-52, on the weights of tools/quant.py
dequantize_int4_groupwise), and rel-L2 <= 5e-5 against the same product with the kernel's
own operand rounding applied first (W and the row-scaled x to FP16), which isolates the
kernel's arithmetic (the tensor cores' FP32 accumulation, in their order, over up to 12288
terms).
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


def f16_round(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float64)


def x_as_f16(x):
    """Each row times 2^sh (its largest |x| into [2^14, 2^15)), rounded to FP16, scaled back."""
    x = np.asarray(x, np.float32)
    _, e = np.frexp(np.max(np.abs(x), axis=1))
    sh = np.clip(15 - e, -126, 126).astype(np.float64)[:, None]
    return f16_round(x * np.exp2(sh).astype(np.float32)) * np.exp2(-sh)


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
    ref16 = x_as_f16(x) @ f16_round(wdq).T
    assert np.isfinite(y).all()
    assert rel_l2(y, ref16) <= 5e-5, rel_l2(y, ref16)
    assert rel_l2(y, ref32) <= 1e-3, rel_l2(y, ref32)


def test_prefill_rejects_unsupported_shapes(cuda):
    L = N.lib()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    # rows not a multiple of 128, group not 128, workspace too small, null pointer
    assert L.fire_b200_linear_w4_prefill(p, p, p, p, p, 100, 128, 128, 128, p, 1 << 20, None, 0) == N.ERR_UNSUPPORTED
    assert L.fire_b200_linear_w4_prefill(p, p, p, p, p, 128, 128, 128, 64, p, 1 << 20, None, 0) == N.ERR_UNSUPPORTED
    assert L.fire_b200_linear_w4_prefill(p, p, p, p, p, 128, 128, 4096, 128, p, 1024, None, 0) == N.ERR_INVALID
    assert L.fire_b200_linear_w4_prefill(None, p, p, p, p, 128, 128, 128, 128, p, 1 << 20, None, 0) == N.ERR_INVALID
    assert L.fire_b200_linear_w4_prefill_workspace_bytes(512, 4096, 4096) == 512 * 4096 * 2 + 512 * 4 + 4096 * 4096 * 2


def test_prefill_refuses_weights_beyond_fp16(cuda):
    """A group whose dequantised weights can exceed the FP16 range (|s| * max(z, 15 - z) >
    65504) is reported through the status word (4) instead of producing infinities."""
    m, n, k = 128, 128, 256
    x, packed, s, z, _ = make(m, n, k, seed=3)
    s = s.copy()
    s[7, 1] = 1e4
    L = N.lib()
    dx, dq, ds, dz = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (x, packed, s, z))
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    wsb = L.fire_b200_linear_w4_prefill_workspace_bytes(m, n, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.fire_b200_linear_w4_prefill(dx.data_ptr(), dq.data_ptr(), ds.data_ptr(), dz.data_ptr(), y.data_ptr(), m,
                                       n, k, 128, ws.data_ptr(), wsb, st.data_ptr(), 0)
    assert rc == N.OK
    torch.cuda.synchronize()
    assert int(st.item()) == 4


# ------------------------------------------------------------ engine prefill ----
from fire_b200 import synth  # noqa: E402
from fire_b200.engine import Qwen3Engine  # noqa: E402
from fire_b200.profiles import TINY, Qwen3Profile  # noqa: E402

SMALL = Qwen3Profile("small-qwen3", 4096, 4096, 512, 1536, 3, 8, 4, 128)
# four q heads per KV head, as Qwen3-8B
G4 = Qwen3Profile("g4-qwen3", 4096, 4096, 1024, 1536, 2, 8, 2, 128)


def _oracle_prefix(O, p, w, prompt, cap):
    ref = O.Qwen3Oracle(p, w, capacity=cap)
    lg = None
    for i, t in enumerate(prompt):
        lg = ref.forward(int(t), i)
    return ref, lg


@pytest.mark.parametrize("profile,n", [(TINY, 200), (SMALL, 200), (G4, 200), (G4, 1100), (TINY, 2100)])
def test_engine_prefill_matches_token_by_token(cuda, profile, n):
    """Batched prefill leaves the last logits and the KV cache as the token-by-token oracle
    does, to FP16-GEMM accuracy: logits rel-L2 <= 1e-2 with the same argmax, and the next
    decode step on the prefilled cache agrees the same way."""
    from oracle import oracle as O

    w = synth.generate(profile, "int4", seed=21)
    cap = n + 8
    eng = Qwen3Engine(profile, w)
    eng.prepare(cap)
    prompt = np.random.default_rng(n).integers(0, profile.vocab_size, n)
    logits = torch.empty(profile.vocab_size, device="cuda")
    eng.prefill(prompt.tolist(), logits)
    assert eng.length == n
    got = logits.cpu().numpy()
    ref, want = _oracle_prefix(O, profile, w, prompt, cap)
    assert rel_l2(got, want) <= 1e-2, rel_l2(got, want)
    assert int(np.argmax(got)) == int(np.argmax(want))
    nxt = int(np.argmax(want))
    eng.forward(nxt, n, logits)
    torch.cuda.synchronize()
    got2, want2 = logits.cpu().numpy(), ref.forward(nxt, n)
    assert rel_l2(got2, want2) <= 1e-2, rel_l2(got2, want2)
    assert int(np.argmax(got2)) == int(np.argmax(want2))


def test_engine_prefill_short_prompt_is_forward_per_token(cuda):
    w = synth.generate(TINY, "int4", seed=3)
    a, b = Qwen3Engine(TINY, w), Qwen3Engine(TINY, w)
    a.prepare(64)
    b.prepare(64)
    prompt = [5, 17, 900, 3, 42]
    la, lb = torch.empty(TINY.vocab_size, device="cuda"), torch.empty(TINY.vocab_size, device="cuda")
    a.prefill(prompt, la)
    for i, t in enumerate(prompt):
        b.forward(t, i, lb)
    torch.cuda.synchronize()
    assert a.length == b.length == len(prompt)
    assert torch.equal(la, lb)
    with pytest.raises(N.FireB200Error):
        a.prefill([TINY.vocab_size], la)  # bad id: rejected, nothing consumed
    assert a.length == len(prompt)


def test_one_pass_dequant_gemm_bit_identical_to_two_pass(cuda, tmp_path):
    """The one-pass kernel (W dequantised into shared memory inside the GEMM, selected with
    FIRE_B200_PREFILL_FUSED=1) gives the same bits as the default two-pass form (W
    dequantised to FP16 in HBM first, then the GEMM): the Linear at the 8B projection shapes
    and a whole engine prefill + one decode step."""
    import os
    import subprocess
    import sys

    from tests import prefill_one_pass_child as child

    path = tmp_path / "one_pass.npz"
    env = dict(os.environ, FIRE_B200_PREFILL_FUSED="1")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    subprocess.run([sys.executable, "-m", "tests.prefill_one_pass_child", str(path)], env=env, cwd=root,
                   check=True, timeout=600)
    want = np.load(path)
    got = child.compute()
    assert set(got) == set(want.files)
    for key, g in got.items():
        assert np.array_equal(g.view(np.uint32), want[key].view(np.uint32)), key
