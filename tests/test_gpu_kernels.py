"""GPU parity of every kernel-level entry point against the oracle (and, where it is
built, against the reference's own CUDA kernels compiled from source).

Tolerances: rel-L2 <= 1e-5 per INT4 / BF16 GEMV (FP32 accumulation in a different
order), the reference tests' own absolute bounds elsewhere.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fire_b200 import _native as N
from fire_b200 import ops, quant
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def w4(x, qw, s, z, y, rows, n, k, group, stream=0):
    return N.lib().fire_b200_linear_w4(x.data_ptr(), qw.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                       rows, n, k, group, stream)


def random_w4(rng, n, k, group=128):
    """Uniform nibbles, positive scales, zero points 0..15 (the stored layout)."""
    qw = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    s = (rng.random((n, k // group), dtype=np.float32) * 0.02 + 1e-3).astype(np.float32)
    z = rng.integers(0, 16, (n, k // group), dtype=np.uint8)
    return qw, s, z


# ------------------------------------------------------------------ INT4 GEMV ----

def test_w4_single_linear_workload(cuda):
    """W 3072x1024 ~ N(0,0.02) seed 0, RTN via the reference rule, x ~ N(0,1)."""
    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (3072, 1024)).astype(np.float32)
    x = rng.normal(0, 1, (1, 1024)).astype(np.float32)[0]
    q, s, z = quant.quantize_int4_groupwise(W, 128)
    p = quant.pack_uint4(q)
    y = torch.empty(3072, device="cuda")
    assert w4(dev(x), dev(p), dev(s), dev(z), y, 1, 3072, 1024, 128) == N.OK
    got = host(y)
    assert rel_l2(got, O.linear_int4(x, p, s, z)) <= REL_L2
    assert rel_l2(got, O.linear_int4_f64(x, p, s, z)) <= REL_L2


@pytest.mark.parametrize("n,k", [(4096, 4096), (1024, 4096), (12288, 4096), (4096, 12288), (6144, 4096),
                                 (24576, 4096), (2048, 1024), (512, 1536), (4096, 512), (151936 // 8, 1024)])
def test_w4_decode_shapes_vs_oracle(cuda, n, k):
    rng = np.random.default_rng(n * 7 + k)
    qw, s, z = random_w4(rng, n, k)
    x = rng.normal(0, 1, k).astype(np.float32)
    y = torch.empty(n, device="cuda")
    assert w4(dev(x), dev(qw), dev(s), dev(z), y, 1, n, k, 128) == N.OK
    got = host(y)
    assert rel_l2(got, O.linear_int4(x, qw, s, z)) <= REL_L2
    assert rel_l2(got, O.linear_int4_f64(x, qw, s, z)) <= REL_L2


def config3_w4(n, k, seed):
    """Qwen3-8B mixed-layout GEMV weights: W ~ N(0, 0.02) from default_rng(seed), RTN INT4
    group 128 by the reference rule (tools/quant.py:14-137), scales rounded to FP16 values
    (stored FP32), 4-bit zero points; x ~ N(0, 1) drawn after W."""
    rng = np.random.default_rng(seed)
    W = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, k).astype(np.float32)
    q, s, z = quant.quantize_int4_groupwise(W, 128)
    return x, quant.pack_uint4(q), s.astype(np.float16).astype(np.float32), z


@pytest.mark.parametrize("name,n,k", [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
                                      ("gate", 12288, 4096), ("up", 12288, 4096), ("down", 4096, 12288)])
def test_w4_qwen3_8b_gemv_sweep_shapes_rtn(cuda, name, n, k):
    """Every Qwen3-8B projection at M=1 on RTN weights with FP16-valued scales, against the
    oracle's dequantise-then-FP32 Linear and its float64 sum (rel-L2 <= 1e-5 each)."""
    x, qw, s, z = config3_w4(n, k, seed=0)
    y = torch.empty(n, device="cuda")
    assert w4(dev(x), dev(qw), dev(s), dev(z), y, 1, n, k, 128) == N.OK
    got = host(y)
    assert rel_l2(got, O.linear_int4(x, qw, s, z)) <= REL_L2
    assert rel_l2(got, O.linear_int4_f64(x, qw, s, z)) <= REL_L2


def test_bf16_head_qwen3_8b_rtn_workload(cuda):
    """The BF16 LM head of the sweep: W [151936, 4096] ~ N(0, 0.02) rounded to BF16, x ~ N(0, 1)."""
    n, k = 151936, 4096
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(k, device="cuda", generator=g)
    y = torch.empty(n, device="cuda")
    rc = N.lib().fire_b200_linear_dense(x.data_ptr(), w.data_ptr(), N.BF16, 1.0, y.data_ptr(), 1, n, k, 0)
    assert rc == N.OK
    ref = O.linear_bf16(host(x), host(w.view(torch.int16)).view(np.uint16))
    assert rel_l2(host(y), ref) <= REL_L2


@pytest.mark.skipif(not O.ref_available(), reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("n,k", [(4096, 4096), (1024, 4096), (12288, 4096), (4096, 12288), (3072, 1024)])
def test_w4_matches_reference_cuda_gemv(cuda, n, k):
    """Against Fire's own GEMV_int4_v1 (src/op/kernels/cuda/matmul_kernel.cu:230-267) on the GPU."""
    rng = np.random.default_rng(n + k)
    qw, s, z = random_w4(rng, n, k)
    x = rng.normal(0, 1, k).astype(np.float32)
    dx, dq, ds, dz = dev(x), dev(qw), dev(s), dev(z)
    y = torch.empty(n, device="cuda")
    yr = torch.empty(n, device="cuda")
    assert w4(dx, dq, ds, dz, y, 1, n, k, 128) == N.OK
    O.ref().ref_matmul_quant_cu(dx.data_ptr(), dq.data_ptr(), ds.data_ptr(), dz.data_ptr(), yr.data_ptr(),
                                1, n, k, 128, None)
    assert rel_l2(host(y), host(yr)) <= REL_L2


@pytest.mark.parametrize("K,group,matrix,in_off,w_off", [
    (128, 128, False, 0, 0), (384, 128, True, 0, 0), (4096, 128, False, 0, 0), (12288, 128, True, 0, 0),
    (384, 128, False, 1, 0), (384, 128, True, 0, 1), (258, 3, False, 0, 0)])
def test_w4_boundaries_guard_cells(cuda, K, group, matrix, in_off, w_off):
    """test/test_op/test_matmul.cpp:476-583: M=7 (inactive tail), misaligned views, odd group,
    guard cells around the output that must keep 321.25."""
    from tests.test_oracle_golden import boundary_case
    x, w, s, z, exp = boundary_case(K, group)
    M = 7
    xs = torch.zeros(K + in_off, device="cuda")
    xs[in_off:] = dev(x)
    ws = torch.zeros(M * K // 2 + w_off, dtype=torch.uint8, device="cuda")
    ws[w_off:] = dev(w.reshape(-1))
    out = torch.full((M + 2,), 321.25, device="cuda")
    xv, wv, ov = xs[in_off:], ws[w_off:], out[1:1 + M]
    assert w4(xv, wv, dev(s), dev(z), ov, 1, M, K, group) == N.OK
    got = host(out)
    assert got[0] == 321.25 and got[-1] == 321.25
    assert np.all(np.abs(got[1:1 + M] - exp) <= 2e-4 + 2e-5 * np.abs(exp))


def test_w4_multi_row_matches_cpu_fp32(cuda):
    """test/test_op/test_matmul.cpp:378-474: M=19, K=256, rows 1 and 17, tolerance 1e-3."""
    K, M, g = 256, 19, 128
    G = K // g
    packed = np.zeros((M, K // 2), np.uint8)
    s = np.zeros((M, G), np.float32)
    z = np.zeros((M, G), np.uint8)
    for m in range(M):
        for gg in range(G):
            s[m, gg] = 0.125 * (1 + (m + gg) % 3)
            z[m, gg] = 4 + (m + 2 * gg) % 8
        for k in range(K):
            q = (m * 7 + k * 3 + (k // g) * 5) % 16
            packed[m, k // 2] |= q << ((k % 2) * 4)
    for rows in (1, 17):
        x = np.array([[0.125 * ((n * 5 + k * 7) % 17 - 8) for k in range(K)] for n in range(rows)], np.float32)
        y = torch.empty((rows, M), device="cuda")
        assert w4(dev(x), dev(packed), dev(s), dev(z), y, rows, M, K, g) == N.OK
        ref = O.linear_int4(x, packed, s, z, g)
        assert np.all(np.abs(host(y) - ref) <= 1e-3)


def test_w4_linear_op_interface(cuda):
    """LinearOp.forward with an Int4GroupWise Parameter (src/op/linear.cpp:11-36)."""
    rng = np.random.default_rng(11)
    qw, s, z = random_w4(rng, 256, 512)
    x = rng.normal(0, 1, 512).astype(np.float32)
    op = ops.LinearOp()
    op.reset_param_size(1)
    op.set_param(0, ops.Parameter(dev(qw), ops.QuantConfig(ops.QuantType.Int4GroupWise, 128, False), dev(s), dev(z)))
    y = torch.empty(256, device="cuda")
    ctx = ops.OpContext(ops.DeviceType.GPU, torch.cuda.Stream())
    assert op.forward(dev(x), y, ctx).ok()
    torch.cuda.synchronize()
    assert rel_l2(host(y), O.linear_int4(x, qw, s, z)) <= REL_L2
    bad = ops.OpContext(ops.DeviceType.CPU)
    assert op.forward(dev(x), y, bad).code == ops.StatusCode.InvalidArgument
    assert op.forward(dev(x[:256]), y, ctx).code == ops.StatusCode.InvalidArgument


# ------------------------------------------------------------- dense GEMV ----

def dense(x, w, dt, scale, y, rows, n, k):
    return N.lib().fire_b200_linear_dense(x.data_ptr(), w.data_ptr(), dt, scale, y.data_ptr(), rows, n, k, 0)


@pytest.mark.parametrize("K", [1, 4, 37, 128, 132, 4096, 12288, 4097])
@pytest.mark.parametrize("bf16", [True, False])
def test_dense_gemv_k_sweep_guard_cells(cuda, K, bf16):
    """test/test_op/test_matmul.cpp:267-376: K sweep, guard cells, 2e-4 + 2e-5|y|."""
    rng = np.random.default_rng(K)
    M = 7
    x = rng.normal(0, 1, K).astype(np.float32)
    wf = rng.normal(0, 0.05, (M, K)).astype(np.float32)
    if bf16:
        bits = (wf.view(np.uint32) >> 16).astype(np.uint16)
        wd = dev(bits).view(torch.bfloat16)
        ref = O.linear_bf16(x, bits)
    else:
        wd = dev(wf)
        ref = O.linear_f32(x, wf)
    out = torch.full((M + 2,), 321.25, device="cuda")
    assert dense(dev(x), wd, N.BF16 if bf16 else N.F32, 1.0, out[1:1 + M], 1, M, K) == N.OK
    got = host(out)
    assert got[0] == 321.25 and got[-1] == 321.25
    assert np.all(np.abs(got[1:1 + M] - ref) <= 2e-4 + 2e-5 * np.abs(ref))


def test_dense_misaligned_views_and_rows(cuda):
    rng = np.random.default_rng(5)
    K, M = 132, 9
    x = rng.normal(0, 1, (3, K)).astype(np.float32)
    wf = rng.normal(0, 0.05, (M, K)).astype(np.float32)
    bits = (wf.view(np.uint32) >> 16).astype(np.uint16)
    wst = torch.zeros(M * K + 1, dtype=torch.int16, device="cuda")
    wst[1:] = dev(bits.view(np.int16).reshape(-1))
    xs = torch.zeros(3 * K + 1, device="cuda")
    xs[1:] = dev(x.reshape(-1))
    y = torch.empty((3, M), device="cuda")
    assert dense(xs[1:], wst[1:], N.BF16, 0.5, y, 3, M, K) == N.OK
    ref = O.linear_bf16(x, bits, 0.5)
    assert np.all(np.abs(host(y) - ref) <= 2e-4 + 2e-5 * np.abs(ref))


def test_lm_head_bf16_shape(cuda):
    rng = np.random.default_rng(151936)
    n, k = 151936, 4096
    bits = rng.integers(0, 2 ** 16, (n, k), dtype=np.uint16)
    bits = (bits & 0x3FFF) | 0x3C00  # finite, moderate magnitudes, both signs via bit 15 below
    bits[:, ::2] |= 0x8000
    x = rng.normal(0, 1, k).astype(np.float32)
    y = torch.empty(n, device="cuda")
    assert dense(dev(x), dev(bits.view(np.int16)), N.BF16, 1.0, y, 1, n, k) == N.OK
    ref = O.linear_bf16(x, bits)
    assert rel_l2(host(y), ref) <= REL_L2


# ------------------------------------------------------------ norms / RoPE ----

@pytest.mark.parametrize("size", [1, 5, 513, 1024, 4096, 16384, 40000])
def test_rmsnorm_vs_oracle(cuda, size):
    rng = np.random.default_rng(size)
    x = rng.normal(0, 2, size).astype(np.float32)
    w = (0.75 + (np.arange(size) % 11) * 0.03125).astype(np.float32)
    y = torch.empty(size, device="cuda")
    op = ops.RmsNormOp(1e-6)
    op.reset_param_size(1)
    op.set_param(0, dev(w))
    assert op.forward(dev(x), y, ops.OpContext(ops.DeviceType.GPU)).ok()
    assert np.allclose(host(y), O.rmsnorm(x, w, 1e-6), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("rows,width", [(3, 5), (32, 128), (8, 128), (16, 1026)])
def test_rmsnorm_rows_vs_oracle(cuda, rows, width):
    rng = np.random.default_rng(rows * width)
    x = rng.normal(0, 3, (rows, width)).astype(np.float32)
    w = rng.normal(1, 0.1, width).astype(np.float32)
    y = torch.empty((rows, width), device="cuda")
    op = ops.RmsNormOp(1e-4)
    op.reset_param_size(1)
    op.set_param(0, dev(w))
    assert op.forward(dev(x), y, ops.OpContext(ops.DeviceType.GPU)).ok()
    assert np.allclose(host(y), O.rmsnorm_rows(x, w, 1e-4), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("head,max_seq,qh,kh,theta", [(2, 1, 1, 1, 1e4), (6, 7, 3, 1, 1e4), (64, 17, 4, 2, 1e4),
                                                       (1026, 9, 3, 2, 1e4), (64, 2048, 4, 2, 1e4),
                                                       (128, 2048, 32, 8, 1e6)])
def test_rope_cache_and_rotation(cuda, head, max_seq, qh, kh, theta):
    """test/test_op/test_rope.cpp: cache vs formula (2e-6 + pos*1e-7), rotation vs oracle."""
    sin = torch.full((max_seq, head // 2), float("nan"), device="cuda")
    cos = torch.full((max_seq, head // 2), float("nan"), device="cuda")
    ops.rope_cache(head, max_seq, theta, sin, cos)
    s_ref, c_ref = O.rope_cache(head, max_seq, theta)
    s, c = host(sin), host(cos)
    pos = np.arange(max_seq)[:, None]
    tol = 2e-6 + pos * 1e-7
    ang = pos * np.power(np.float64(theta), -2.0 * np.arange(head // 2)[None, :] / head)
    assert np.all(np.abs(s - np.sin(ang)) <= tol) and np.all(np.abs(c - np.cos(ang)) <= tol)
    # against the oracle (glibc powf/sinf/cosf) within the same bound
    assert np.all(np.abs(s - s_ref) <= tol) and np.all(np.abs(c - c_ref) <= tol)
    rng = np.random.default_rng(head)
    q = rng.normal(0, 1, (qh, head)).astype(np.float32)
    k = rng.normal(0, 1, (kh, head)).astype(np.float32)
    for p in (max_seq - 1, 0):
        dq, dk = dev(q), dev(k)
        assert ops.RoPEOp().forward(dq, dk, cos, sin, p, ops.OpContext(ops.DeviceType.GPU)).ok()
        qr, kr = O.rope(q, k, c, s, p)  # same cache -> bit-exact rotation
        assert np.array_equal(host(dq), qr) and np.array_equal(host(dk), kr)


# -------------------------------------------------------------- attention ----

@pytest.mark.parametrize("shape,layer,pos", [((2, 5, 4, 2, 3), 1, 3), ((2, 257, 4, 2, 5), 1, 256),
                                             ((1, 2048, 32, 8, 128), 0, 2047), ((3, 300, 16, 8, 128), 2, 129),
                                             ((2, 384, 16, 8, 128), 1, 0), ((1, 100, 32, 4, 64), 0, 63)])
def test_mha_vs_oracle(cuda, shape, layer, pos):
    """test/test_op/test_mha.cpp:204-215: score within 2e-5, output within 3e-5, tail untouched."""
    layers, cap, qh, kvh, hd = shape

    def vals(size, mul, off, scale):
        i = np.arange(size)
        return ((((i * mul + off) % 31).astype(np.int64) - 15) * scale).astype(np.float32)

    q = vals(qh * hd, 7, 3, 0.125).reshape(qh, hd)
    kc = vals(layers * cap * kvh * hd, 11, 5, 0.0625).reshape(layers, cap, kvh, hd)
    vc = vals(layers * cap * kvh * hd, 13, 9, 0.1875).reshape(layers, cap, kvh, hd)
    out_ref, score_ref = O.mha(q, kc, vc, layer, pos)
    score = torch.full((qh, cap), -777.0, device="cuda")
    out = torch.empty((qh, hd), device="cuda")
    dq, dk, dv = dev(q), dev(kc), dev(vc)
    ctx = ops.OpContext(ops.DeviceType.GPU, torch.cuda.Stream())
    op = ops.MultiHeadAttentionOp()
    for _ in range(2):  # second call reuses the (self-cleaning) workspace
        assert op.forward(dq, dk, dv, score, out, layer, pos, ctx).ok()
        torch.cuda.synchronize()
        sc = host(score)
        assert np.all(np.abs(sc[:, :pos + 1] - score_ref[:, :pos + 1]) <= 2e-5)
        assert np.all(sc[:, pos + 1:] == -777.0)
        assert np.all(np.abs(sc[:, :pos + 1].sum(1) - 1.0) <= 3e-5)
        assert np.all(np.abs(host(out) - out_ref) <= 3e-5)
    assert np.array_equal(host(dk), kc) and np.array_equal(host(dq), q)


# ------------------------------------------------------ embedding / misc ----

def test_embedding_bf16_bits_and_fp32(cuda):
    bits = np.array([0x0000, 0x8000, 0x3F80, 0xC020, 0x3F81, 0x3380, 0x7180, 0xBF00], np.uint16)
    vals = np.array([0.0, -0.0, 1.0, -2.5, 1.0078125, 2.0 ** -24, 2.0 ** 100, -0.5], np.float32)
    for dim in (1, 5, 257):
        vocab = 6
        table = bits[np.arange(vocab * dim) % 8].reshape(vocab, dim)
        ref_t = vals[np.arange(vocab * dim) % 8].reshape(vocab, dim)
        for toks in ([4], [3, 0, 5, 3]):
            t = dev(np.array(toks, np.int32))
            out = torch.empty((len(toks), dim), device="cuda")
            op = ops.EmbeddingOp()
            op.reset_param_size(1)
            op.set_param(0, dev(table.view(np.int16)).view(torch.bfloat16))
            assert op.forward(t, out, ops.OpContext(ops.DeviceType.GPU)).ok()
            got = host(out)
            assert np.array_equal(got, ref_t[toks]) and np.array_equal(np.signbit(got), np.signbit(ref_t[toks]))
    tab = np.arange(5 * 3, dtype=np.float32).reshape(5, 3) + 0.25
    out = torch.empty((3, 3), device="cuda")
    op = ops.EmbeddingOp()
    op.reset_param_size(1)
    op.set_param(0, dev(tab))
    assert op.forward(dev(np.array([3, 0, 4], np.int32)), out, ops.OpContext(ops.DeviceType.GPU)).ok()
    assert np.array_equal(host(out), tab[[3, 0, 4]])


@pytest.mark.parametrize("n", [1, 255, 256, 257, 1025])
def test_swiglu_and_add(cuda, n):
    i = np.arange(n)
    g = ((i % 17) - 8).astype(np.float32) * 0.375
    u = ((i % 11) - 5).astype(np.float32) * 0.25
    out = torch.empty(n, device="cuda")
    ctx = ops.OpContext(ops.DeviceType.GPU, torch.cuda.Stream())
    assert ops.SwiGLUOp().forward(dev(g), dev(u), out, ctx).ok()
    torch.cuda.synchronize()
    assert np.all(np.abs(host(out) - O.swiglu(g, u)) <= 1e-6)
    assert ops.VecAddOp().forward(dev(g), dev(u), out, ctx).ok()
    torch.cuda.synchronize()
    assert np.array_equal(host(out), O.add(g, u))


@pytest.mark.parametrize("n", [1, 7, 1000, 151936, 1 << 20])
def test_argmax_first_index_on_ties(cuda, n):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 1, n).astype(np.float32)
    if n > 10:
        m = x.max() + 1
        x[[n // 3, n // 2, n - 1]] = m  # ties: smallest index wins
    ws = torch.zeros(N.lib().fire_b200_argmax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    for _ in range(3):
        idx = ops.argmax(dev(x), workspace=ws)
        assert int(idx.item()) == O.argmax(x)
