"""CPU: pin the oracle and the data tools against the reference's own outputs.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py from the
reference itself (its Python tools and its CPU kernels compiled from source).
"""
import hashlib
import json
import os

import numpy as np
import pytest

from fire_b200 import fire_format, quant, synth
from fire_b200.profiles import Qwen3Profile
from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
META = json.load(open(os.path.join(GOLD, "golden.json")))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ----------------------------------------------------------- oracle vs ref CPU ----

@pytest.fixture(scope="module")
def refk():
    return np.load(os.path.join(GOLD, "ref_cpu_kernels.npz"))


def test_oracle_rmsnorm_bit_exact_vs_reference_cpu(refk):
    assert np.array_equal(O.rmsnorm(refk["rms_x"], refk["rms_w"], 1e-6), refk["rms_y"])
    assert np.array_equal(O.rmsnorm_rows(refk["rmsr_x"], refk["rmsr_w"], 1e-6), refk["rmsr_y"])


def test_oracle_rope_bit_exact_vs_reference_cpu(refk):
    s, c = O.rope_cache(128, 2048, 1e6)
    assert sha(s) == str(refk["rope_sin_sha"]) and sha(c) == str(refk["rope_cos_sha"])
    rows = refk["rope_rows"]
    assert np.array_equal(s[rows], refk["rope_sin_rows"])
    q, k = O.rope(refk["rope_q"], refk["rope_k"], c, s, 1791)
    assert np.array_equal(q, refk["rope_q_out"]) and np.array_equal(k, refk["rope_k_out"])


def test_oracle_mha_bit_exact_vs_reference_cpu(refk):
    out, score = O.mha(refk["mha_q"], refk["mha_kc"], refk["mha_vc"], layer=1, pos=257)
    assert np.array_equal(out, refk["mha_out"])
    assert np.array_equal(score, refk["mha_score"])  # includes the untouched -777 tail


# ------------------------------------------------------------------ quant KATs ----

def test_nibble_order_and_zero_group_kat():
    v = np.array(META["nibble_order"]["values"], np.uint8)
    assert quant.pack_uint4(v).tolist() == META["nibble_order"]["packed"] == [[0x21, 0x0F]]
    q, s, z = quant.quantize_int4_groupwise(np.zeros((1, 128), np.float32), 128)
    assert s.tolist() == META["zero_group"]["scales"] == [[1.0]]
    assert z.tolist() == META["zero_group"]["zeros"] == [[0]]
    assert quant.pack_uint4(q).tolist() == META["zero_group"]["packed"]


def test_rtn_quantiser_matches_reference_tools_bit_exact():
    g = np.load(os.path.join(GOLD, "rtn_small.npz"))
    q, s, z = quant.quantize_int4_groupwise(g["w"], 128)
    assert np.array_equal(q, g["q"]) and np.array_equal(s, g["scales"]) and np.array_equal(z, g["zeros"])
    p = quant.pack_uint4(q)
    assert np.array_equal(p, g["packed"])
    assert np.array_equal(quant.unpack_uint4(p), g["q"])
    assert np.array_equal(quant.dequantize_int4_groupwise(p, s, z, 128), g["dequant"])
    # the oracle's element-wise dequantisation is the same FP32 value
    assert np.array_equal(O.dequant_int4(p, s, z, 128), g["dequant"])


def test_single_linear_workload_pinned():
    """W 3072x1024 ~ N(0,0.02) seed 0 -> RTN -> x ~ N(0,1): hashes from the reference tools."""
    meta = META["linear_3072x1024"]
    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (3072, 1024)).astype(np.float32)
    x = rng.normal(0, 1, (1, 1024)).astype(np.float32)
    assert sha(W) == meta["sha_W"] and sha(x) == meta["sha_x"]
    q, s, z = quant.quantize_int4_groupwise(W, 128)
    p = quant.pack_uint4(q)
    assert (sha(p), sha(s), sha(z)) == (meta["sha_packed"], meta["sha_scales"], meta["sha_zeros"])
    y = O.linear_int4(x[0], p, s, z, 128)
    ref = np.load(os.path.join(GOLD, "linear_3072x1024.npz"))["y_f64"]
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 1e-6, rel


def test_awq_gemm_unpack_matches_reference_exporter():
    g = np.load(os.path.join(GOLD, "awq_unpack.npz"))
    u = quant.unpack_awq_gemm(g["words"])
    assert np.array_equal(u, g["unpacked"])
    assert np.array_equal(quant.pack_uint4(u), g["packed"])
    # test/test_model/test_export_qwen3.py:652-654 golden bytes: column 0 is q[k, out]=(k+out)%16
    p = g["packed"]
    assert (p[0, 0], p[1, 0], p[0, 4]) == (0x10, 0x21, 0x98)


def test_bf16_bit_patterns_widen_exactly():
    # test/test_op/test_emb.cpp:280-283
    bits = np.array([0x0000, 0x8000, 0x3F80, 0xC020, 0x3F81, 0x3380, 0x7180, 0xBF00], np.uint16)
    vals = np.array([0.0, -0.0, 1.0, -2.5, 1.0078125, 2.0 ** -24, 2.0 ** 100, -0.5], np.float32)
    got = O.embedding(np.arange(8, dtype=np.int32), bits.reshape(8, 1))[:, 0]
    assert np.array_equal(got, vals) and np.array_equal(np.signbit(got), np.signbit(vals))


# ------------------------------------------------------------ .fire container ----

MICRO = Qwen3Profile("micro", 32, 64, 128, 128, 1, 1, 1, 128)


@pytest.mark.parametrize("layout", ["int4", "mixed"])
def test_fire_writer_matches_reference_writer_bytes(tmp_path, layout):
    weights = synth.generate(MICRO, layout, seed=7)
    path = tmp_path / "m.fire"
    fire_format.write(str(path), synth.container_entries(weights), version=2)
    gold = open(os.path.join(GOLD, f"micro_{layout}.fire"), "rb").read()
    assert path.read_bytes() == gold
    assert hashlib.sha256(gold).hexdigest() == META[f"micro_{layout}"]["sha"]
    f = fire_format.FireFile(str(path))
    assert len(f) == META[f"micro_{layout}"]["count"]
    for name, arr in weights.items():
        assert np.array_equal(f.array(name), arr)
    assert f.records["layers.0.attention.wq.qweight"].group_size == 128


def test_fire_reader_rejects_malformed(tmp_path):
    weights = synth.generate(MICRO, "int4", seed=7)
    path = tmp_path / "m.fire"
    fire_format.write(str(path), synth.container_entries(weights), version=2)
    raw = bytearray(path.read_bytes())
    bad = tmp_path / "bad.fire"
    for mutate in (lambda b: b.__setitem__(0, ord("X")),           # magic
                   lambda b: b.__setitem__(8, 3),                   # version
                   lambda b: b.__setitem__(32 + 64, b[32 + 64] + 1)):  # payload offset
        b = bytearray(raw)
        mutate(b)
        bad.write_bytes(bytes(b))
        with pytest.raises(fire_format.FireFormatError):
            fire_format.FireFile(str(bad))
    bad.write_bytes(bytes(raw[:-1]))  # truncated payload
    with pytest.raises(fire_format.FireFormatError):
        fire_format.FireFile(str(bad))


def test_tensor_counts_match_loader_rules():
    """Qwen3Loader::load_weights (src/model/qwen_loader.cpp:129-136) tensor counts."""
    p = MICRO
    assert len(synth.generate(p, "int4")) == p.tensor_count + 2 * (p.num_layers * 7 + 1)
    assert len(synth.generate(p, "mixed")) == p.tensor_count + 2 * p.num_layers * 7


# ------------------------------------------------ oracle vs formula references ----

def boundary_case(K, group, M=7):
    """test/test_op/test_matmul.cpp:476-583 formula inputs and double-precision expectations."""
    G = K // group
    x = (0.0314159 * (((np.arange(K) * 7) % 43) - 21)).astype(np.float32)
    w = np.zeros((M, K // 2), np.uint8)
    s = np.zeros((M, G), np.float32)
    z = np.zeros((M, G), np.uint8)
    exp = np.zeros(M)
    for m in range(M):
        for g in range(G):
            s[m, g] = np.float32(0.006172839) * np.float32(1 + (m * 5 + g * 3) % 11)
            z[m, g] = (m + g * 5) % 16
        for k in range(K):
            q = (m * 11 + k * 7 + (k // 2) * 3) % 16
            w[m, k // 2] |= q << (4 * (k % 2))
            wt = np.float32(q - int(z[m, k // group])) * s[m, k // group]
            exp[m] += float(x[k]) * float(wt)
    return x, w, s, z, exp


@pytest.mark.parametrize("K,group", [(128, 128), (384, 128), (4096, 128), (258, 3)])
def test_oracle_int4_boundary_cases(K, group):
    x, w, s, z, exp = boundary_case(K, group)
    y = O.linear_int4(x, w, s, z, group)
    assert np.all(np.abs(y - exp) <= 2e-4 + 2e-5 * np.abs(exp))


def test_oracle_qwen3_forward_runs_and_resets():
    from fire_b200.profiles import TINY
    w = synth.generate(TINY, "int4", seed=3)
    m = O.Qwen3Oracle(TINY, w, capacity=8)
    a = [m.forward(t, i) for i, t in enumerate([5, 17, 999])]
    assert all(np.isfinite(l).all() for l in a)
    m.reset()
    b = [m.forward(t, i) for i, t in enumerate([5, 17, 999])]
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    with pytest.raises(ValueError):
        m.forward(1, 7)


@pytest.mark.parametrize("n,k,group", [(7, 258, 3), (19, 256, 128), (33, 1024, 128), (13, 132, 4),
                                       (1027, 4096, 128), (9, 12288, 128)])
def test_oracle_row_blocked_int4_equals_one_row_loops(n, k, group):
    """The oracle's INT4 Linear runs eight rows in vector lanes; each row must still sum in
    the reference's sequential order, so it equals the one-row loop bit for bit."""
    import ctypes as C
    rng = np.random.default_rng(n + k)
    q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    s = rng.random((n, k // group), dtype=np.float32) * 0.02
    z = rng.integers(0, 16, (n, k // group), dtype=np.uint8)
    x = rng.standard_normal((2, k), dtype=np.float32)
    L = O.lib()
    L.fo_linear_int4_scalar.argtypes = [O._f32p, O._u8p, O._f32p, O._u8p, O._f32p, C.c_int64, C.c_int64,
                                        C.c_int64, C.c_int]
    want = np.empty((2, n), np.float32)
    L.fo_linear_int4_scalar(x, q, s, z, want, 2, n, k, group)
    got = O.linear_int4(x, q, s, z, group)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n,k", [(33, 37), (1000, 4096), (17, 2)])
def test_oracle_row_blocked_dense_equals_one_row_loops(n, k):
    import ctypes as C
    rng = np.random.default_rng(n * k)
    x = rng.standard_normal((1, k), dtype=np.float32)
    wf = rng.standard_normal((n, k), dtype=np.float32)
    wb = (wf.view(np.uint32) >> 16).astype(np.uint16)
    L = O.lib()
    L.fo_linear_bf16_scalar.argtypes = [O._f32p, O._u16p, C.c_float, O._f32p, C.c_int64, C.c_int64, C.c_int64]
    L.fo_linear_f32_scalar.argtypes = [O._f32p, O._f32p, C.c_float, O._f32p, C.c_int64, C.c_int64, C.c_int64]
    want = np.empty((1, n), np.float32)
    L.fo_linear_bf16_scalar(x, wb, 1.0, want, 1, n, k)
    assert np.array_equal(O.linear_bf16(x, wb).view(np.uint32), want.view(np.uint32))
    L.fo_linear_f32_scalar(x, wf, 0.5, want, 1, n, k)
    assert np.array_equal(O.linear_f32(x, wf, 0.5).view(np.uint32), want.view(np.uint32))
