"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference source tree (default /root/reference,
override with FIRE_REFERENCE) and the built oracle/_ref library:

    make -C oracle all ref && python tests/golden/make_golden.py

It imports the reference's own Python tools (tools/quant.py, tools/fire_writer.py,
tools/export_qwen3.py) and calls the reference's own compiled CPU kernels
(oracle/_ref/libfire_ref.so, built from src/op/kernels/cpu/*.cpp) on seeded inputs,
and saves inputs + outputs. The tests read only the saved files, so they need
neither the reference tree nor oracle/_ref at run time.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("FIRE_REFERENCE", "/root/reference")
sys.path.insert(0, os.path.join(REF, "tools"))
sys.path.insert(0, ROOT)

import quant as ref_quant  # noqa: E402  (reference tools/quant.py)
import fire_writer as ref_writer  # noqa: E402  (reference tools/fire_writer.py)

from oracle import oracle as O  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def quant_fixtures(meta: dict) -> None:
    # tools/quant.py contract (test/test_model/test_quant.py:22-40)
    meta["nibble_order"] = {"values": [[1, 2, 15, 0]],
                            "packed": ref_quant.pack_uint4(
                                np.array([[1, 2, 15, 0]], np.uint8)).tolist()}
    q, s, z = ref_quant.quantize_int4_groupwise(np.zeros((1, 128), np.float32), group_size=128)
    meta["zero_group"] = {"scales": s.tolist(), "zeros": z.tolist(),
                          "packed": ref_quant.pack_uint4(q).tolist()}

    # Small seeded matrix: full arrays (ties, negative/positive-only groups, a zero group).
    rng = np.random.default_rng(1234)
    w = rng.normal(0, 0.02, (48, 512)).astype(np.float32)
    w[3, 128:256] = 0.0                       # all-zero group
    w[5, :128] = np.abs(w[5, :128])           # positive-only group
    w[6, 256:384] = -np.abs(w[6, 256:384])    # negative-only group
    q, s, z = ref_quant.quantize_int4_groupwise(w, group_size=128)
    packed = ref_quant.pack_uint4(q)
    deq = ref_quant.dequantize_int4_groupwise(packed, s, z, group_size=128)
    np.savez_compressed(os.path.join(HERE, "rtn_small.npz"), w=w, q=q, scales=s, zeros=z,
                        packed=packed, dequant=deq)

    # The single-Linear workload: W 3072x1024 ~ N(0,0.02) seed 0, then x ~ N(0,1) [1,1024].
    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (3072, 1024)).astype(np.float32)
    x = rng.normal(0, 1, (1, 1024)).astype(np.float32)
    q, s, z = ref_quant.quantize_int4_groupwise(W, group_size=128)
    packed = ref_quant.pack_uint4(q)
    deq = ref_quant.dequantize_int4_groupwise(packed, s, z, group_size=128)
    y64 = (deq.astype(np.float64) @ x[0].astype(np.float64))
    meta["linear_3072x1024"] = {"sha_W": sha(W), "sha_x": sha(x), "sha_packed": sha(packed),
                                "sha_scales": sha(s), "sha_zeros": sha(z), "sha_dequant": sha(deq)}
    np.savez_compressed(os.path.join(HERE, "linear_3072x1024.npz"), y_f64=y64,
                        packed_rows0_7=packed[:8], scales_rows0_7=s[:8], zeros_rows0_7=z[:8])


def writer_fixtures(meta: dict) -> None:
    """Tiny checkpoints written by the reference FireWriter (v2 int4 + mixed, v1 fp32)."""
    from fire_b200 import synth
    from fire_b200.profiles import Qwen3Profile

    micro = Qwen3Profile("micro", 32, 64, 128, 128, 1, 1, 1, 128)
    for layout in ("int4", "mixed"):
        weights = synth.generate(micro, layout, seed=7)
        infos, off = [], 32 + 96 * len(weights)
        for name, arr in weights.items():
            dt = {np.dtype(np.float32): ref_writer.WireDType.FP32,
                  np.dtype(np.uint8): ref_writer.WireDType.UINT8,
                  np.dtype(np.uint16): ref_writer.WireDType.BF16}[arr.dtype]
            off = (off + 3) & ~3
            qi = ref_writer.QuantizationInfo(128) if name.endswith(".qweight") else None
            infos.append(ref_writer.TensorInfo(name, dt, tuple(arr.shape), off, arr.nbytes, qi))
            off += arr.nbytes
        path = os.path.join(HERE, f"micro_{layout}.fire")
        w = ref_writer.FireWriter(version=2)
        with open(path, "wb") as f:
            w.write_header_and_directory(f, infos)
            for info, arr in zip(infos, weights.values()):
                w.write_tensor(f, info, np.ascontiguousarray(arr))
        meta[f"micro_{layout}"] = {"sha": hashlib.sha256(open(path, "rb").read()).hexdigest(),
                                   "count": len(infos)}


def awq_fixture(meta: dict) -> None:
    import export_qwen3 as ref_export  # reference tools/export_qwen3.py

    # Same construction as test/test_model/test_export_qwen3.py:567-600, plus random words.
    awq_order = (0, 2, 4, 6, 1, 3, 5, 7)
    words = np.zeros((128, 2), np.uint32)
    for k in range(128):
        vals = [(k + out) % 16 for out in range(8)]
        words[k, 0] = sum(vals[out] << (4 * i) for i, out in enumerate(awq_order))
    words[:, 1] = np.random.default_rng(5).integers(0, 2**32, 128, dtype=np.uint64)
    unpacked = ref_export._unpack_awq_gemm(words.view(np.int32))
    np.savez_compressed(os.path.join(HERE, "awq_unpack.npz"), words=words, unpacked=unpacked,
                        packed=ref_quant.pack_uint4(unpacked))


def ref_cpu_kernel_fixtures() -> None:
    """Outputs of the reference's own CPU kernels (oracle/_ref) on seeded inputs."""
    R = O.ref()
    rng = np.random.default_rng(2024)
    out = {}
    x = rng.normal(0, 1, 4096).astype(np.float32)
    w = rng.normal(1, 0.1, 4096).astype(np.float32)
    y = np.empty_like(x)
    R.ref_rmsnorm_cpu(x, w, y, 1, 4096, 0, 1e-6)
    out.update(rms_x=x, rms_w=w, rms_y=y)
    xr = rng.normal(0, 3, (32, 128)).astype(np.float32)
    wr = rng.normal(1, 0.1, 128).astype(np.float32)
    yr = np.empty_like(xr)
    R.ref_rmsnorm_cpu(xr.reshape(-1), wr, yr.reshape(-1), 32, 128, 1, 1e-6)
    out.update(rmsr_x=xr, rmsr_w=wr, rmsr_y=yr)
    sn = np.empty((2048, 64), np.float32)
    cs = np.empty_like(sn)
    R.ref_rope_cache_cpu(128, 2048, 1e6, sn.reshape(-1), cs.reshape(-1))
    q = rng.normal(0, 1, (32, 128)).astype(np.float32)
    k = rng.normal(0, 1, (8, 128)).astype(np.float32)
    q2, k2 = q.copy(), k.copy()
    R.ref_rope_cpu(q2.reshape(-1), k2.reshape(-1), cs.reshape(-1), sn.reshape(-1), 32, 8, 128,
                   2048, 1791)
    rows = np.array([0, 1, 17, 1791, 2047])
    out.update(rope_rows=rows, rope_sin_rows=sn[rows], rope_cos_rows=cs[rows],
               rope_sin_sha=np.array(sha(sn)), rope_cos_sha=np.array(sha(cs)),
               rope_q=q, rope_k=k, rope_q_out=q2, rope_k_out=k2)
    # GQA 4:1 over a cache past one 256-thread block (pos 257), half-size heads.
    qm = rng.normal(0, 1, (8, 64)).astype(np.float32)
    kc = rng.normal(0, 1, (2, 300, 2, 64)).astype(np.float32)
    vc = rng.normal(0, 1, (2, 300, 2, 64)).astype(np.float32)
    score = np.full((8, 300), -777.0, np.float32)
    o = np.empty((8, 64), np.float32)
    R.ref_mha_cpu(qm.reshape(-1), kc.reshape(-1), vc.reshape(-1), score.reshape(-1),
                  o.reshape(-1), 2, 300, 8, 2, 64, 1, 257)
    out.update(mha_q=qm)
    out.update(mha_kc=kc, mha_vc=vc, mha_score=score, mha_out=o)
    np.savez_compressed(os.path.join(HERE, "ref_cpu_kernels.npz"), **out)


def main() -> None:
    meta: dict = {"generated_from": "reference tools/ and src/op/kernels/cpu (compiled)"}
    quant_fixtures(meta)
    writer_fixtures(meta)
    awq_fixture(meta)
    ref_cpu_kernel_fixtures()
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
