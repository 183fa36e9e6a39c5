#!/usr/bin/env python
"""Qwen3-8B W4 single-token decode throughput on B200 (tok/s), tensor parallel over --gpus N.

Workload (the metric's configuration): Qwen3-8B architecture (36 layers, hidden 4096,
32 q / 8 kv heads, head_dim 128, FFN 12288, vocab 151936), random-init weights in the
AWQ-style mixed layout (INT4 group-128 projections with FP16-valued scales and 4-bit
zeros, BF16 embedding and LM head, FP32 norms), FP32 activations and KV cache. A
1792-token prompt of uniform ids is prefilled once; one *step* is a 256-token greedy
decode from the end of the prompt, ending at context 2048.

  value  = device-resident greedy loop (token ids and positions stay on the GPU; the
           step is one CUDA graph per token) -> tokens/s
  e2e    = the reference's host loop through the C ABI (per token: H2D of the input id
           from pinned memory, one step, D2H of the sampled id, stream synchronise)
  roofline = the dominant kernel, timed live: at TP1 the persistent layer-stack kernel
           (all 36 layers in one launch; bytes = INT4 weights + scales/zeros + the FP32
           K/V rows it reads + norms), under tensor parallelism the INT4 GEMV on the
           decode shapes

  parity = the engine's KV prefix (positions 0..1790 after the prefill) is exported into
           the oracle (the FP32 CPU restatement of Qwen3Model::forward, oracle/), which then
           decodes the same 256 steps fed the GPU's tokens: every sampled id must equal the
           oracle's argmax, and the logits of the first steps are compared (rel-L2, max |d|)
  gemv_sweep = the INT4 group-128 GEMV at M=1 on every Qwen3-8B projection shape and the
           BF16 LM head (seed-0 RTN N(0,0.02) weights, FP16-valued scales), working sets
           larger than L2, GB/s against the measured HBM peak; plus the 3072x1024 single
           Linear (L2-resident, microseconds) beside the CPU FP32 Linear on the dequantised
           weights

`--impl reference` times the CPU restatement of the same decode (oracle/, FP32 on the
host cores) on a bounded sample of the workload (see `cpu_baseline.sample`).
`--gemv` runs only the GEMV sweep (it sizes the ncu captures of the GEMV kernels).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PROMPT = 1792
GEN = 256
CAPACITY = 2048
METRIC = "Qwen3-8B W4 decode tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="fire_b200", choices=["fire_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # profiling knobs (defaults are the measured workload)
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens prefilled once")
    ap.add_argument("--gen", type=int, default=GEN, help="greedy tokens per step")
    ap.add_argument("--prefill", action="store_true",
                    help="only the M=512 INT4 prefill GEMM sweep over the 8B projection shapes")
    ap.add_argument("--gemv", action="store_true",
                    help="only the M=1 INT4 / BF16 GEMV sweep over the 8B decode shapes")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle parity leg")
    ap.add_argument("--gemv-shape", default=None,
                    help="with --gemv: only this shape (q, k, v, o, gate, up, down, qkv_fused, gate_up_fused, "
                         "lm_head), to size an ncu capture")
    ap.add_argument("--trace-phases", action="store_true",
                    help="only the per-phase timeline of one layer-stack launch at position 1791 (GPU timer)")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder layers (0 = the model's 36); fewer only to size an ncu capture")
    return ap.parse_args()


# ------------------------------------------------------------------ helpers ----

def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.out.flush()
        rows = []
        try:
            for line in open(self.out.name):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9 and f[1].replace(".", "").isdigit():
                    rows.append(f)
        except OSError:
            pass
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(float(r[2]) for r in rows),
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3] not in ("", "[N/A]")),
                "reasons": reasons}


# ------------------------------------------------------------ CPU baseline ----

def host_weights(weights_dev):
    """Device checkpoint (torch) -> host numpy arrays in Fire's wire dtypes."""
    import torch

    out = {}
    for k, v in weights_dev.items():
        a = v.cpu()
        if a.dtype == torch.int16:
            out[k] = a.numpy().view(np.uint16)
        else:
            out[k] = a.numpy()
    return out


def workload_config(world: int, n_prompt: int = PROMPT, n_gen: int = GEN, layers: int = 36) -> dict:
    """The measured workload, identical in both arms' lines."""
    return {"workload": "qwen3-8b-w4-decode-ctx2048", "model": "Qwen3-8B (random init)",
            "layout": "mixed: INT4 g128 projections, BF16 embedding/head, FP32 norms/activations/KV",
            "prompt": n_prompt, "generated_per_step": n_gen, "context": n_prompt + n_gen,
            "parallelism": f"tp{world}", "layers": layers,
            "l2": "weights 4.99 GB/token > 126 MB L2 (no flush needed)"}


# ------------------------------------------------------------ reference arm ----

REF_TOKENS_PER_STEP = 4


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    import torch

    from fire_b200 import synth
    from fire_b200.profiles import QWEN3_8B

    torch.manual_seed(0)
    w = synth.generate_torch(QWEN3_8B, "mixed", seed=0, device="cpu")
    wn = host_weights(w)
    del w
    from oracle import oracle as O

    O.set_threads(os.cpu_count() or 1)
    m = O.Qwen3Oracle(QWEN3_8B, wn, capacity=CAPACITY)
    rng = np.random.default_rng(1)
    pos0 = PROMPT - 1
    m.kc[:, :pos0] = rng.standard_normal(m.kc[:, :pos0].shape, dtype=np.float32)
    m.vc[:, :pos0] = rng.standard_normal(m.vc[:, :pos0].shape, dtype=np.float32)
    m.length = pos0
    tok = 1234
    gen = CAPACITY - pos0

    def step(i):
        # REF_TOKENS_PER_STEP greedy tokens; successive steps walk the decode range 1791..2047
        nonlocal tok
        start = (i * REF_TOKENS_PER_STEP) % (gen - REF_TOKENS_PER_STEP)
        m.length = pos0 + start
        for j in range(REF_TOKENS_PER_STEP):
            tok = int(np.argmax(m.forward(tok, m.length)))

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    dt = time.perf_counter() - t0
    val = args.steps * REF_TOKENS_PER_STEP / dt
    cores = O.lib().fo_get_threads()
    line = {"metric": METRIC, "value": val, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": workload_config(world),
            "cpu_baseline": {"value": val, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"a bounded sample of the workload: {REF_TOKENS_PER_STEP} greedy decode "
                                       "tokens per step, successive steps walking positions 1791..2047 (KV prefix "
                                       "N(0,1)); FP32 dequantised INT4 on the fly, all 36 layers + BF16 head; the "
                                       "oracle port, since the reference's CPU Linear needs Armadillo, absent here"},
            "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# -------------------------------------------------------------- our arm ----

def time_w4_gemv(stream, reps: int = 4):
    """Live roofline of the INT4 GEMV on the 8B decode shapes (q/k/v fused, o, gate/up
    fused, down) over 4 layers of distinct weights (416 MB > L2), CUDA-graph replayed."""
    import torch

    from fire_b200 import _native as N

    L = N.lib()
    shapes = [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)]
    mats = []
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    for _ in range(4):
        for n, k in shapes:
            mats.append((n, k, torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device="cuda", generator=g),
                         torch.rand((n, k // 128), device="cuda", generator=g) * 0.02,
                         torch.randint(0, 16, (n, k // 128), dtype=torch.uint8, device="cuda", generator=g)))
    x = torch.randn(12288, device="cuda")
    y = torch.empty(24576, device="cuda")
    by = sum(n * k // 2 + n * (k // 128) * 5 + 4 * k + 4 * n for n, k, *_ in mats)

    def run():
        for n, k, q, s, z in mats:
            rc = L.fire_b200_linear_w4(x.data_ptr(), q.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(), 1, n,
                                       k, 128, stream.cuda_stream)
            assert rc == 0, rc

    with torch.cuda.stream(stream):
        run()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            run()
        for _ in range(2):
            graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    ms = e0.elapsed_time(e1) / reps
    launches = len(mats)
    return by / launches, ms * 1e3 / launches  # bytes per launch, us per launch


GEMV_SHAPES = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
               ("gate", 12288, 4096), ("up", 12288, 4096), ("down", 4096, 12288),
               ("qkv_fused", 6144, 4096), ("gate_up_fused", 24576, 4096)]
L2_BYTES = 126 * 1024 * 1024


def gemv_sweep(reps_min: int = 100, only=None):
    """fire_b200_linear_w4 (M=1, group 128) on every Qwen3-8B projection shape, and
    fire_b200_linear_dense on the BF16 LM head. Weights: W ~ N(0, 0.02) from a seeded
    generator, RTN INT4 (the reference rule), scales rounded to FP16 values; x ~ N(0, 1).
    Each shape is replicated until the copies exceed twice the L2, and the launches cycle
    through the copies (every launch streams its matrix from HBM); >= reps_min launches in
    a CUDA graph, timed with CUDA events. Bytes per launch = N*K/2 + N*K/128*(4+1) + 4K + 4N
    (INT4) or 2*N*K + 4K + 4N (BF16)."""
    import torch

    from fire_b200 import _native as N
    from fire_b200.quant import quantize_torch

    L = N.lib()
    peak = float(peaks().get("hbm_gbs", 6650.0))
    stream = torch.cuda.Stream()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    out = []

    def timed(launch, copies):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for c in range(copies):
                launch(c)
            with torch.cuda.graph(graph, stream=stream):
                for c in range(copies):
                    launch(c)
            for _ in range(3):
                graph.replay()
            reps = max(1, -(-reps_min // copies))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        stream.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (reps * copies), reps * copies

    for name, n, k in GEMV_SHAPES:
        if only is not None and only != name:
            continue
        w = torch.empty(n, k, device="cuda").normal_(0.0, 0.02, generator=gen)
        x = torch.empty(k, device="cuda").normal_(0.0, 1.0, generator=gen)
        q, sc, z = quantize_torch(w, 128)
        del w
        sc = sc.to(torch.float16).to(torch.float32)
        by = n * k // 2 + n * (k // 128) * 5 + 4 * k + 4 * n
        copies = max(1, -(-2 * L2_BYTES // by))
        mats = [(q.clone(), sc.clone(), z.clone()) for _ in range(copies)]
        y = torch.empty(n, device="cuda")

        def launch(c, mats=mats, x=x, y=y, n=n, k=k):
            qq, ss, zz = mats[c]
            rc = L.fire_b200_linear_w4(x.data_ptr(), qq.data_ptr(), ss.data_ptr(), zz.data_ptr(), y.data_ptr(), 1,
                                       n, k, 128, stream.cuda_stream)
            assert rc == 0, rc

        us, launches = timed(launch, copies)
        gbs = by / (us * 1e3)
        out.append({"name": name, "n": n, "k": k, "bytes": by, "us": round(us, 2), "gbs": round(gbs, 1),
                    "frac": round(gbs / peak, 3), "launches": launches, "copies": copies})
        del mats, q, sc, z
    if only is not None and only != "lm_head":
        return {"shapes": out, "peak_gbs": peak}
    n, k = 151936, 4096
    w = (torch.empty(n, k, device="cuda").normal_(0.0, 0.02, generator=gen)).to(torch.bfloat16)
    x = torch.empty(k, device="cuda").normal_(0.0, 1.0, generator=gen)
    y = torch.empty(n, device="cuda")
    by = 2 * n * k + 4 * k + 4 * n

    def launch_head(c):
        rc = L.fire_b200_linear_dense(x.data_ptr(), w.data_ptr(), N.BF16, 1.0, y.data_ptr(), 1, n, k,
                                      stream.cuda_stream)
        assert rc == 0, rc

    us, launches = timed(launch_head, 1)
    gbs = by / (us * 1e3)
    head = {"name": "lm_head_bf16", "n": n, "k": k, "bytes": by, "us": round(us, 2), "gbs": round(gbs, 1),
            "frac": round(gbs / peak, 3), "launches": launches}
    del w
    if only is not None:
        return {"shapes": out, "lm_head": head, "peak_gbs": peak}
    big = [r for r in out if r["bytes"] > 20e6]
    return {"shapes": out, "lm_head": head, "peak_gbs": peak,
            "int4_large_shape_frac": round(sum(r["bytes"] for r in big) / (sum(r["us"] for r in big) * 1e3) / peak, 3),
            "why_not_higher": "each INT4 launch is one short burst per warp (1-2.6 row tiles of 16 KB or less): "
                              "~3-4 us of launch, x staging and tail per launch against 1.4-8.4 us of bytes; "
                              "the 1.24 GB BF16 head streams at the copy peak",
            "kernels": "w4g128 K-specialised streaming GEMV (INT4); dense_gemv_kernel (BF16 head)",
            "l2": "copies of each matrix cycled, >= 2x L2 (126 MB) per cycle"}


def single_linear(reps: int = 1000):
    """The 3072x1024 single Linear (seed-0 N(0,0.02) RTN INT4 weights, x ~ N(0,1) drawn after
    W): the GPU INT4 GEMV in microseconds (L2-resident, median of per-call CUDA-event times
    of graph replays), beside the CPU FP32 Linear on the dequantised weights."""
    import torch

    from fire_b200 import _native as N
    from fire_b200 import quant

    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (3072, 1024)).astype(np.float32)
    x = rng.normal(0, 1, (1, 1024)).astype(np.float32)[0]
    q, s, z = quant.quantize_int4_groupwise(W, 128)
    p = quant.pack_uint4(q)
    L = N.lib()
    dq, ds, dz, dx = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (p, s, z, x))
    y = torch.empty(3072, device="cuda")
    stream = torch.cuda.Stream()
    per_graph = 20

    def call():
        rc = L.fire_b200_linear_w4(dx.data_ptr(), dq.data_ptr(), ds.data_ptr(), dz.data_ptr(), y.data_ptr(), 1,
                                   3072, 1024, 128, stream.cuda_stream)
        assert rc == 0, rc

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        call()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(per_graph):
                call()
        graph.replay()
        times = []
        for _ in range(reps // per_graph):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3 / per_graph)
    gpu_us = statistics.median(times)
    return {"shape": [3072, 1024], "gpu_us": round(gpu_us, 3),
            "note": "L2-resident (1.7 MB); launch-bound, not a roofline case"}, (x, p, s, z)


def cpu_linear(x, p, s, z, reps: int = 1000):
    """Fire's CPU FP32 Linear on the dequantised weights (src/op/kernels/cpu/matmul_kernel.cpp,
    restated by the oracle), median microseconds per call on all host threads and on one."""
    from oracle import oracle as O

    w = O.dequant_int4(p, s, z, 128)
    res = {}
    for threads in (os.cpu_count() or 1, 1):
        O.set_threads(threads)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            O.linear_f32(x, w)
            ts.append(time.perf_counter() - t0)
        res[threads] = statistics.median(ts) * 1e6
    O.set_threads(os.cpu_count() or 1)
    allc = os.cpu_count() or 1
    return {"cpu_fp32_us": round(res[allc], 2), "cpu_cores": allc, "cpu_fp32_us_1core": round(res[1], 2),
            "kind": "port"}


PREFILL_M = 512
PREFILL_SHAPES = [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)]  # q/k/v, o, gate/up, down


def prefill_sweep(reps: int = 10):
    """The tensor-core INT4 prefill Linear (fire_b200_linear_w4_prefill) at M = 512 on every
    Qwen3-8B projection shape, timed with CUDA events per call (x conversion + GEMM)."""
    import torch

    from fire_b200 import _native as N

    L = N.lib()
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    out, tot_fl, tot_us = [], 0.0, 0.0
    for n, k in PREFILL_SHAPES:
        x = torch.randn(PREFILL_M, k, device="cuda", generator=g)
        q = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device="cuda", generator=g)
        s = torch.rand(n, k // 128, device="cuda", generator=g) * 0.02
        z = torch.randint(0, 16, (n, k // 128), dtype=torch.uint8, device="cuda", generator=g)
        y = torch.empty(PREFILL_M, n, device="cuda")
        wsb = L.fire_b200_linear_w4_prefill_workspace_bytes(PREFILL_M, n, k)
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream()

        def call():
            rc = L.fire_b200_linear_w4_prefill(x.data_ptr(), q.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                               PREFILL_M, n, k, 128, ws.data_ptr(), wsb, st.data_ptr(),
                                               stream.cuda_stream)
            assert rc == 0, rc

        for _ in range(3):
            call()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        us = e0.elapsed_time(e1) * 1e3 / reps
        fl = 2.0 * PREFILL_M * n * k
        tot_fl += fl
        tot_us += us
        out.append({"n": n, "k": k, "us": round(us, 1), "tflops": round(fl / us / 1e6, 1)})
        del x, q, s, z, y, ws
    peak = float(peaks().get("bf16_tflops", 1590.0))
    sweep = tot_fl / tot_us / 1e6
    return {"m": PREFILL_M, "shapes": out, "sweep_tflops": round(sweep, 1), "peak_tflops": peak,
            "frac": round(sweep / peak, 3),
            "note": "useful flops 2*M*N*K per call (INT4 W dequantised to FP16 scratch, x to FP16 with a "
                    "power-of-two row scale, tcgen05 GEMM with one FP16 MMA per K16; "
                    "FIRE_B200_PREFILL_FUSED=1 times the one-pass form); peak = "
                    "MEASURED_PEAKS.json bf16_tflops (of measured; FP16 runs at the BF16 rate)"}


def parity_leg(eng, p, wn, pos0, first, gpu_tokens, world, rank, logit_steps: int = 4):
    """Greedy-token identity against the oracle from the engine's own KV prefix.

    Every rank exports its KV shard (positions < pos0); rank 0 assembles the full cache
    (heads in rank order) into the oracle and decodes the GPU's 256 steps, fed the GPU's
    tokens: each GPU token must be the oracle's argmax. The first `logit_steps` logits are
    compared too (all ranks run those forwards: under tensor parallelism they are
    collective). Returns (parity dict, cpu tokens/s over the first ~20 s, tokens timed)
    on rank 0, (None, None, None) elsewhere."""
    import torch
    import torch.distributed as dist

    from oracle import oracle as O

    kc, vc = eng.kv_export(pos0)
    logits = torch.empty(p.vocab_size, device="cuda")
    eng.truncate(pos0)
    gpu_logits = []
    tok = first
    for i in range(logit_steps):
        eng.forward(tok, pos0 + i, logits)
        torch.cuda.synchronize()
        gpu_logits.append(logits.cpu().numpy().copy())
        tok = gpu_tokens[i]
    if world > 1:
        kt, vt = torch.from_numpy(kc), torch.from_numpy(vc)
        kl = [torch.empty_like(kt) for _ in range(world)] if rank == 0 else None
        vl = [torch.empty_like(vt) for _ in range(world)] if rank == 0 else None
        dist.gather(kt, kl, dst=0)
        dist.gather(vt, vl, dst=0)
        if rank == 0:
            kc = np.concatenate([t.numpy() for t in kl], axis=2)
            vc = np.concatenate([t.numpy() for t in vl], axis=2)
    if rank != 0:
        return None, None, None
    O.set_threads(os.cpu_count() or 1)
    ref = O.Qwen3Oracle(p, wn, capacity=CAPACITY)
    ref.kc[:, :pos0] = kc
    ref.vc[:, :pos0] = vc
    ref.length = pos0
    tok = first
    mism, rels, absd, margins = [], [], [], []
    t0 = time.perf_counter()
    cpu_n, cpu_s = 0, None
    for i in range(len(gpu_tokens)):
        lg = ref.forward(tok, pos0 + i)
        if cpu_s is None:
            cpu_n += 1
            if time.perf_counter() - t0 >= 20.0:
                cpu_s = time.perf_counter() - t0
        top2 = np.partition(lg, -2)[-2:]
        margins.append(float(top2[1] - top2[0]))
        if int(np.argmax(lg)) != int(gpu_tokens[i]):
            mism.append(i)
        if i < logit_steps:
            g = gpu_logits[i]
            rels.append(float(np.linalg.norm(g - lg) / np.linalg.norm(lg)))
            absd.append(float(np.max(np.abs(g - lg))))
        tok = int(gpu_tokens[i])
    if cpu_s is None:
        cpu_s = time.perf_counter() - t0
    parity = {"tokens_equal": not mism, "steps": len(gpu_tokens), "first_mismatch": mism[0] if mism else None,
              "logit_steps": logit_steps, "max_rel_l2": max(rels), "max_abs_diff": max(absd),
              "min_top2_margin": min(margins),
              "prefix": f"the engine's KV cache of positions 0..{pos0 - 1} (after its prefill), exported to the "
                        f"oracle; the oracle is fed the GPU's tokens and must pick each of them",
              "bar": "ids identical; logits rel-L2 < 1e-4, max |d| < 1e-2 (test_qwen_profile.cpp:451-453)"}
    return parity, cpu_n / cpu_s, cpu_n


PHASES = ("qkv", "attention", "o", "gate_up", "down")


def trace_phases(layers: int = 0):
    """Per-phase timeline of one Qwen3-8B layer-stack launch at position 1791 (random FP32
    KV prefix imported into the engine), from the kernel's %globaltimer trace
    (FIRE_B200_STACK_TRACE=1): per phase, averaged over layers 1..L-2, the time from the
    previous phase's last CTA finishing to this phase's last CTA finishing, split into the
    dependency wait (until the last CTA saw its input ready) and the input staging (median
    CTA), next to the phase's bytes at the measured HBM peak."""
    import dataclasses

    import torch

    os.environ["FIRE_B200_STACK_TRACE"] = "1"
    from fire_b200 import synth
    from fire_b200.engine import Qwen3Engine
    from fire_b200.profiles import QWEN3_8B

    p = QWEN3_8B if not layers else dataclasses.replace(QWEN3_8B, num_layers=layers)
    w = synth.generate_torch(p, "mixed", seed=0, device="cuda")
    eng = Qwen3Engine(p, w)
    del w
    eng.prepare(CAPACITY)
    pos0 = PROMPT - 1
    kc = np.random.default_rng(1).standard_normal((p.num_layers, pos0, p.num_kv_heads, 128), dtype=np.float32)
    eng.kv_import(kc, kc)
    for _ in range(3):
        eng.truncate(pos0)
        eng.forward(5, pos0)
    torch.cuda.synchronize()
    tr = eng.stack_trace().astype(np.int64)  # [cta, layer, phase, slot]
    L = tr.shape[1]
    done = [[tr[:, l, ph, 3][tr[:, l, ph, 3] > 0] for ph in range(5)] for l in range(L)]
    peak = float(peaks().get("hbm_gbs", 6650.0))
    H, F, Q, KV = p.hidden_size, p.intermediate_size, p.q_dim, p.kv_dim
    w4 = lambda n, k: n * k // 2 + n * (k // 128) * 5
    phase_bytes = [w4(Q + 2 * KV, H), 2 * pos0 * KV * 4, w4(H, Q), w4(2 * F, H), w4(H, F)]
    rows = []
    for ph in range(5):
        span, wait, stage = [], [], []
        for l in range(1, L - 1):
            prev_l, prev_ph = (l, ph - 1) if ph > 0 else (l - 1, 4)
            prev_end = done[prev_l][prev_ph].max()
            act = tr[:, l, ph, 3] > 0
            span.append((done[l][ph].max() - prev_end) / 1e3)
            wait.append((tr[act, l, ph, 1].max() - prev_end) / 1e3)
            stage.append(float(np.median(tr[act, l, ph, 2] - tr[act, l, ph, 1])) / 1e3)
        rows.append({"phase": PHASES[ph], "us": round(float(np.mean(span)), 2),
                     "dependency_wait_us": round(float(np.mean(wait)), 2),
                     "staging_us": round(float(np.mean(stage)), 2) if ph != 1 else None,
                     "bytes": phase_bytes[ph], "byte_ideal_us": round(phase_bytes[ph] / (peak * 1e3), 2)})
    total = (done[L - 1][4].max() - tr[:, 0, 0, 0][tr[:, 0, 0, 0] > 0].min()) / 1e3
    eng.close()
    return {"metric": "layer-stack per-phase timeline (Qwen3-8B, position 1791)", "phases": rows,
            "layer_us": round(sum(r["us"] for r in rows), 2),
            "layer_byte_ideal_us": round(sum(r["byte_ideal_us"] for r in rows), 2),
            "launch_us": round(total, 1), "layers": L, "peak_gbs": peak}


def layer_stack_bytes(p, world: int, pos: int) -> float:
    """Algorithmic HBM bytes of one layer-stack launch at position `pos`: per layer the
    INT4 q/k/v, o, gate/up and down matrices (0.5 B per weight, 4 B scale + 1 B zero point
    per 128-group), the RMSNorm weights, the FP32 K and V rows 0..pos-1 and the row it
    writes at pos."""
    H, F, Q, KV = p.hidden_size, p.intermediate_size // world, p.q_dim // world, p.kv_dim // world
    mats = [(Q + 2 * KV, H), (H, Q), (2 * F, H), (H, F)]
    w = sum(n * k // 2 + n * (k // 128) * 5 for n, k in mats)
    norms = (2 * H + 2 * 128) * 4
    kv = 2 * (pos + 1) * KV * 4
    return float(p.num_layers * (w + norms + kv))


def run_ours(args):
    import torch
    import torch.distributed as dist

    from fire_b200 import synth
    from fire_b200.engine import Qwen3Engine, nccl_unique_id
    from fire_b200.profiles import QWEN3_8B

    rank, local, world = dist_env()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    nid = None
    if world > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    p = QWEN3_8B
    if args.layers:
        import dataclasses

        p = dataclasses.replace(p, num_layers=args.layers)
    w = synth.generate_torch(p, "mixed", seed=0, device="cuda")
    eng = Qwen3Engine(p, w, tp_rank=rank, tp_size=world, nccl_id=nid)
    cpu_w = None
    if rank == 0 and not args.no_parity:
        cpu_w = host_weights(w)
    del w
    torch.cuda.empty_cache()
    eng.prepare(CAPACITY)
    stream = torch.cuda.Stream()
    n_prompt, n_gen = args.prompt, args.gen
    assert 1 <= n_prompt and n_prompt + n_gen - 1 <= CAPACITY
    prompt = np.random.default_rng(0).integers(0, p.vocab_size, n_prompt)
    # the prompt (all but its last token) through the batched prefill, timed (TTFT part)
    stream.synchronize()
    t_pf = time.perf_counter()
    if n_prompt > 1:
        eng.prefill(prompt[:-1].tolist(), stream=stream)
    stream.synchronize()
    prefill_ms = (time.perf_counter() - t_pf) * 1e3
    first = int(prompt[-1])

    def barrier():
        if world > 1:
            dist.barrier()

    def step():
        eng.truncate(n_prompt - 1)
        return eng.generate(first, n_gen, stream=stream)

    for _ in range(args.warmup):
        toks = step()
    stream.synchronize()
    ref_tokens = toks.cpu().tolist()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            toks = step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    same = toks.cpu().tolist() == ref_tokens
    # end to end through the C ABI with host buffers (reference-style loop)
    eng.truncate(n_prompt - 1)
    eng.generate_host([first], n_gen, stream=stream)  # warm
    barrier()
    torch.cuda.synchronize()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    h0.record(stream)
    e2e_tokens = None
    for _ in range(args.steps):
        eng.truncate(n_prompt - 1)
        e2e_tokens = eng.generate_host([first], n_gen, stream=stream)
    h1.record(stream)
    torch.cuda.synchronize()
    wall_e2e = time.perf_counter() - t0
    barrier()
    ms_e2e = max(h0.elapsed_time(h1), wall_e2e * 1e3)
    # roofline of the dominant kernel, measured live
    if eng.kernels_per_step <= 5:  # persistent layer-stack kernel (+ the TP rank select)
        pos = eng.length
        kern_name = "stack_kernel"
        kern_bytes = layer_stack_bytes(p, world, pos)
        kern_us = eng.time_layer_stack(5, stream=stream) * 1e3
    else:
        kern_name = "w4g128_gemv_kernel"
        kern_bytes, kern_us = time_w4_gemv(stream)
    # max over ranks
    if world > 1:
        t = torch.tensor([ms, ms_e2e, kern_us], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e, kern_us = t.tolist()
    clocks = clk.summary()
    cpu = parity = None
    if not args.no_parity:
        parity, tps, n = parity_leg(eng, p, cpu_w, n_prompt - 1, first, ref_tokens, world, rank)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            from oracle import oracle as O

            cpu = {"value": tps, "unit": "tok/s", "cores": O.lib().fo_get_threads(), "kind": "port",
                   "sample": f"the first {n} greedy decode steps (about 20 s) of the parity leg: the FP32 CPU "
                             f"restatement of Qwen3Model::forward from the engine's KV prefix at position "
                             f"{n_prompt - 1}, INT4 dequantised on the fly, all 36 layers + BF16 head"}
    gemv = lin = None
    if rank == 0 and world == 1:
        gemv = gemv_sweep()
        lin, lin_data = single_linear()
        if not args.no_cpu_baseline:
            lin.update(cpu_linear(*lin_data))
    if rank == 0:
        pk = peaks()
        peak = float(pk.get("hbm_gbs", 6650.0))
        tok_s = n_gen * args.steps / (ms / 1e3)
        tok_s_e2e = n_gen * args.steps / (ms_e2e / 1e3)
        step_bytes = eng.step_weight_bytes  # per GPU per token
        per_tok_s = (ms / 1e3) / (n_gen * args.steps)
        traffic = None
        try:
            tr = json.load(open(os.path.join(ROOT, "profiles", "dram_traffic.json")))
            # the committed capture is of the TP1 launch; no TP capture exists
            traffic = tr.get(kern_name, {}).get("bytes_per_launch_scaled") if world == 1 else None
        except (OSError, ValueError):
            pass
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(world, n_prompt, n_gen, p.num_layers),
            "e2e": {"value": tok_s_e2e, "unit": "tok/s", "h2d_bytes_per_step": 16 * n_gen,
                    "d2h_bytes_per_step": 16 * n_gen},
            "gpu_launches": (eng.kernels_per_step * n_gen + 1) * args.steps,
            "roofline": {"bound": "hbm", "kernel": kern_name, "achieved": kern_bytes / (kern_us * 1e3),
                         "peak": peak, "unit": "GB/s", "frac": kern_bytes / (kern_us * 1e3) / peak,
                         "traffic": traffic, "bytes_per_launch": kern_bytes, "us_per_launch": kern_us,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "when" in pk else "fallback"},
            "decode_roofline": {"bytes_per_token_per_gpu": step_bytes, "achieved": step_bytes / per_tok_s / 1e9,
                                "unit": "GB/s", "frac": step_bytes / per_tok_s / 1e9 / peak,
                                "us_per_token": per_tok_s * 1e6},
            "clocks": clocks,
            "tokens_repeatable": same,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if parity is not None:
            line["parity"] = parity
        if gemv is not None:
            line["gemv_sweep"] = gemv
            line["single_linear"] = lin
        line["prefill"] = {"prompt_tokens": n_prompt - 1, "ms": round(prefill_ms, 2),
                           "tok_s": round((n_prompt - 1) / (prefill_ms / 1e3), 1) if prefill_ms > 0 else None,
                           "path": "batched tcgen05 prefill" + (f" (tensor parallel over {world}, o/down "
                                                                 f"all-reduced)" if world > 1 else ""),
                           "note": "host wall clock around fire_b200_qwen3_prefill (synchronising)"}
        if world == 1:
            line["prefill_gemm"] = prefill_sweep()
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.prefill:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps({"metric": "INT4 prefill GEMM TFLOP/s (M=512, Qwen3-8B projection shapes)",
                          **prefill_sweep()}), flush=True)
        return 0
    if args.trace_phases:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps(trace_phases(args.layers)), flush=True)
        return 0
    if args.gemv:
        import torch

        torch.cuda.set_device(0)
        if args.gemv_shape:
            print(json.dumps({"metric": "INT4 GEMV HBM GB/s vs peak (M=1, Qwen3-8B shapes)",
                              **gemv_sweep(only=args.gemv_shape)}), flush=True)
            return 0
        print(json.dumps({"metric": "INT4 GEMV HBM GB/s vs peak (M=1, Qwen3-8B shapes)", **gemv_sweep(),
                          "single_linear": single_linear()[0]}), flush=True)
        return 0
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
