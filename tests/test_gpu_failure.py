"""Failure detection of the decode engine, exercised without faulting a GPU.

A step that cannot finish must come back as a status, never as a hang or as silently wrong
logits. Every wait inside the persistent layer-stack kernel is bounded (0.2 s of GPU time);
when one runs out the kernel records code 3 in the device decode state and returns. The
injected failure is a wait that cannot be met: with FIRE_B200_FAULT_STALL=1 at engine
creation, layer 0's o phase waits for one CTA more than the grid has (a counter that nothing
bumps), until the engine is reset. Under tensor parallelism the stalled rank makes the other
rank's poll of its exchange words run out; both report the failure and recover after reset.
(A peer that stops launching altogether leaves the other rank's NCCL collective waiting; the
host deadline that aborts the communicator for that case is not exercised here.) The
reference's transactional rule is kept: a failed step is reported and the sequence restarts clean after reset
(src/model/kv_cache.cpp:76-83, include/Fire/model/model.h:37-44).
"""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from fire_b200 import _native as N
from fire_b200 import synth
from fire_b200.profiles import Qwen3Profile

pytestmark = pytest.mark.gpu

SMALL = Qwen3Profile("small-qwen3", 4096, 4096, 512, 1536, 3, 8, 4, 128)
STACK = Qwen3Profile("tp-stack", 4096, 512, 512, 2048, 2, 8, 4, 128)
PROMPT = [11, 2024, 7, 99, 3000]
STEPS = 12


def oracle_greedy(prof, w, prompt, steps, cap):
    from oracle import oracle as O

    ref = O.Qwen3Oracle(prof, w, capacity=cap)
    for i, t in enumerate(prompt):
        lg = ref.forward(t, i)
    want = []
    for i in range(steps):
        want.append(O.argmax(lg))
        if i + 1 < steps:
            lg = ref.forward(want[-1], len(prompt) + i)
    return want


def test_stack_wait_timeout_is_reported_then_reset_recovers(cuda, monkeypatch):
    from fire_b200.engine import Qwen3Engine

    p = SMALL
    w = synth.generate(p, "mixed", seed=9)
    monkeypatch.setenv("FIRE_B200_FAULT_STALL", "1")
    eng = Qwen3Engine(p, w)
    monkeypatch.delenv("FIRE_B200_FAULT_STALL")
    assert eng.kernels_per_step == 4  # the layer-stack path
    eng.prepare(64)
    eng.forward(PROMPT[0], 0)
    assert eng.status() == 3  # a bounded wait ran out
    # every step entry point now fails fast, without launching
    for call in (lambda: eng.forward(PROMPT[1], 1), lambda: eng.generate(PROMPT[1], 4),
                 lambda: eng.generate_host(PROMPT, 2)):
        with pytest.raises(N.FireB200Error) as e:
            call()
        assert e.value.status == N.ERR_DEVICE
    # reset clears the failure (and the injected stall): decoding is correct again
    eng.reset()
    got = eng.generate_host(PROMPT, STEPS)
    assert eng.status() == 0
    want = oracle_greedy(p, w, PROMPT, STEPS, 64)
    assert got.tolist() == want
    # and a fresh engine agrees
    fresh = Qwen3Engine(p, w)
    fresh.prepare(64)
    assert fresh.generate_host(PROMPT, STEPS).tolist() == want
    fresh.close()
    eng.close()


def _tp_rank(rank, world, nid, prof, w, q):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        if rank == 1:
            os.environ["FIRE_B200_FAULT_STALL"] = "1"
        torch.cuda.set_device(rank)
        from fire_b200.engine import Qwen3Engine

        eng = Qwen3Engine(prof, w, tp_rank=rank, tp_size=world, nccl_id=nid, deadline_ms=30000)
        os.environ.pop("FIRE_B200_FAULT_STALL", None)
        eng.prepare(64)
        out = {"kps": eng.kernels_per_step}
        # both ranks launch every step: rank 1 stalls in its own bounded wait, rank 0's poll
        # of rank 1's exchange words runs out; nobody waits on a peer that stopped launching
        eng.forward(PROMPT[0], 0)
        out["code"] = eng.status()
        eng.reset()
        out["toks"] = eng.generate_host(PROMPT, STEPS).tolist()
        out["code_after"] = eng.status()
        eng.close()
        q.put((rank, out, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


def test_tp2_peer_timeout_is_reported_on_both_ranks_then_reset_recovers(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from fire_b200.engine import nccl_unique_id

    prof = STACK
    w = synth.generate(prof, "mixed", seed=11)
    nid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, nid, prof, w, q), daemon=True) for r in range(2)]
    try:
        for p in procs:
            p.start()
        res = {}
        for _ in range(2):
            rank, out, err = q.get(timeout=240)
            assert err is None, f"rank {rank}: {err}"
            res[rank] = out
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:  # no rank may outlive the test
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    want = oracle_greedy(prof, w, PROMPT, STEPS, 64)
    for r in (0, 1):
        assert res[r]["kps"] <= 5  # layer-stack path with the in-kernel exchange
        assert res[r]["code"] == 3, (r, res[r])  # rank 1 stalled, rank 0's exchange poll ran out
        assert res[r]["code_after"] == 0
        assert res[r]["toks"] == want, r
