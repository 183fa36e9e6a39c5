"""Failure detection of the decode engine, exercised without faulting a GPU.

A step that cannot finish must come back as a status, never as a hang or as silently wrong
logits. Every wait inside the persistent layer-stack kernel is bounded (0.2 s of GPU time);
when one runs out the kernel records code 3 in the device decode state and returns. The
injected failure is a wait that cannot be met: with FIRE_B200_FAULT_STALL=1 at engine
creation, layer 0's o phase waits for one CTA more than the grid has (a counter that nothing
bumps), until the engine is reset. Under tensor parallelism a peer that stops answering is
met by the host-side deadline of the synchronising calls, which aborts the communicator
(ncclCommAbort) and returns FIRE_B200_ERR_TIMEOUT. The reference's transactional rule is
kept: a failed step is reported and the sequence restarts clean after reset
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


def _tp_rank(rank, world, nid, prof, w, q, mode, release):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        if mode == "stall" and rank == 1:
            os.environ["FIRE_B200_FAULT_STALL"] = "1"
        torch.cuda.set_device(rank)
        from fire_b200 import _native as NN
        from fire_b200.engine import Qwen3Engine

        eng = Qwen3Engine(prof, w, tp_rank=rank, tp_size=world, nccl_id=nid, deadline_ms=3000)
        os.environ.pop("FIRE_B200_FAULT_STALL", None)
        eng.prepare(64)
        out = {"kps": eng.kernels_per_step}
        if mode == "stall":
            eng.forward(PROMPT[0], 0)
            out["code"] = eng.status()
            eng.reset()
            out["toks"] = eng.generate_host(PROMPT, STEPS).tolist()
            out["code_after"] = eng.status()
            eng.close()
        else:  # "leave": rank 1 stops launching after one good step; rank 0 meets the deadline
            eng.forward(PROMPT[0], 0)
            out["code"] = eng.status()
            if rank == 0:
                eng.forward(PROMPT[1], 1)
                try:
                    eng.status()
                    out["late"] = "no error"
                except NN.FireB200Error as e:
                    out["late"] = e.status
                eng.close()
                q.put((rank, out, None))
                return
            # rank 1: stays alive (its memory stays mapped) without launching, until the
            # parent says rank 0 is done; then leaves the group without waiting for it
            q.put((rank, out, None))
            release.get(timeout=300)
            eng.abort()
            eng.close()
            return
        q.put((rank, out, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


def _spawn(prof, w, mode, world=2):
    from fire_b200.engine import nccl_unique_id

    nid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = []
    release = ctx.Queue()
    for r in range(world):
        procs.append(ctx.Process(target=_tp_rank, args=(r, world, nid, prof, w, q, mode, release)))
    for p in procs:
        p.start()
    return procs, q, release


def test_tp2_peer_timeout_is_reported_on_both_ranks_then_reset_recovers(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    prof = STACK
    w = synth.generate(prof, "mixed", seed=11)
    procs, q, _ = _spawn(prof, w, "stall")
    res = {}
    for _ in range(2):
        rank, out, err = q.get(timeout=600)
        assert err is None, f"rank {rank}: {err}"
        res[rank] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = oracle_greedy(prof, w, PROMPT, STEPS, 64)
    for r in (0, 1):
        assert res[r]["kps"] <= 5  # layer-stack path with the in-kernel exchange
        assert res[r]["code"] == 3, (r, res[r])  # rank 1 stalled, rank 0's exchange poll ran out
        assert res[r]["code_after"] == 0
        assert res[r]["toks"] == want, r


def test_tp2_rank_that_stops_launching_meets_the_host_deadline(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    prof = STACK
    w = synth.generate(prof, "mixed", seed=11)
    procs, q, release = _spawn(prof, w, "leave")
    res = {}
    for _ in range(2):
        rank, out, err = q.get(timeout=600)
        assert err is None, f"rank {rank}: {err}"
        res[rank] = out
        if rank == 0:
            release.put(1)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0]["code"] == 0 and res[1]["code"] == 0
    assert res[0]["late"] == N.ERR_TIMEOUT, res[0]
