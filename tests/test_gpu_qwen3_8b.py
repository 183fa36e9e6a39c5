"""Qwen3-8B, the decode benchmark's own configuration, against the oracle.

Same construction as the benchmark: Qwen3-8B architecture (36 layers, hidden 4096, 32 q /
8 kv heads, FFN 12288, vocab 151936), seed-0 random-init weights in the AWQ mixed layout
(INT4 group-128 projections with FP16-valued scales, BF16 embedding and LM head), a
1792-token prompt of uniform ids whose first 1791 tokens go through the batched prefill,
then greedy decode from position 1791 to the end of the 2048-token context.

The engine's KV prefix (positions 0..1790) is exported into the oracle, so both decode from
the same FP32 prefix and every difference comes from the decode path itself: the
persistent layer-stack kernel with its K = 4096 / 12288 unit shapes, the BF16 LM head and
the device argmax. Bars: the reference's GPU-vs-CPU model test
(test/test_model/test_qwen_profile.cpp:451-453: max |logit difference| < 1e-2, same argmax)
plus rel-L2 < 1e-4 on the first 16 steps, then 256 greedy token ids identical to the
oracle's (src/model/qwen.cpp:155-303 restated in FP32 on the CPU).
"""
import os

import numpy as np
import pytest
import torch

from fire_b200 import synth
from fire_b200.engine import Qwen3Engine
from fire_b200.profiles import QWEN3_8B
from oracle import oracle as O

pytestmark = pytest.mark.gpu

PROMPT = 1792
CAPACITY = 2048
GEN = CAPACITY - PROMPT + 1  # 257 positions 1791..2047: 256 sampled ids + the last step
LOGIT_STEPS = 16


def host(w):
    out = {}
    for k, v in w.items():
        a = v.cpu()
        out[k] = a.numpy().view(np.uint16) if a.dtype == torch.int16 else a.numpy()
    return out


def test_qwen3_8b_decode_matches_oracle_from_shared_prefix(cuda):
    p = QWEN3_8B
    w = synth.generate_torch(p, "mixed", seed=0, device="cuda")
    eng = Qwen3Engine(p, w)
    wn = host(w)
    del w
    torch.cuda.empty_cache()
    eng.prepare(CAPACITY)
    prompt = np.random.default_rng(0).integers(0, p.vocab_size, PROMPT)
    eng.prefill(prompt[:-1].tolist())
    first = int(prompt[-1])
    pos0 = PROMPT - 1
    assert eng.length == pos0
    kc, vc = eng.kv_export(pos0)

    # GPU: the benchmark's step, 256 greedy ids on the device
    got = eng.generate(first, 256).cpu().tolist()
    assert eng.status() == 0

    O.set_threads(os.cpu_count() or 1)
    ref = O.Qwen3Oracle(p, wn, capacity=CAPACITY)
    ref.kc[:, :pos0] = kc
    ref.vc[:, :pos0] = vc
    ref.length = pos0

    # logits of the first steps, both sides fed the GPU's tokens
    eng.truncate(pos0)
    logits = torch.empty(p.vocab_size, device="cuda")
    tok = first
    want, margins, rels = [], [], []
    for i in range(LOGIT_STEPS):
        eng.forward(tok, pos0 + i, logits)
        r = ref.forward(tok, pos0 + i)
        torch.cuda.synchronize()
        g = logits.cpu().numpy()
        rel = float(np.linalg.norm(g - r) / np.linalg.norm(r))
        rels.append(rel)
        assert rel < 1e-4, (i, rel)
        assert float(np.max(np.abs(g - r))) < 1e-2, i
        assert int(np.argmax(g)) == int(np.argmax(r)), i
        top2 = np.partition(r, -2)[-2:]
        margins.append(float(top2[1] - top2[0]))
        want.append(O.argmax(r))
        tok = want[-1]
    assert eng.status() == 0
    # the oracle alone for the rest of the 256 greedy steps
    lg = r
    for i in range(LOGIT_STEPS, 256):
        lg = ref.forward(want[-1], pos0 + i)
        top2 = np.partition(lg, -2)[-2:]
        margins.append(float(top2[1] - top2[0]))
        want.append(O.argmax(lg))
    mismatch = [i for i in range(256) if got[i] != want[i]]
    print(f"8B decode parity: max rel-L2 {max(rels):.2e} over {LOGIT_STEPS} steps, "
          f"min top-2 margin {min(margins):.3e}")
    assert not mismatch, f"first mismatch at step {mismatch[0]}, top-2 margin {margins[mismatch[0]]:.3e}"
