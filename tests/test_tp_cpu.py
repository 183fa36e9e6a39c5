"""CPU (gloo, world size 2 and 4): the tensor-parallel decomposition the engine uses.

Each rank keeps the shard fire_b200's engine keeps (src/model TP layer, see
fire_b200/csrc/engine/qwen3.cpp import_weights): q/k/v and gate/up rows of its heads /
FFN slice (column parallel), o/down K-slices on group boundaries (row parallel), its
vocabulary slice of the LM head, and the KV heads of its q heads. Partial sums are
all-reduced in rank order and the sampler all-gathers one (max, index) pair per rank.
The decode of every rank must equal the unsharded oracle.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fire_b200 import synth
from fire_b200.profiles import Qwen3Profile

P = Qwen3Profile("tp-test", 512, 64, 256, 512, 2, 4, 4, 128)


def shard_rows(w, base, r0, n, group=128):
    return {".qweight": w[base + ".qweight"][r0:r0 + n], ".scales": w[base + ".scales"][r0:r0 + n],
            ".zero_points": w[base + ".zero_points"][r0:r0 + n]}


def shard_cols(w, base, c0, k, group=128):
    return {".qweight": w[base + ".qweight"][:, c0 // 2:(c0 + k) // 2],
            ".scales": w[base + ".scales"][:, c0 // group:(c0 + k) // group],
            ".zero_points": w[base + ".zero_points"][:, c0 // group:(c0 + k) // group]}


def lin(x, m):
    from oracle import oracle as O
    return O.linear_int4(x, m[".qweight"], m[".scales"], m[".zero_points"], 128)


def tp_decode(rank, world, w, tokens, steps):
    """One rank's decode; collectives through torch.distributed (gloo)."""
    from oracle import oracle as O

    p = P
    hq, hkv, f, v = p.num_attention_heads // world, p.num_kv_heads // world, p.intermediate_size // world, \
        p.vocab_size // world
    q_, kv_ = hq * 128, hkv * 128
    sin, cos = O.rope_cache(128, p.max_seq_len, p.rope_theta)
    kc = np.zeros((p.num_layers, p.max_seq_len, hkv, 128), np.float32)
    vc = np.zeros_like(kc)

    def allreduce(x):
        t = torch.from_numpy(np.ascontiguousarray(x))
        dist.all_reduce(t)
        return t.numpy()

    out = []
    tok = tokens[0]
    pos = 0
    n_total = len(tokens) + steps - 1
    for i in range(n_total):
        hidden = O.embedding([tok], w["tok_embeddings.weight"])[0]
        for l in range(p.num_layers):
            pre = f"layers.{l}."
            x = O.rmsnorm(hidden, w[pre + "attention_norm.weight"], p.rms_norm_eps)
            q = lin(x, shard_rows(w, pre + "attention.wq", rank * q_, q_)).reshape(hq, 128)
            k = lin(x, shard_rows(w, pre + "attention.wk", rank * kv_, kv_)).reshape(hkv, 128)
            vv = lin(x, shard_rows(w, pre + "attention.wv", rank * kv_, kv_)).reshape(hkv, 128)
            q = O.rmsnorm_rows(q, w[pre + "attention.q_norm.weight"], p.rms_norm_eps)
            k = O.rmsnorm_rows(k, w[pre + "attention.k_norm.weight"], p.rms_norm_eps)
            q, k = O.rope(q, k, cos, sin, pos)
            kc[l, pos], vc[l, pos] = k, vv
            att, _ = O.mha(q, kc, vc, l, pos)
            o_part = lin(att.reshape(-1), shard_cols(w, pre + "attention.wo", rank * q_, q_))
            attn_res = O.add(hidden, allreduce(o_part))
            x = O.rmsnorm(attn_res, w[pre + "ffn_norm.weight"], p.rms_norm_eps)
            g = lin(x, shard_rows(w, pre + "feed_forward.w1", rank * f, f))
            u = lin(x, shard_rows(w, pre + "feed_forward.w3", rank * f, f))
            d_part = lin(O.swiglu(g, u), shard_cols(w, pre + "feed_forward.w2", rank * f, f))
            hidden = O.add(attn_res, allreduce(d_part))
        x = O.rmsnorm(hidden, w["norm.weight"], p.rms_norm_eps)
        logits = lin(x, shard_rows(w, "output", rank * v, v))
        # sampling: all-gather (max, global index) pairs, fold in rank order, first max wins
        j = O.argmax(logits)
        pair = torch.tensor([float(logits[j]), float(rank * v + j)], dtype=torch.float64)
        pairs = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(pairs, pair)
        best_v, best_i = -np.inf, None
        for pr in pairs:
            if pr[0].item() > best_v:
                best_v, best_i = pr[0].item(), int(pr[1].item())
        pos += 1
        if i + 1 < len(tokens):
            tok = tokens[i + 1]
        else:
            out.append(best_i)
            tok = best_i
    return out


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = synth.generate(P, "int4", seed=21)
        q.put((rank, tp_decode(rank, world, w, [3, 77, 401], 6)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_decode_matches_unsharded_oracle(world):
    from oracle import oracle as O

    w = synth.generate(P, "int4", seed=21)
    ref = O.Qwen3Oracle(P, w, capacity=16)
    prompt = [3, 77, 401]
    for i, t in enumerate(prompt):
        lg = ref.forward(t, i)
    want = []
    for i in range(6):
        nxt = O.argmax(lg)
        want.append(nxt)
        lg = ref.forward(nxt, len(prompt) + i)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + world * 7 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    for r in range(world):
        assert results[r] == want, (r, results[r], want)


def test_sharded_sampler_breaks_ties_to_the_smallest_index():
    """Ties across shards: the lower rank holds the lower global index and wins."""
    world, v = 4, 10
    logits = np.zeros(world * v, np.float32)
    logits[[7, 13, 25]] = 5.0  # tie across ranks 0, 1, 2
    best_v, best_i = -np.inf, None
    for r in range(world):
        sl = logits[r * v:(r + 1) * v]
        j = int(np.argmax(sl))
        if sl[j] > best_v:
            best_v, best_i = float(sl[j]), r * v + j
    assert best_i == 7 == int(np.argmax(logits))
