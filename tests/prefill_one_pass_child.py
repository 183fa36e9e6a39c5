"""Child process of test_gpu_prefill.py: the same prefill cases with the one-pass form
selected (FIRE_B200_PREFILL_FUSED=1 in the environment, read once per process), results
saved to the .npz path given as the only argument."""
import sys

import numpy as np


def cases():
    """(m, n, k, seed) of the Linear cases and (profile name, prompt length) of the engine case."""
    return [(128, 128, 256, 1), (256, 384, 1024, 2), (512, 6144, 4096, 3), (512, 4096, 12288, 4)], ("small", 200)


def compute():
    import torch

    from fire_b200 import synth
    from fire_b200.engine import Qwen3Engine
    from fire_b200.profiles import Qwen3Profile
    from tests.test_gpu_prefill import make, run

    out = {}
    lin, (_, n) = cases()
    for m, nn, k, seed in lin:
        x, packed, s, z, _ = make(m, nn, k, seed)
        out[f"lin_{m}_{nn}_{k}"] = run(x, packed, s, z, m, nn, k)
    p = Qwen3Profile("small-qwen3", 4096, 4096, 512, 1536, 3, 8, 4, 128)
    w = synth.generate(p, "int4", seed=21)
    eng = Qwen3Engine(p, w)
    eng.prepare(n + 8)
    prompt = np.random.default_rng(n).integers(0, p.vocab_size, n)
    logits = torch.empty(p.vocab_size, device="cuda")
    eng.prefill(prompt.tolist(), logits)
    eng.forward(int(torch.argmax(logits)), n, logits)
    torch.cuda.synchronize()
    out["engine"] = logits.cpu().numpy()
    return out


if __name__ == "__main__":
    np.savez(sys.argv[1], **compute())
