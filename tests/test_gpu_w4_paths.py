"""Alternate kernel paths of the decode engine, each checked against the oracle.

* FIRE_B200_W4_PATH=mma: fire_b200_linear_w4 runs the tensor-core kernel (exact u8 x s8
  integer MMAs) instead of the FP32 streaming kernels.
* FIRE_B200_LAYER_STACK=0: the engine runs one kernel per op instead of the persistent
  layer-stack kernel (the default at tensor-parallel size 1).
Both are read once per process, so the parity tests re-run in a child process."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENGINE = ["tests/test_gpu_engine.py::test_engine_forward_matches_oracle",
          "tests/test_gpu_engine.py::test_engine_greedy_device_and_host_loops_match_oracle",
          "tests/test_gpu_engine.py::test_engine_reset_is_deterministic_and_graph_matches_eager"]


@pytest.mark.parametrize("var,value,targets", [
    ("FIRE_B200_W4_PATH", "mma", ["tests/test_gpu_kernels.py", "-k", "w4"] + ENGINE),
    ("FIRE_B200_LAYER_STACK", "0", ENGINE),
])
def test_parity_on_alternate_path(cuda, var, value, targets):
    env = dict(os.environ, **{var: value})
    cmd = [sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider"] + targets
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
