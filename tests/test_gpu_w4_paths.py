"""The INT4 GEMV has two kernel families behind fire_b200_linear_w4: FP32 streaming
kernels (default) and the tensor-core kernel with exact u8 x s8 integer MMAs
(FIRE_B200_W4_PATH=mma). The path is chosen once per process, so the MMA family is
checked by re-running the W4 parity tests and the engine parity test in a child process."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("path", ["mma"])
def test_w4_parity_on_alternate_path(cuda, path):
    env = dict(os.environ, FIRE_B200_W4_PATH=path)
    cmd = [sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider",
           "tests/test_gpu_kernels.py", "-k", "w4",
           "tests/test_gpu_engine.py::test_engine_forward_matches_oracle",
           "tests/test_gpu_engine.py::test_engine_greedy_device_and_host_loops_match_oracle"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
