"""CPU: the C-ABI library loads, exports every symbol include/*.h declares, and rejects
bad arguments on the host before touching a GPU (no kernel is launched here)."""
import ctypes as C
import subprocess

import pytest

from fire_b200 import _native as N


def test_library_exports_every_declared_symbol():
    declared = N.declared_symbols()
    assert "fire_b200_linear_w4" in declared and len(declared) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    L = N.lib()  # binds every signature (raises on a missing symbol)
    for s in declared:
        assert hasattr(L, s)


def test_abi_version_and_status_strings():
    L = N.lib()
    assert L.fire_b200_abi_version() == 1
    assert N.status_string(N.OK) == "ok"
    assert N.status_string(N.ERR_INVALID) == "invalid argument"


def test_host_side_argument_checks_reject_without_launch():
    L = N.lib()
    p = C.c_void_p(16)  # never dereferenced: every call below fails validation first
    # null pointers
    assert L.fire_b200_linear_w4(None, p, p, p, p, 1, 8, 256, 128, None) == N.ERR_INVALID
    # odd k, group not dividing k, non-positive sizes
    assert L.fire_b200_linear_w4(p, p, p, p, p, 1, 8, 255, 128, None) == N.ERR_INVALID
    assert L.fire_b200_linear_w4(p, p, p, p, p, 1, 8, 256, 100, None) == N.ERR_INVALID
    assert L.fire_b200_linear_w4(p, p, p, p, p, 0, 8, 256, 128, None) == N.ERR_INVALID
    assert L.fire_b200_linear_dense(p, p, 7, 1.0, p, 1, 8, 8, None) == N.ERR_INVALID
    assert L.fire_b200_rope(p, p, p, p, 4, 2, 7, 16, 0, None) == N.ERR_INVALID       # odd head
    assert L.fire_b200_rope(p, p, p, p, 4, 2, 8, 16, 16, None) == N.ERR_INVALID      # pos == max_seq
    assert L.fire_b200_rope(p, p, p, p, 2, 4, 8, 16, 0, None) == N.ERR_INVALID       # k heads > q heads
    ws = L.fire_b200_mha_workspace_bytes(32, 8, 128, 2048)
    assert ws > 0
    assert L.fire_b200_mha_decode(p, p, p, None, p, 2, 16, 6, 4, 8, 0, 0, p, ws, None) == N.ERR_INVALID
    assert L.fire_b200_mha_decode(p, p, p, None, p, 2, 16, 4, 2, 8, 2, 0, p, ws, None) == N.ERR_INVALID
    assert L.fire_b200_mha_decode(p, p, p, None, p, 2, 16, 4, 2, 8, 0, 16, p, ws, None) == N.ERR_INVALID
    assert L.fire_b200_mha_decode(p, p, p, None, p, 2, 16, 4, 2, 8, 0, 0, p, 0, None) == N.ERR_INVALID
    assert L.fire_b200_embedding(p, 1, p, 3, 10, 4, p, None) == N.ERR_INVALID
    assert L.fire_b200_argmax(p, 0, p, p, 1 << 20, None) == N.ERR_INVALID
    assert L.fire_b200_argmax(p, 10, p, p, 1, None) == N.ERR_INVALID
    assert L.fire_b200_rmsnorm(p, p, p, 0, 1e-6, None) == N.ERR_INVALID
