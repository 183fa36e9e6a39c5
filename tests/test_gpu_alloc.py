"""The device allocator drop-in (include/fire_b200_alloc.h) that replaces Fire's GPU
DeviceAllocator (src/base/alloc_cu.cpp:11-151, src/base/alloc.cpp:8-68): alignment,
disjoint live blocks under contention from many host threads, reuse of released blocks,
errors returned instead of aborts, and memset_zero / memcpy in every direction."""
import ctypes as C
import threading

import numpy as np
import pytest

from fire_b200 import _native as N

pytestmark = pytest.mark.gpu


def alloc(n):
    p = C.c_void_p()
    rc = N.lib().fire_b200_device_alloc(n, C.byref(p))
    assert rc == N.OK, rc
    return p.value


def stats(dev=0):
    r, u, l = C.c_size_t(), C.c_size_t(), C.c_size_t()
    assert N.lib().fire_b200_device_pool_stats(dev, C.byref(r), C.byref(u), C.byref(l)) == N.OK
    return r.value, u.value, l.value


def test_alloc_release_contention_keeps_blocks_disjoint_and_aligned(cuda):
    L = N.lib()
    live0 = stats()[2]
    errors, spans = [], []
    lock = threading.Lock()

    def worker(seed):
        rng = np.random.default_rng(seed)
        mine = []
        try:
            for it in range(400):
                if mine and rng.random() < 0.45:
                    p, n = mine.pop(int(rng.integers(len(mine))))
                    with lock:
                        spans.remove((p, n))
                    assert L.fire_b200_device_release(p) == N.OK
                else:
                    n = int(rng.choice([1, 100, 256, 4097, 70_000, 1 << 20, 3 << 20]))
                    p = alloc(n)
                    assert p % 256 == 0
                    with lock:
                        spans.append((p, n))
                    mine.append((p, n))
            for p, n in mine:
                with lock:
                    spans.remove((p, n))
                assert L.fire_b200_device_release(p) == N.OK
        except Exception as e:  # reported below
            errors.append(repr(e))

    # a snapshot check of disjointness while the threads run
    def overlap_free():
        with lock:
            s = sorted(spans)
        return all(a + n <= b for (a, n), (b, _) in zip(s, s[1:]))

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(8)]
    for t in threads:
        t.start()
    checks = 0
    while any(t.is_alive() for t in threads):
        assert overlap_free()
        checks += 1
    for t in threads:
        t.join()
    assert not errors, errors
    assert stats()[2] == live0  # every block released
    assert checks > 0


def test_release_reuses_blocks_and_rejects_unknown_or_double_release(cuda):
    L = N.lib()
    a = alloc(5000)
    assert L.fire_b200_device_release(a) == N.OK
    b = alloc(5000)  # same size class: the cached block comes back
    assert b == a
    assert L.fire_b200_device_release(b) == N.OK
    assert L.fire_b200_device_release(b) == N.ERR_INVALID  # released twice
    assert L.fire_b200_device_release(C.c_void_p(0x1234)) == N.ERR_INVALID  # not ours
    assert L.fire_b200_device_release(None) == N.OK
    r0 = stats()[0]
    assert L.fire_b200_device_pool_trim(0) == N.OK
    assert stats()[0] <= r0
    assert L.fire_b200_device_memcpy(None, None, 4, N.GPU2GPU, None, 1) == N.ERR_INVALID
    assert L.fire_b200_device_memcpy(C.c_void_p(1), C.c_void_p(1), 4, 9, None, 1) == N.ERR_INVALID


def test_memset_zero_and_memcpy_every_direction(cuda):
    L = N.lib()
    n = 1 << 20
    src = np.arange(n // 4, dtype=np.float32)
    d1, d2 = alloc(n), alloc(n)
    assert L.fire_b200_device_memcpy(src.ctypes.data, d1, n, N.CPU2GPU, None, 0) == N.OK
    assert L.fire_b200_device_memcpy(d1, d2, n, N.GPU2GPU, None, 0) == N.OK
    out = np.empty_like(src)
    assert L.fire_b200_device_memcpy(d2, out.ctypes.data, n, N.GPU2CPU, None, 1) == N.OK
    assert np.array_equal(out, src)
    assert L.fire_b200_device_memset_zero(d2, n, None, 1) == N.OK
    assert L.fire_b200_device_memcpy(d2, out.ctypes.data, n, N.GPU2CPU, None, 1) == N.OK
    assert not out.any()
    host2 = np.empty_like(src)
    assert L.fire_b200_device_memcpy(src.ctypes.data, host2.ctypes.data, n, N.CPU2CPU, None, 0) == N.OK
    assert np.array_equal(host2, src)
    for p in (d1, d2):
        assert L.fire_b200_device_release(p) == N.OK
