"""The ``.fire`` v1/v2 tensor container: writer and reader.

Wire format (Fire ``docs/qwen3_quantization_plan.md`` and
``src/model/fire_reader.cpp:20-385``; the bytes must match, so the layout is
the same while the code is this project's own):

* 32-byte header ``<8sIIQQ``: magic ``FIRECKPT``, version (1 or 2), tensor count,
  directory offset (32), data offset (32 + 96 * count).
* 96-byte records ``<64sQQIIBB6s``: NUL-padded ASCII name, byte offset, byte size,
  shape0, shape1 (0 for rank 1), wire dtype (1 FP32, 2 UInt8, 3 BF16), rank, and six
  metadata bytes. v2 INT4 ``qweight`` records carry ``kind=1, group_size:u32, 0``.
* Payloads in directory order; v1 packs them back to back (FP32 only), v2 pads each
  one with zeros to a 4-byte boundary.
"""
from __future__ import annotations

import math
import mmap
import os
import struct
from dataclasses import dataclass
from typing import BinaryIO, Dict, Iterable, List, Optional, Tuple

import numpy as np

MAGIC = b"FIRECKPT"
HEADER = struct.Struct("<8sIIQQ")
RECORD = struct.Struct("<64sQQIIBB6s")
assert HEADER.size == 32 and RECORD.size == 96

FP32, UINT8, BF16 = 1, 2, 3
_NP = {FP32: np.dtype("<f4"), UINT8: np.dtype("u1"), BF16: np.dtype("<u2")}
_SIZE = {FP32: 4, UINT8: 1, BF16: 2}


class FireFormatError(ValueError):
    pass


@dataclass(frozen=True)
class Record:
    name: str
    dtype: int
    shape: Tuple[int, ...]
    offset: int
    size: int
    group_size: int = 0  # non-zero only on INT4 qweight records (v2)


def wire_dtype(array: np.ndarray) -> int:
    if array.dtype == np.float32:
        return FP32
    if array.dtype == np.uint8:
        return UINT8
    if array.dtype == np.uint16:  # raw BF16 bits
        return BF16
    raise FireFormatError(f"unsupported payload dtype {array.dtype}")


def plan(entries: Iterable[Tuple[str, np.ndarray, int]], version: int = 2) -> List[Record]:
    """Directory for (name, array, group_size) entries in payload order."""
    entries = list(entries)
    if version not in (1, 2):
        raise FireFormatError(f"unsupported version {version}")
    off = HEADER.size + RECORD.size * len(entries)
    recs, seen = [], set()
    for name, arr, group in entries:
        raw = name.encode("ascii")
        if not raw or len(raw) >= 64 or b"\0" in raw or name in seen:
            raise FireFormatError(f"invalid or duplicate tensor name {name!r}")
        seen.add(name)
        dt = wire_dtype(arr)
        if version == 1 and dt != FP32:
            raise FireFormatError("v1 holds FP32 payloads only")
        if arr.ndim not in (1, 2) or any(d <= 0 for d in arr.shape):
            raise FireFormatError(f"invalid shape for {name}: {arr.shape}")
        if group:
            if version != 2 or dt != UINT8 or arr.ndim != 2 or group % 2 or \
                    (2 * arr.shape[1]) % group:
                raise FireFormatError(f"invalid quantization metadata for {name}")
        if version == 2:
            off = (off + 3) & ~3
        size = math.prod(arr.shape) * _SIZE[dt]
        recs.append(Record(name, dt, tuple(arr.shape), off, size, group))
        off += size
    return recs


def write(path: str, entries: Iterable[Tuple[str, np.ndarray, int]], version: int = 2) -> None:
    """Write a complete container. ``entries``: (name, C-contiguous array, group_size)."""
    entries = [(n, np.ascontiguousarray(a), g) for n, a, g in entries]
    recs = plan(entries, version)
    with open(path, "wb") as f:
        f.write(HEADER.pack(MAGIC, version, len(recs), HEADER.size,
                            HEADER.size + RECORD.size * len(recs)))
        for r in recs:
            meta = struct.pack("<BIB", 1, r.group_size, 0) if r.group_size else bytes(6)
            shape1 = r.shape[1] if len(r.shape) == 2 else 0
            f.write(RECORD.pack(r.name.encode("ascii").ljust(64, b"\0"), r.offset, r.size,
                                r.shape[0], shape1, r.dtype, len(r.shape), meta))
        for r, (_, arr, _) in zip(recs, entries):
            pad = r.offset - f.tell()
            if pad < 0 or pad > 3:
                raise FireFormatError(f"payload offset mismatch for {r.name}")
            f.write(bytes(pad))
            f.write(memoryview(arr.astype(_NP[r.dtype], copy=False)).cast("B"))


class FireFile:
    """Read-only mmap of a validated container; arrays are zero-copy views."""

    def __init__(self, path: str):
        self.path = path
        fd = os.open(path, os.O_RDONLY)
        try:
            size = os.fstat(fd).st_size
            if size < HEADER.size:
                raise FireFormatError("file shorter than the header")
            self._mm = mmap.mmap(fd, size, prot=mmap.PROT_READ)
        finally:
            os.close(fd)
        magic, self.version, count, dir_off, data_off = HEADER.unpack_from(self._mm, 0)
        if magic != MAGIC or self.version not in (1, 2):
            raise FireFormatError("bad magic or unsupported version")
        if dir_off != HEADER.size or data_off != HEADER.size + RECORD.size * count:
            raise FireFormatError("bad directory or data offset")
        self.records: Dict[str, Record] = {}
        self.order: List[str] = []
        expect = data_off
        for i in range(count):
            raw, off, nbytes, s0, s1, dt, nd, meta = RECORD.unpack_from(
                self._mm, HEADER.size + i * RECORD.size)
            name = raw.split(b"\0", 1)[0].decode("ascii")
            if dt not in _SIZE or (self.version == 1 and dt != FP32) or nd not in (1, 2):
                raise FireFormatError(f"bad dtype/rank for {name}")
            shape = (s0,) if nd == 1 else (s0, s1)
            kind, group, reserved = struct.unpack("<BIB", meta)
            if kind == 0:
                if group or reserved:
                    raise FireFormatError(f"bad metadata for {name}")
            elif not (self.version == 2 and kind == 1 and dt == UINT8 and group and
                      group % 2 == 0 and reserved == 0 and nd == 2 and (2 * s1) % group == 0):
                raise FireFormatError(f"invalid quantization metadata for {name}")
            if self.version == 2:
                expect = (expect + 3) & ~3
            if off != expect or nbytes != math.prod(shape) * _SIZE[dt] or off + nbytes > size:
                raise FireFormatError(f"bad payload range for {name}")
            if name in self.records:
                raise FireFormatError(f"duplicate tensor {name}")
            self.records[name] = Record(name, dt, shape, off, nbytes, group if kind else 0)
            self.order.append(name)
            expect = off + nbytes

    def __contains__(self, name: str) -> bool:
        return name in self.records

    def __len__(self) -> int:
        return len(self.records)

    def array(self, name: str) -> np.ndarray:
        r = self.records[name]
        return np.frombuffer(self._mm, dtype=_NP[r.dtype], count=math.prod(r.shape),
                             offset=r.offset).reshape(r.shape)

    def arrays(self) -> Dict[str, np.ndarray]:
        return {n: self.array(n) for n in self.order}
