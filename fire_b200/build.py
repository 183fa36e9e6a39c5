"""Build the fire_b200 native library in-tree for sm_100a.

    python -m fire_b200.build          # -> fire_b200/libfire_b200.so

Each source compiles to its own object under fire_b200/_build (rebuilt only when the
source or a header changed), then nvcc links one shared library. The library is
in-tree on purpose: it travels with the repository snapshot to the GPU machine.
"""
from __future__ import annotations

import glob
import hashlib
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(PKG, "libfire_b200.so")
BUILD = os.path.join(PKG, "_build")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCLUDES = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True) +
                  glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True) +
                    glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True) +
                    glob.glob(os.path.join(ROOT, "include", "*.h"))):
        h.update(p.encode())
        h.update(open(p, "rb").read())
    return h.hexdigest()[:16]


def _compile(src: str, digest: str) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    sh = hashlib.sha256(open(src, "rb").read() + digest.encode()).hexdigest()[:16]
    obj = os.path.join(BUILD, f"{rel}.{sh}.o")
    if not os.path.exists(obj):
        cmd = [NVCC, *ARCH, *NVFLAGS, *INCLUDES, "-c", src, "-o", obj]
        if src.endswith(".cpp"):
            cmd = [NVCC, *NVFLAGS, *INCLUDES, "-x", "c++", "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    digest = _headers_digest()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(lambda s: _compile(s, digest), _sources()))
    stamp = hashlib.sha256("".join(objs).encode()).hexdigest()[:16]
    stamp_path = os.path.join(BUILD, "link.stamp")
    if os.path.exists(OUT) and os.path.exists(stamp_path) and open(stamp_path).read() == stamp:
        return OUT
    cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-L" + os.path.join(CUDA, "lib64"), "-lcudart",
           "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
    with open(stamp_path, "w") as f:
        f.write(stamp)
    # drop objects of sources that no longer exist or changed
    keep = set(objs)
    for o in glob.glob(os.path.join(BUILD, "*.o")):
        if o not in keep:
            os.remove(o)
    if verbose:
        print("built", OUT)
    return OUT


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
