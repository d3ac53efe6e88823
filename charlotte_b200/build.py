"""Builds libcharlotte_b200.so in-tree from charlotte_b200/csrc with nvcc for
sm_100a. `python -m charlotte_b200.build` or charlotte_b200.build.build()."""
from __future__ import annotations

import concurrent.futures
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcharlotte_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

# sm_100a only. --fmad=false: only explicit fmaf() fuses, so each kernel's
# order of operations is the one its source states (numerics.cuh).
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--fmad=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_digest() -> str:
    h = hashlib.sha256()
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".h", ".cuh")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(f.encode() + fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def _compile(src: str, digest: str) -> str:
    # An object is named by the digest of its own source, every header and
    # the flags: a name that exists was compiled from exactly these bytes,
    # whatever the files' times say (a copy of the tree keeps no mtimes).
    with open(src, "rb") as fh:
        own = hashlib.sha256(digest.encode() + fh.read()).hexdigest()[:16]
    obj = os.path.join(OBJ, os.path.basename(src) + "." + own + ".o")
    if os.path.exists(obj):
        return obj
    cmd = [NVCC, *NVCC_FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    digest = _headers_digest()
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, digest), srcs))
    # objects of earlier header or flag states are never linked again
    keep = {os.path.basename(o) for o in objs}
    for f in os.listdir(OBJ):
        if f.endswith(".o") and f not in keep:
            os.remove(os.path.join(OBJ, f))
    # The library is relinked unless its stamp names exactly these objects.
    stamp = LIB + ".objects"
    want = "\n".join(sorted(keep))
    have = open(stamp).read() if os.path.exists(stamp) and os.path.exists(LIB) else None
    if have != want:
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
               *objs, "-o", LIB]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        with open(stamp, "w") as fh:
            fh.write(want)
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
