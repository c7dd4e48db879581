"""Compile the in-tree CUDA library ``liblvsa_b200.so`` for sm_100a.

``python -m longvideosparseattention_b200.build`` (or ``__graft_entry__.build()``)
runs nvcc on ``csrc/*.cu`` and writes the shared library next to this file, so
it travels with the source tree.  A stamp file beside the library holds a
SHA-256 of every source, header and nvcc flag it was built from; the library
is rebuilt whenever that digest differs (never trusted by modification time,
since the library is shipped alongside the sources and its mtime says nothing).
"""

import glob
import hashlib
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "liblvsa_b200.so")
STAMP = LIB + ".sha256"
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-shared", "-Xcompiler", "-fPIC", "-Xptxas", "-v", "--expt-relaxed-constexpr"]


def sources():
    return sorted(glob.glob(os.path.join(PKG, "csrc", "*.cu")))


def _deps():
    return sources() + sorted(glob.glob(os.path.join(PKG, "csrc", "*.cuh"))) + \
        sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def source_digest() -> str:
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for p in _deps():
        h.update(os.path.relpath(p, ROOT).encode())
        with open(p, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def up_to_date() -> bool:
    if not (os.path.exists(LIB) and os.path.exists(STAMP)):
        return False
    with open(STAMP) as fh:
        return fh.read().strip() == source_digest()


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), *sources(), "-o", LIB + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    with open(STAMP, "w") as fh:
        fh.write(source_digest() + "\n")
    if verbose:
        print(r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
