"""Build libcxkv.so in-tree with nvcc for sm_100a.

    python -m chenxing_b200.build

The library is one translation unit (csrc/cxkv.cu includes the parts), linked
against the static CUDA runtime, so it only needs the NVIDIA driver at run
time.  Rebuilds unless the stamp file beside the library records the SHA-256
of exactly the current sources, headers, nvcc flags and nvcc version (file
times are not trusted: a library copied along with the tree keeps them).
"""
from __future__ import annotations

import glob
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libcxkv.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-shared", "-Xcompiler", "-fPIC,-O2",
         "-Xptxas", "-v"]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) +
                  glob.glob(os.path.join(HERE, "csrc", "*.cuh")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(home, "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


STAMP = LIB + ".sha256"


def nvcc_version() -> str:
    try:
        return subprocess.run([nvcc(), "--version"], capture_output=True, text=True).stdout
    except OSError:
        return "nvcc missing"


def content_hash() -> str:
    """SHA-256 over every source and header (path and bytes), the nvcc
    command-line flags and the nvcc version."""
    h = hashlib.sha256()
    for path in sources():
        h.update(os.path.relpath(path, ROOT).encode())
        with open(path, "rb") as f:
            h.update(f.read())
    h.update(repr((ARCH, FLAGS)).encode())
    h.update(nvcc_version().encode())
    return h.hexdigest()


def up_to_date() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(STAMP):
        return False
    with open(STAMP) as f:
        return f.read().strip() == content_hash()


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    digest = content_hash()
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", os.path.join(ROOT, "include"),
           os.path.join(HERE, "csrc", "cxkv.cu"), "-o", tmp]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed to build libcxkv.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    with open(STAMP, "w") as f:
        f.write(digest + "\n")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
