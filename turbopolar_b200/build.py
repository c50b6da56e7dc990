"""Build ``libturbopolar.so`` (C ABI, sm_100a) in-tree with nvcc.

``python -m turbopolar_b200.build`` or ``turbopolar_b200.build.build()``.  The library has
no PyTorch dependency; Python loads it with ctypes.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libturbopolar.so")
SOURCES = ["tp_encode.cu", "tp_attention.cu", "tp_misc.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; cannot build libturbopolar.so")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(HERE, "..", "include", "turbopolar.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    if not force and not _stale():
        return LIB
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []), "-o", LIB + ".tmp",
           *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, flush=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    flags = [a for a in sys.argv[1:] if a.startswith("-")]
    print(build(force=True, verbose=True, extra_flags=flags))
