"""Build ``libturbopolar.so`` (C ABI, sm_100a) in-tree with nvcc.

``python -m turbopolar_b200.build`` or ``turbopolar_b200.build.build()``.  The library has
no PyTorch dependency; Python loads it with ctypes.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libturbopolar.so")
STAMP = LIB + ".stamp"
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


def _deps():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)) + [os.path.join(HERE, "..", "include", "turbopolar.h")]


def source_hash(extra_flags=None) -> str:
    """SHA-256 (first 16 hex digits) of the library's sources, header and nvcc flags."""
    h = hashlib.sha256()
    for d in _deps():
        if os.path.exists(d):
            h.update(os.path.basename(d).encode())
            with open(d, "rb") as f:
                h.update(f.read())
    h.update(" ".join([*NVCC_FLAGS, *(extra_flags or [])]).encode())
    return h.hexdigest()[:16]


# What the last build() call in this process did: the sources' hash and whether it ran nvcc.
last_build = {"source_sha16": None, "compiled": None}


def _stamped(want: str) -> bool:
    try:
        with open(STAMP) as f:
            return os.path.exists(LIB) and f.read().strip() == want
    except OSError:
        return False


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile the library unless the one in place was built from exactly these sources and
    flags (the hash in libturbopolar.so.stamp, written beside the library)."""
    want = source_hash(extra_flags)
    last_build.update(source_sha16=want, compiled=False)
    if not force and _stamped(want):
        if verbose:
            print(f"{LIB}: up to date (sources {want})", flush=True)
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
    with open(STAMP, "w") as f:
        f.write(want + "\n")
    last_build["compiled"] = True
    return LIB


if __name__ == "__main__":
    flags = [a for a in sys.argv[1:] if a.startswith("-")]
    print(build(force=True, verbose=True, extra_flags=flags))
