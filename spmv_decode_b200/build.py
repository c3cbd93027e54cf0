"""Build libnmsparse_b200.so in-tree with nvcc for sm_100a.

The library is one CUDA translation unit (csrc/nms_lib.cu) compiled with
``-gencode arch=compute_100a,code=sm_100a``; it links only the CUDA runtime.
No JIT cache is involved, so the built file travels with the source tree.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "lib" / "libnmsparse_b200.so"
INCLUDE = PKG.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build libnmsparse_b200)")
    return cand


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + [INCLUDE / "nmsparse_b200.h"])


def source_hash() -> str:
    """SHA-256 over the library's sources (names and contents, in order); the
    build embeds it and ``nms_source_hash()`` returns it."""
    h = hashlib.sha256()
    for p in sources():
        h.update(p.name.encode() + b"\0" + p.read_bytes() + b"\0")
    return h.hexdigest()


def built_hash() -> str | None:
    """The hash embedded in the built library, or None if there is none.
    Read in a child process so this process never maps a library it may
    replace a moment later."""
    if not OUT.exists():
        return None
    code = ("import ctypes,sys; L=ctypes.CDLL(sys.argv[1]); f=L.nms_source_hash; "
            "f.restype=ctypes.c_char_p; print(f().decode())")
    res = subprocess.run([sys.executable, "-c", code, str(OUT)], capture_output=True, text=True)
    return res.stdout.strip() if res.returncode == 0 else None


def needs_build() -> bool:
    return built_hash() != source_hash()


def check_current() -> None:
    """Raise if the built library was not built from the current sources."""
    got, want = built_hash(), source_hash()
    if got != want:
        raise RuntimeError(f"{OUT} is stale (built from sources {got}, the tree has {want}); rebuild it with "
                           "`python -m spmv_decode_b200.build`")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library unless it was built from exactly these sources."""
    if not force and not needs_build():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, f"-DNMS_SOURCE_HASH=\"{source_hash()}\"", "-o", str(tmp),
           str(CSRC / "nms_lib.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
