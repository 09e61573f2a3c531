"""Builds libkta_b200.so in-tree from kta_b200/csrc/*.cu with nvcc for sm_100a.

``python -m kta_b200.build [-v] [--ptxas]`` compiles every translation unit in parallel into
``kta_b200/_build/`` and links ``kta_b200/libkta_b200.so``. The library links only the
static CUDA runtime; tensor maps come from the driver through cudaGetDriverEntryPoint, so no
libcuda, cuBLAS or torch library is linked (the anti-cheat rule of
src/kta/checks/anticheat.py:38-58 in the reference).
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libkta_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps_hash(src: Path, extra: list[str]) -> str:
    h = hashlib.sha256()
    h.update(" ".join(ARCH + FLAGS + extra).encode())
    h.update(src.read_bytes())
    for hdr in sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")]):
        h.update(hdr.read_bytes())
    return h.hexdigest()[:16]


def _compile(src: Path, extra: list[str], verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    stamp = BUILD / (src.stem + ".hash")
    key = _deps_hash(src, extra)
    if obj.exists() and stamp.exists() and stamp.read_text() == key:
        return obj, ""
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    stamp.write_text(key)
    return obj, res.stdout + res.stderr


def build(verbose: bool = False, ptxas: bool = False) -> Path:
    """Compiles and links the library; returns its path. Raises on any compiler error."""
    BUILD.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas else []
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(lambda s: _compile(s, extra, verbose), srcs))
    for _, log in results:
        if ptxas and log:
            print(log)
    objs = [str(o) for o, _ in results]
    newest = max(Path(o).stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def main(argv: list[str]) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v resource usage")
    args = ap.parse_args(argv)
    path = build(args.verbose, args.ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
