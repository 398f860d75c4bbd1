"""Builds libmegaslide_b200.so (sm_100a) in-tree with nvcc.

Usage: ``python -m megaslide_b200.build [--force] [--verbose]``.  The library lands in
``megaslide_b200/lib/`` next to the package so it travels with the source tree; object files go to
``megaslide_b200/_build/``.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJDIR = PKG / "_build"
LIBDIR = PKG / "lib"
LIBNAME = "libmegaslide_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-O3,-fopenmp",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def lib_path() -> Path:
    return LIBDIR / LIBNAME


def stamp_path() -> Path:
    return LIBDIR / (LIBNAME + ".srchash")


def source_hash() -> str:
    """sha256 over every source, header and flag the library is built from: the stamp that ties a built
    library to the sources it came from (file times do not survive copies to another machine)."""
    h = hashlib.sha256()
    for p in sorted(CSRC.glob("*.cu")) + _headers():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def is_current() -> bool:
    """True when the built library exists and was built from the present sources."""
    try:
        return lib_path().exists() and stamp_path().read_text().strip() == source_hash()
    except OSError:
        return False


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every ``csrc/*.cu`` for sm_100a and links the shared library; returns its path.  Object
    files are reused only while the library's source stamp matches the sources (else everything is
    recompiled)."""
    nvcc = _nvcc()
    OBJDIR.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    want = source_hash()
    if not is_current():
        force = True
    hdr_mtime = max((p.stat().st_mtime for p in _headers()), default=0.0)
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = OBJDIR / (src.stem + ".o")
        objs.append(obj)
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
            continue
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    out = lib_path()
    if force or not out.exists() or out.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC,-fopenmp", *map(str, objs), "-o", str(out), "-lgomp"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    stamp_path().write_text(want + "\n")
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
