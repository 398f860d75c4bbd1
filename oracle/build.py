"""Builds the CPU oracle library ``oracle/_build/libdsa_oracle.so`` with gcc (test infrastructure).

``-ffp-contract=off`` keeps the float32 coordinate arithmetic un-fused, so it rounds exactly like
the reference's float32 CPU path; ``-march=x86-64-v3`` (AVX2/FMA baseline) keeps the binary
runnable on any current x86-64 host, including the GPU box.
"""

from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "dsa_oracle.c"
OUT = HERE / "_build" / "libdsa_oracle.so"
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-std=gnu11"]


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if not force and OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc not found")
    subprocess.run([cc, *CFLAGS, str(SRC), "-o", str(OUT), "-lm"], check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
