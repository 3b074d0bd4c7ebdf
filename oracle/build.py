"""Build the oracle's C restatement (oracle/conv.c) into oracle/_build/liboracle.so with gcc and OpenMP.

    python -m oracle.build

Test infrastructure and the CPU baseline only: the library's product path never loads it.  Compiled for x86-64-v3
(AVX2/FMA), not -march=native, so a build made on one host runs on the GPU hosts as well.
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "liboracle.so"
SRC = [HERE / "conv.c"]


def build(force: bool = False) -> Path | None:
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        return None
    if not force and OUT.exists() and OUT.stat().st_mtime >= max(s.stat().st_mtime for s in SRC):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [cc, "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-o", str(tmp), *map(str, SRC)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
