"""Build the in-tree CUDA library ``promptmoge_b200/libpmg_b200.so`` for sm_100a with nvcc.

    python -m promptmoge_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (rebuilt when it or a header changed) and linked into
one shared library exposing the C ABI of ``include/pmg_b200.h``.  No JIT cache: the .so lives next to this file so it
travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libpmg_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the B200 library needs the CUDA toolkit to build")


def flags(extra=()) -> list:
    return ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=default",
                   f"-I{ROOT / 'include'}", f"-I{CSRC}", "--expt-relaxed-constexpr", *extra]


def _compile(src: Path, obj: Path, verbose: bool, extra=()) -> None:
    cmd = [nvcc(), *flags(extra), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr)


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
        if stale:
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, verbose, extra) for s, o in jobs]
            for f in futs:
                f.result()
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart", "-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / shared-memory usage per kernel")
    a = ap.parse_args()
    extra = ("-Xptxas", "-v") if a.ptxas_v else ()
    lib = build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra)
    print(lib)


if __name__ == "__main__":
    sys.exit(main())
