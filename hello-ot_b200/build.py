"""Build libhello_b200.so in-tree with nvcc for sm_100a.

    python hello-ot_b200/build.py [--force]

Each CUDA source compiles to an object under hello-ot_b200/_build/ (in
parallel) and the objects link into hello-ot_b200/libhello_b200.so with the
CUDA runtime linked statically.  pdlp.cu is compiled without fma contraction
so the PDHG update arithmetic matches the reference operation by operation;
exact.cu likewise, so its fp64 scores round like the written expressions.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libhello_b200.so"
INCLUDE = HERE.parent / "include"
SOURCES = ["abi.cu", "scan_l2sq.cu", "scan_norm.cu", "pairs.cu", "pdlp.cu", "support.cu", "exact.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + str(INCLUDE), "-Xptxas", "-warn-spills"]
PER_FILE = {"pdlp.cu": ["-fmad=false"], "exact.cu": ["-fmad=false"]}


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libhello_b200.so")
    return path


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    jobs = []
    for src in SOURCES:
        obj = BUILD / (src + ".o")
        if force or _stale(obj, [CSRC / src, *headers, Path(__file__)]):
            cmd = [cc, *ARCH, *FLAGS, *PER_FILE.get(src, []), "-c", str(CSRC / src), "-o", str(obj)]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = []
    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4) or 1) as pool:
        for src, r in pool.map(run, jobs):
            out = (r.stdout + r.stderr).strip()
            if r.returncode != 0:
                failed.append(f"--- {src}\n{out}")
            elif verbose and out:
                print(out)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    objs = [BUILD / (s + ".o") for s in SOURCES]
    if force or jobs or _stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
