"""Build ``libkab.so``, the library's CUDA code for sm_100a, in-tree with nvcc.

    python kernel-agent_b200/build.py [--force] [--verbose]

Objects go to ``kernel-agent_b200/_build/``; the library to
``kernel-agent_b200/kernel_agent_b200/_native/libkab.so`` (it travels with the source tree
to a GPU machine; no JIT cache is involved). Translation units compile in parallel and
only when a source or header changed.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
OUT = HERE / "kernel_agent_b200" / "_native" / "libkab.so"
SOURCES = ["kab_core.cu", "kab_quant.cu", "kab_compare.cu", "kab_gemm.cu", "kab_attention.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libkab.so")
    return found


def _headers_mtime() -> float:
    paths = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((p.stat().st_mtime for p in paths), default=0.0)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile what changed and link ``libkab.so``; returns its path."""
    BUILD.mkdir(exist_ok=True)
    OUT.parent.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    exe = nvcc()
    jobs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (Path(src).stem + ".o")
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr):
            cmd = [exe, *FLAGS, "-c", str(s), "-o", str(o)]
            if ptxas_info:
                cmd[1:1] = ["-Xptxas", "-v"]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = []
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as pool:
        for src, r in pool.map(run, jobs):
            if verbose or r.returncode:
                sys.stdout.write(r.stdout)
                sys.stderr.write(r.stderr)
            if r.returncode:
                failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed on {', '.join(failed)}")
    objs = [str(BUILD / (Path(s).stem + ".o")) for s in SOURCES]
    newest = max(Path(o).stat().st_mtime for o in objs)
    if force or jobs or not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = [exe, *ARCH, "-shared", "-o", str(OUT), *objs, "-lcuda" if False else "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("linking libkab.so failed")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="pass -Xptxas -v (registers, spills)")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_info))
