"""Build ``libomniwave_b200.so`` (the C-ABI library) in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into
``omniwave_b200/libomniwave_b200.so``.  Objects go to ``omniwave_b200/_build``;
files whose sources and headers are older than their object are not rebuilt.

Usage: ``python -m omniwave_b200.build [--force] [--verbose]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libomniwave_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", INCLUDE, "-I", CSRC,
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; set NVCC or put CUDA on PATH")
    return cand


def _headers() -> list[str]:
    out = [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return out


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compile and link the library; returns its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    headers = _headers()
    extra = list(extra or [])
    jobs = []
    objects = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objects.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append([nvcc, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, sep="\n", flush=True)

    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objects):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objects, "-lcudart"]
        run(cmd)
    return LIB


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print register/smem usage")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    print(build(force=a.force or a.ptxas_verbose, verbose=a.verbose or a.ptxas_verbose, extra=extra))


if __name__ == "__main__":
    main(sys.argv[1:])
