"""Build ``libgravity_b200.so`` in-tree with nvcc for sm_100a (no GPU needed: nvcc cross-compiles).

    python -m gravityocr_b200.build [--verbose] [--ptxas-info] [--timeline]

Objects go to ``gravityocr_b200/_build/``; the shared library lands next to this file, where ``_lib.py`` loads it.
``--timeline`` builds ``libgravity_b200_timeline.so`` instead: the same kernels compiled with ``-DGR_TIMELINE``, which
record per-CTA globaltimer stamps for ``bench.py case timeline`` (load it with ``GRAVITY_B200_LIB``).
The CUDA runtime is linked shared so the library uses the same runtime (current device, streams) as PyTorch.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgravity_b200.so")
TIMELINE_LIB = os.path.join(HERE, "libgravity_b200_timeline.so")
SOURCES = ["linear.cu", "attention.cu", "attention_tc.cu", "rowwise.cu", "sampling.cu", "capi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc())))


def _compile(src: str, extra: list, verbose: bool, build_dir: str = BUILD) -> str:
    obj = os.path.join(build_dir, os.path.splitext(src)[0] + ".o")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
           "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-c", os.path.join(CSRC, src), "-o", obj,
           *extra]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr, flush=True)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False, timeline: bool = False) -> str:
    build_dir = BUILD + ("_timeline" if timeline else "")
    lib = TIMELINE_LIB if timeline else LIB
    os.makedirs(build_dir, exist_ok=True)
    extra = (["-Xptxas", "-v"] if ptxas_info else []) + (["-DGR_TIMELINE"] if timeline else [])
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, verbose or ptxas_info, build_dir), SOURCES))
    tmp = lib + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-o", tmp, *objs,
           "-Xlinker", "-rpath", "-Xlinker", os.path.join(cuda_home(), "lib64")]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib)
    return lib


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--timeline", action="store_true", help="build the timeline-recording library variant")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_info, a.timeline))
    return 0


if __name__ == "__main__":
    sys.exit(main())
