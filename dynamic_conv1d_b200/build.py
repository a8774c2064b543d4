"""Build libdynconv.so in-tree with nvcc for sm_100a (B200).

    python -m dynamic_conv1d_b200.build        # or: python dynamic_conv1d_b200/build.py

Compiles every ``csrc/*.cu`` into ``dynamic_conv1d_b200/libdynconv.so`` (position
independent, static CUDA runtime, no libcuda link: the TMA tensor-map encoder is
fetched through cudaGetDriverEntryPoint at run time).  Objects go to
``dynamic_conv1d_b200/_build/``; a source is recompiled only when it or a header
changed.  The built library is git-ignored but travels with the repository
snapshot to the GPU box.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdynconv.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I" + os.path.join(ROOT, "include"),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set $NVCC)")


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(nvcc: str, src: str, obj: str, extra: list[str]) -> str:
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}\n{r.stdout}")
    return r.stderr


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_t = _headers_mtime()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        if force or ptxas_info or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_t):
            jobs.append((s, o))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, nvcc, s, o, extra): s for s, o in jobs}
            for f in cf.as_completed(futs):
                msg = f.result()
                if verbose and msg:
                    print(f"== {os.path.basename(futs[f])}\n{msg}", file=sys.stderr)
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}\n{r.stdout}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem per kernel")
    a = ap.parse_args()
    print(build(verbose=True, force=a.force, ptxas_info=a.ptxas_info))
