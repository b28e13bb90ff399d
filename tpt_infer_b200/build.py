"""Builds ``libtpt_cuda.so`` (the C-ABI library declared in include/tpt_cuda.h)
in-tree for sm_100a with nvcc.

Every ``csrc/*.cu`` file is compiled to an object under ``_build/`` (in
parallel, skipped when up to date) and linked into
``tpt_infer_b200/libtpt_cuda.so``. No fast-math: the quantizers and the W8A8
epilogue rely on IEEE division and separately rounded multiply/add.

    python tpt_infer_b200/build.py [--force] [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libtpt_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _host_cxx() -> str:
    for cand in ("/usr/bin/g++-13", "/usr/bin/g++", shutil.which("g++")):
        if cand and os.path.exists(cand):
            return cand
    return "g++"


def _flags(verbose_ptxas: bool):
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                "-I", os.path.join(ROOT, "include"), "-ccbin", _host_cxx()]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "tpt_cuda.h")]
    hdr_time = _newest(headers)
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or verbose_ptxas or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_time):
            jobs.append([nvcc(), *_flags(verbose_ptxas), "-c", s, "-o", o])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = False
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for cmd, r in ex.map(run, jobs):
                out = (r.stdout + r.stderr).strip()
                if r.returncode != 0:
                    failed = True
                    sys.stderr.write(f"FAILED: {' '.join(cmd)}\n{out}\n")
                elif out:
                    sys.stderr.write(out + "\n")
    if failed:
        raise RuntimeError("nvcc compilation failed")
    if force or jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-ccbin", _host_cxx()]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {r.stdout}{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose_ptxas))
