"""Builds libacediar_b200.so (all CUDA sources, sm_100a) in-tree.

Usage: python acedia-r_b200/build.py [--force] [--jobs N]

Objects go to acedia-r_b200/_build/, the shared library to
acedia-r_b200/lib/libacediar_b200.so.  A source is recompiled when it or any
header under csrc/ or include/ is newer than its object.
"""
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
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libacediar_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # one rounding per R operator: never contract a*b+c into an fma
    "--fmad=false",
    "-Xcompiler", "-fPIC",
    "-I" + os.path.join(ROOT, "include"),
]


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    hs = []
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in os.listdir(d):
            if f.endswith((".cuh", ".h")):
                hs.append(os.path.join(d, f))
    return hs


def _compile(nvcc, src, obj, verbose):
    cmd = [nvcc] + NVCC_FLAGS + ["-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
    return r.stderr if verbose else ""


def build(force=False, jobs=None, verbose=False):
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), newest_header):
            todo.append((s, o))
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for log in ex.map(lambda so: _compile(nvcc, so[0], so[1], verbose), todo):
                logs.append(log)
    if todo or not os.path.exists(LIB):
        # cuBLAS (contraction launchers only) is opened with dlopen at first use: -ldl, no -lcublas
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs + ["-lcudart", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s%s" % (r.stdout, r.stderr))
    return LIB, "".join(logs)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    a = ap.parse_args()
    lib, log = build(a.force, a.jobs, a.verbose)
    if log:
        sys.stdout.write(log)
    print(lib)
