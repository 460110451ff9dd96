"""Build the native library libda3b.so in-tree (sm_100a only).

Every CUDA/C++ source under csrc/ is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared object
next to this file, so the built library travels with the source tree. Objects
are rebuilt only when a source or header is newer than its object.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
INCLUDE = os.path.join(ROOT, "include")
OBJDIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libda3b.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE,
]


# Per-file extra flags. raypose.cu's double arithmetic must round like the reference's
# host code, so no multiply-add contraction there.
FILE_FLAGS = {"raypose.cu": ["-fmad=false"]}


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    out = []
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, f))
    return out


def _headers_mtime() -> float:
    m = 0.0
    for d in (CSRC, INCLUDE, os.path.join(INCLUDE, "da3cpp")):
        if not os.path.isdir(d):
            continue
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def build(verbose: bool = False, force: bool = False) -> str:
    nvcc = _nvcc()
    os.makedirs(OBJDIR, exist_ok=True)
    hdr = _headers_mtime()
    jobs = []
    objs = []
    for src in _sources():
        obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr):
            extra = FILE_FLAGS.get(os.path.basename(src), [])
            cmd = [nvcc] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
            if src.endswith(".cpp"):
                cmd = [nvcc] + NVCC_FLAGS + extra + ["-x", "cu", "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(run, jobs))
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread", "-ldl"]
        run(cmd)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
