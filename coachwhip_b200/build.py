"""Builds libcwx.so (the CUDA library behind include/cwx.h) in-tree, for sm_100a.

Each source under csrc/ is compiled separately with nvcc (gguf.cpp, host code only, as CUDA too)
and linked into one shared library next to this file. bank.cu (synthetic-bank quantisers) is
compiled with -fmad=false so its f32 arithmetic rounds step by step like the CPU code it mirrors.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libcwx.so")
SOURCES = ["api.cu", "bank.cu", "route.cu", "gemv.cu", "act.cu", "noalloc.cu", "mma.cu", "ep.cu", "ep_nccl.cu",
           "decode_layer.cu", "gdn.cu", "attn.cu", "gguf.cpp"]
NO_FMA = {"bank.cu"}
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    inc = os.path.join(HERE, "..", "include")
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(inc, "cwx.h"))
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs, cmds = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(objdir, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        if not force and not _stale(obj, [path] + headers):
            continue
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", inc, "-I", CSRC,
               "--expt-relaxed-constexpr", "-x", "cu", "-c", path, "-o", obj]
        if src in NO_FMA:
            cmd.insert(1, "-fmad=false")
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
    # the sources compile independently: one nvcc per source, in parallel (the longest, gemv.cu
    # with its per-format instantiations, sets the build time)
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as pool:
        for r in list(pool.map(lambda c: subprocess.run(c, capture_output=not verbose, text=True), cmds)):
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed ({r.returncode}): {' '.join(r.args)}\n{r.stdout or ''}{r.stderr or ''}")
    if force or _stale(LIB, objs):
        subprocess.run([nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-ldl"], check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
