"""Build ``libmie.so`` in-tree with nvcc for sm_100a (B200).

    python -m moe_engine.build          # from moe-inference-engine_b200/

The library is written to ``moe_engine/_native/libmie.so``; it carries no
torch dependency (plain C ABI, static CUDA runtime).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
OUT_DIR = os.path.join(PKG, "_native")
OUT = os.path.join(OUT_DIR, "libmie.so")
SOURCES = ["capi.cu", "moe.cu", "moe_q.cu", "attention.cu", "gemv.cu", "step.cu", "step_wide.cu", "step_cluster.cu", "gemm.cu",
           "prefill.cu", "peer.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs():
    files = [os.path.join(CSRC, s) for s in SOURCES]
    files += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    files.append(os.path.join(INCLUDE, "mie.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every source to an object file (in parallel), then link the
    shared library; returns its path."""
    if not force and up_to_date():
        return OUT
    from concurrent.futures import ThreadPoolExecutor

    os.makedirs(OUT_DIR, exist_ok=True)
    obj_dir = os.path.join(OUT_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    tmp = OUT + ".tmp"
    # MIE_NVCC_FLAGS adds flags, e.g. "-DMIE_DEBUG_CHECKS" for the self-checking build.
    extra = os.environ.get("MIE_NVCC_FLAGS", "").split()
    common = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", *extra, "-I", INCLUDE]
    if verbose:
        common.insert(1, "-Xptxas=-v")

    def compile_one(src: str):
        obj = os.path.join(obj_dir, os.path.splitext(src)[0] + ".o")
        cmd = [*common, "-c", "-o", obj, os.path.join(CSRC, src)]
        return obj, subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(max_workers=max(1, min(len(SOURCES), os.cpu_count() or 1))) as pool:
        results = list(pool.map(compile_one, SOURCES))
    objs = []
    for (obj, res), src in zip(results, SOURCES):
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src} ({res.returncode}):\n{res.stdout}\n{res.stderr}")
        if verbose:
            print(src, res.stderr)
        objs.append(obj)
    res = subprocess.run([nvcc(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    for obj in objs:
        os.remove(obj)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
