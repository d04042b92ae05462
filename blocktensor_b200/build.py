"""Build recipe for the sm_100a shared library ``blocktensor_b200/libbt_cuda.so``.

nvcc cross-compiles without a GPU, so this runs on any machine with CUDA 12.8+.
The library is built in-tree so that it travels with the repository snapshot.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libbt_cuda.so")

SOURCES = ["bt_quant.cu", "bt_prims.cu", "bt_engine.cu", "bt_noalloc.cu", "bt_prefill.cu", "bt_batch.cu", "bt_q4.cu", "bt_sample.cu"]
HEADERS = ["bt_attn_mma.cuh", "bt_common.cuh", "bt_gemv.cuh", "bt_gemv_mma.cuh", "bt_ptx.cuh", "bt_attention.cuh", "bt_step.cuh",
           "bt_gemm.cuh", "bt_engine_impl.h", "bt_internal.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"] + ARCH


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int = 0, defines: tuple = ()) -> str:
    """defines: extra preprocessor symbols, e.g. BT_STAGE_TRACE for the step kernel's per-stage
    timeline (a diagnostic build; build it in a copy of the package)."""
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "bt_cuda.h")]
    if not force and not defines and not _stale(LIB, deps):
        return LIB
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    extra = (["-Xptxas", "-v"] if verbose_ptxas else []) + [f"-D{d}" for d in defines]
    procs = []
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(obj)
        cmd = [nvcc(), "-c", os.path.join(CSRC, src), "-o", obj, "-I", os.path.join(ROOT, "include")] + NVCC_FLAGS + extra
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if out.strip():
            sys.stderr.write(out)
        if p.returncode != 0:
            failed = True
            sys.stderr.write(f"nvcc failed on {src}\n")
    if failed:
        raise RuntimeError("CUDA build failed")
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-lcudart"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("--define", action="append", default=[], help="preprocessor symbol (e.g. BT_STAGE_TRACE)")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.ptxas_v, defines=tuple(a.define)))
