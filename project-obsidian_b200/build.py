"""Build libobsmoe.so (the sm_100a MoE hot path) in-tree with nvcc.

    python project-obsidian_b200/build.py [--verbose-ptxas]

Each .cu file under csrc/ is compiled for sm_100a only and linked into one
shared library next to this file; the C ABI is include/obs_moe.h.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libobsmoe.so")
BUILD = os.path.join(HERE, "_build")
SOURCES = ["obs_api.cu", "obs_static.cu", "obs_safetensors.cu", "k_synth.cu", "k_router.cu", "k_dispatch.cu",
           "k_decode.cu", "k_gemm.cu", "k_ep.cu", "k_head.cu", "k_attn.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "obs_moe.h"))
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                    "-I", os.path.join(ROOT, "include")]
    if verbose_ptxas:
        flags += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or verbose_ptxas or _stale(o, [s] + headers):
            cmd = [nvcc(), "-c", s, "-o", o] + flags
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0 or verbose_ptxas:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}")
    if force or _stale(OUT, objs):
        cmd = [nvcc(), "-shared", "-o", OUT] + objs + ARCH + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.force))
