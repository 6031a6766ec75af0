"""Builds the native libraries in-tree.

- ``wcb/libwcb.so``: the CUDA kernels and the C++ host runtime behind
  ``include/wcb.h``, compiled by nvcc for sm_100a only.
- ``wcb/libwcb_synth.so``: the host-only synthetic-model generator.

Run ``python -m wcb.build`` (with ``wasm-chord_b200`` on ``sys.path``) or call
``build_all()``. Objects go to ``wasm-chord_b200/_build``; a target is rebuilt
when any of its sources or headers is newer.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)  # wasm-chord_b200
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libwcb.so")
SYNTH_LIB = os.path.join(PKG, "libwcb_synth.so")

CUDA_SOURCES = ["kernels.cu", "gemm_tc.cu", "decode_step.cu", "noalloc.cu", "batch_decode.cu", "attn_prefill.cu", "sample_dev.cu"]
HOST_SOURCES = ["gguf.cpp", "sampler.cpp", "model.cpp", "api.cpp", "nccl_rt.cpp", "tokenizer.cpp"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(REPO, "include", "wcb.h"))
    return hs


def _stale(target, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build_synth(verbose: bool = False) -> str:
    src = os.path.join(CSRC, "synth.cpp")
    if _stale(SYNTH_LIB, [src]):
        cxx = os.environ.get("CXX", "g++")
        _run([cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", "-o", SYNTH_LIB + ".tmp", src])
        os.replace(SYNTH_LIB + ".tmp", SYNTH_LIB)
        if verbose:
            print("built", SYNTH_LIB)
    return SYNTH_LIB


def build_lib(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    hdrs = _headers()
    common = ["-std=c++17", "-O3", "-Xcompiler", "-fPIC", "-I", os.path.join(REPO, "include")]
    jobs = []
    objs = []
    for f in CUDA_SOURCES + HOST_SOURCES:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if not _stale(obj, [src] + hdrs):
            continue
        cmd = [nvcc] + common + GENCODE + ["-c", src, "-o", obj]
        if f.endswith(".cu"):
            cmd += ["-lineinfo", "--expt-relaxed-constexpr"]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
        else:
            cmd += ["-x", "c++"]
        jobs.append(cmd)
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for r in ex.map(_run, jobs):
                if verbose and (r.stdout or r.stderr):
                    print(r.stdout, r.stderr, file=sys.stderr)
    if jobs or _stale(LIB, objs):
        _run([nvcc, "-shared"] + GENCODE + ["-o", LIB + ".tmp"] + objs + ["-ldl", "-lpthread"])
        os.replace(LIB + ".tmp", LIB)
        if verbose:
            print("built", LIB)
    return LIB


def build_all(verbose: bool = False) -> None:
    build_synth(verbose)
    build_lib(verbose)


if __name__ == "__main__":
    build_all(verbose=True)
