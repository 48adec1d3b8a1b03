"""Builds libtorchless_b200.so (sm_100a) in place with nvcc.

    python -m torchless_b200.build            # incremental
    python -m torchless_b200.build --force    # rebuild everything

Every translation unit is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); objects go to
torchless_b200/_build/ and the shared library next to this file, so it ships
with the source tree.  nvcc cross-compiles without a GPU.
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
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libtorchless_b200.so")

SOURCES = ["tl_errors.cpp", "tl_ops.cu", "tl_gemv.cu", "tl_attention.cu", "tl_decode.cu", "tl_gemm.cu", "tl_gemm_q8.cu", "tl_prefill.cu", "tl_attn_tc.cu", "tl_batch.cu", "tl_sample.cu", "tl_tokenizer.cu", "tl_model.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _flags():
    return ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                   "-I" + INCLUDE, "-I" + CSRC, "--expt-relaxed-constexpr"]


def _deps(src: str):
    """Headers a source depends on (every header in csrc and include)."""
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs + [os.path.join(CSRC, src)]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, src + ".o")
    if force or _stale(obj, _deps(src)):
        cmd = [nvcc()] + _flags() + ["-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    try:
        build(force=args.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
