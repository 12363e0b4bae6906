"""Build libds_kernels_sm100.so in-tree with nvcc for sm_100a.

    python deepseek-v2-lite-cuda_b200/build.py [--verbose]

Objects go to deepseek-v2-lite-cuda_b200/_build/, the shared library to
deepseek-v2-lite-cuda_b200/ds_kernels/libds_kernels_sm100.so.  The library is plain CUDA
C++ with a C ABI (include/ds_kernels.h); it links the CUDA runtime statically and does not
depend on torch.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "ds_kernels", "libds_kernels_sm100.so")

SOURCES = ["common.cu", "moe_kernels.cu", "mla_kernels.cu", "gemm_sm100.cu", "moe_layer.cu",
           "moe_noalloc.cu", "moe_stages.cu", "ep_p2p.cu", "mla_attention.cu", "mla_decode.cu"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")
    return cand


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)
    return obj


def _stale(objs_and_srcs) -> bool:
    if not os.path.exists(LIB):
        return True
    lib_t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(ROOT, "include", "ds_kernels.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > lib_t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    """Compile every source for sm_100a and link the shared library; returns its path."""
    if not force and not _stale(None):
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static",
           "-Xcompiler", "-fPIC", "-Xlinker", "--no-undefined"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="pass -Xptxas -v")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
