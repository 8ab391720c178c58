"""Build the sdvk-b200 CUDA back end (libsdvk_b200.so) in-tree with nvcc for sm_100a.

The library exports the C ABI declared in include/sdvk_cuda.h.  It is built here (nvcc
cross-compiles without a GPU) and the .so travels with the source tree to the GPU machine.

    python -m sdvk_b200.build            # incremental (rebuilds when a source is newer)
    python -m sdvk_b200.build --force
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJDIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libsdvk_b200.so")
HOST = os.path.join(PKG, "host")
ENGINE_LIB = os.path.join(PKG, "libsdvk_engine.so")  # C++ ofc::gpu::Engine mirror over the C ABI
SOURCES = ["sdvk_abi.cu", "gemm_q8.cu", "attention.cu", "block.cu", "collective.cu", "no_alloc.cu", "ingest.cu", "conv.cu", "sampler.cu", "unet.cu", "table.cu"]
HEADERS = ["ptx.cuh", "gemm_q8.cuh", "gemm_q8_2sm.cuh", "attention.cuh", "attention_tc.cuh", "attention_fp32.cuh", "attention_tc_short.cuh", "conv_tc2.cuh", "backend.hpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.splitext(src)[0] + ".o")
    deps = [os.path.join(CSRC, src)] + [os.path.join(CSRC, h) for h in HEADERS]
    deps.append(os.path.join(ROOT, "include", "sdvk_cuda.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= _newest(deps):
        return obj
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", os.path.join(ROOT, "include"),
           "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    if force:
        for f in os.listdir(OBJDIR):
            os.remove(os.path.join(OBJDIR, f))
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), SOURCES))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        # Static cudart keeps the library independent of which libcudart the host process loaded.
        subprocess.run([nvcc(), *ARCH, "-shared", "-Xlinker", "-soname=libsdvk_b200.so", "-o", LIB, *objs, "-lcuda",
                        "-ldl"], check=True)
    build_engine(force)
    return LIB


def build_engine(force: bool = False) -> str:
    """The C++ engine mirror (host/engine.cpp) as libsdvk_engine.so, linked against libsdvk_b200.so."""
    src = os.path.join(HOST, "engine.cpp")
    deps = [src, LIB, os.path.join(ROOT, "include", "sdvk_cuda.h"),
            os.path.join(HOST, "Modules", "GPU", "vk_engine.hpp"), os.path.join(HOST, "Modules", "GPU", "fused_attn.hpp"),
            os.path.join(HOST, "Modules", "GPU", "gpu_ops.hpp")]
    if force or not os.path.exists(ENGINE_LIB) or os.path.getmtime(ENGINE_LIB) < _newest(deps):
        cxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else (shutil.which("g++") or "g++")
        subprocess.run([cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"), "-I", HOST,
                        "-o", ENGINE_LIB, src, "-L", PKG, "-lsdvk_b200", "-Wl,-rpath,$ORIGIN"], check=True)
    return ENGINE_LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage per kernel")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose_ptxas=args.ptxas_v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
