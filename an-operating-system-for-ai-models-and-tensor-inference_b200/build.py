"""Build the in-tree native libraries with nvcc / g++ (no PyTorch involved).

Outputs (git-ignored, carried to the GPU box with the tree):
  lib/libmyos_cuda.so   CUDA kernels + the C ABI of include/myos_cuda.h (sm_100a)
  lib/libmyos_synth.so  seeded synthetic weights/prompts (host C++)
  lib/myos              C++ command-line runner mirroring the reference CLI

Usage: python build.py [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")
OBJ = os.path.join(HERE, "lib", "obj")
INCLUDE = os.path.join(REPO, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "-I" + INCLUDE,
                     "--expt-relaxed-constexpr"]


def cutlass_include() -> list:
    """CUTLASS/CuTe header trees (SM100 collectives) vendored in the Python
    environment; only gemm_sm100.cu includes them."""
    import site
    for sp in site.getsitepackages():
        root = os.path.join(sp, "flashinfer", "data", "cutlass")
        if os.path.exists(os.path.join(root, "include", "cutlass", "version.h")):
            return ["-I" + os.path.join(root, "include"),
                    "-I" + os.path.join(root, "tools", "util", "include")]
    raise RuntimeError("CUTLASS headers (sm100 collectives) not found")
CUDA_SOURCES = ["kernels.cu", "engine.cu", "ops.cu", "noalloc.cu",
                "prefill.cu", "gemm_sm100.cu", "safetensors.cpp", "tp.cpp"]
HEADERS = ["common.cuh", "kernels.h", "safetensors.h", "prefill.h",
           "gemm_sm100.h", "tp.h"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd[:3]) + " ...")
    return r


def build(force: bool = False, verbose: bool = False) -> dict:
    os.makedirs(OBJ, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "myos_cuda.h")]
    objs = []
    for src in CUDA_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.rsplit(".", 1)[0] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [nvcc()] + NVCC_FLAGS + ["-c", s, "-o", o]
            if src == "gemm_sm100.cu":
                cmd = [nvcc()] + NVCC_FLAGS + cutlass_include() + [
                    "-DCUTLASS_ENABLE_GDC_FOR_SM100=1", "-c", s, "-o", o]
            if src.endswith(".cpp"):
                cmd = [nvcc()] + NVCC_FLAGS + ["-x", "cu", "-c", s, "-o", o]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            _run(cmd)
    so = os.path.join(LIB, "libmyos_cuda.so")
    if force or _stale(so, objs):
        _run([nvcc()] + ARCH + ["-shared", "-o", so] + objs + ["-lcudart_static", "-lrt", "-ldl",
                                                               "-lpthread"])
    synth_src = os.path.join(HERE, "synth", "synth.cpp")
    synth_so = os.path.join(LIB, "libmyos_synth.so")
    if force or _stale(synth_so, [synth_src]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", "-o", synth_so,
              synth_src, "-lm"])
    cli_src = os.path.join(HERE, "cli", "myos_cli.cpp")
    cli_bin = os.path.join(LIB, "myos")
    if os.path.exists(cli_src) and (force or _stale(cli_bin, [cli_src, so])):
        _run(["g++", "-O2", "-std=c++17", "-I" + INCLUDE, "-o", cli_bin, cli_src,
              "-L" + LIB, "-lmyos_cuda", "-Wl,-rpath,$ORIGIN", "-pthread"])
    return {"cuda": so, "synth": synth_so, "cli": cli_bin}


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    for k, v in out.items():
        print(k, v, os.path.exists(v))
