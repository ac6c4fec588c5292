"""Build libqsa.so in-tree with nvcc for sm_100a (and the CPU oracle with make).

    python -m qwfnfer_b200.build [--verbose]

The library links the CUDA runtime statically, so it loads beside PyTorch's own runtime without
a version clash; it shares the driver's primary context with it, so PyTorch streams and device
pointers are valid arguments.  No fast-math: the pooled-key arithmetic (sqrt, divide, rounding)
must be IEEE to match the reference's CPU rounding.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
SOURCES = ["qsa_api.cu", "qsa_append.cu", "qsa_select.cu", "qsa_attn.cu", "qsa_shard.cu", "qsa_prefill_tc.cu", "qsa_prefill_attn.cu", "qsa_peer.cu", "qsa_static_ws.cu", "qsa_stage.cu", "qsa_front.cu", "qsa_proj_gemm.cu", "qsa_gguf.cpp", "qsa_shard_nccl.cu"]
OUT = os.path.join(PKG, "libqsa.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def host_cxx() -> str:
    # the system g++ (the image's /opt/gcc wrapper lacks OpenMP specs; nvcc only needs a C++17 host compiler)
    return "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"


def build_lib(verbose: bool = False) -> str:
    objs = []
    bdir = os.path.join(PKG, "_build")
    os.makedirs(bdir, exist_ok=True)
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-ccbin", host_cxx(),
             "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")] + ARCH
    if verbose:
        flags += ["-Xptxas", "-v"]
    for src in SOURCES:
        obj = os.path.join(bdir, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        path = os.path.join(CSRC, src)
        deps = [path] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")] + \
               [os.path.join(ROOT, "include", "qsa.h")]
        if os.path.exists(obj) and all(os.path.getmtime(obj) >= os.path.getmtime(p) for p in deps) and not verbose:
            continue
        cmd = [nvcc(), "-c", path, "-o", obj] + flags
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
    cmd = [nvcc(), "-shared", "-o", OUT] + objs + ARCH + ["-ccbin", host_cxx(), "-cudart", "static", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link of libqsa.so failed")
    return OUT


def build_oracle() -> str:
    r = subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("oracle build failed")
    return os.path.join(ROOT, "oracle", "libqsa_oracle.so")


def main() -> None:
    verbose = "--verbose" in sys.argv
    print(build_lib(verbose))
    print(build_oracle())


if __name__ == "__main__":
    main()
