"""Builds librg_npu.so (all CUDA kernels + the C ABI) in-tree for sm_100a."""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "librg_npu.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is None or not spec.submodule_search_locations:
        raise RuntimeError("NCCL (nvidia-nccl) not found")
    base = list(spec.submodule_search_locations)[0]
    return os.path.join(base, "include"), os.path.join(base, "lib")


def _flags():
    inc, _ = nccl_dirs()
    return ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC",
            "-Xcompiler", "-ffp-contract=off", "-Xptxas", "-v" if os.environ.get("RG_PTXAS_V") else "-O3",
            "-I", os.path.join(ROOT, "include"), "-I", inc]


def _compile(src: str) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    deps = [src] + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        [os.path.join(ROOT, "include", "rg_npu.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC] + ARCH + _flags() + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC] + _flags() + ["-x", "c++", "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if os.environ.get("RG_PTXAS_V"):
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(_compile, srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    _, libdir = nccl_dirs()
    cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + [
        "-L", libdir, "-l:libnccl.so.2", "-Xlinker", "-rpath," + libdir, "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
