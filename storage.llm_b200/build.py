"""Builds libmoe_b200.so (in this directory) for sm_100a with nvcc.

    python storage.llm_b200/build.py [--debug]

The library is the product: the C ABI of include/moe_b200.h.  It links only
the CUDA runtime (the driver's tensor-map encoder is fetched at run time with
cudaGetDriverEntryPoint, NCCL for the expert-parallel entry points is opened
with dlopen), so it loads on any host with the NVIDIA driver.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB = HERE / "libmoe_b200.so"
SOURCES = ["api.cu", "route.cu", "repack.cu", "gemm_tc.cu", "gemm_simt.cu", "group.cu", "group_noalloc.cu", "gemm_bs.cu", "block.cu", "cache.cu",
           "ep.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def flags(debug: bool) -> list[str]:
    f = ARCH + ["-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                "--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("MOE_PTXAS_V") else "-O3"]
    f += ["-O0", "-G"] if debug else ["-O3"]
    return f


def compile_one(src: str, debug: bool) -> Path:
    out = OBJ / (Path(src).stem + ".o")
    srcp = CSRC / src
    deps = [srcp, CSRC / "common.cuh", CSRC / "kernels.h", CSRC / "engine.h", HERE.parent / "include" / "moe_b200.h"]
    if out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    cmd = [NVCC] + flags(debug) + ["-c", str(srcp), "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed on {src}")
    if os.environ.get("MOE_PTXAS_V"):
        sys.stderr.write(r.stderr)
    return out


def build(debug: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, debug), SOURCES))
    if LIB.exists() and all(LIB.stat().st_mtime >= o.stat().st_mtime for o in objs):
        return LIB
    # static CUDA runtime: the library needs only the driver at run time
    cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", str(LIB)] + [str(o) for o in objs] + ["-ldl"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(debug="--debug" in sys.argv))
