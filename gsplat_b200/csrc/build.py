"""Builds libgsplat_b200.so: every kernel of the package for sm_100a.

Each .cu file is compiled to an object with nvcc (in parallel) and the objects
are linked into one shared library next to the package's __init__.py. The
library exports only the C ABI declared in include/gsplat_b200.h.

Usage: python -m gsplat_b200.csrc.build  (or gsplat_b200.csrc.build.build()).
"""

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
INCLUDE = os.path.join(ROOT, "include")
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(PKG, "libgsplat_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda_home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def sources():
    return sorted(f for f in os.listdir(HERE) if f.endswith(".cu"))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
    src_path = os.path.join(HERE, src)
    deps = [src_path] + [
        os.path.join(HERE, h) for h in os.listdir(HERE) if h.endswith((".h", ".cuh"))
    ] + [os.path.join(INCLUDE, "gsplat_b200.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", HERE, "-c", src_path, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < newest:
        cmd = [_nvcc(), *ARCH, "-shared", "-o", LIB_PATH, *objs, "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
