"""Builds the CPU oracle (test infrastructure only) into oracle/_build/.

gcc compiles gsb_oracle.c with OpenMP and without floating-point contraction so
the tile-intersection arithmetic rounds exactly like the GPU's explicitly
rounded operations (both use gsplat_b200/csrc/detmath.h).
"""

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libgsb_oracle.so")
SRC = os.path.join(HERE, "gsb_oracle.c")
DETMATH = os.path.join(ROOT, "gsplat_b200", "csrc", "detmath.h")


def build() -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    newest = max(os.path.getmtime(SRC), os.path.getmtime(DETMATH))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-I", os.path.dirname(DETMATH), SRC, "-o", LIB, "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build())
