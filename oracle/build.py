"""TEST INFRASTRUCTURE ONLY: builds oracle/c/oracle.c into oracle/_build/liboracle.so with gcc + OpenMP.

    python -m oracle.build
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "c", "oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")
# correctly rounded IEEE float operations only: no fast-math, no FMA contraction
CFLAGS = ["-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-std=c11"]


def build(force=False, log=print):
    os.makedirs(OUT_DIR, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    tmp = LIB + ".tmp"
    r = subprocess.run(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"gcc failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    log(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
