"""Builds the CUDA C-ABI library `comp_b200/libcompb200.so` for sm_100a with nvcc (no GPU needed).

Each `csrc/*.cu` file compiles to an object under `comp_b200/_build/` (in parallel, skipped when up to date), then
all objects link into one shared library next to this file, where `comp_b200._lib` loads it.

    python -m comp_b200.build            # build (incremental)
    python -m comp_b200.build --force    # rebuild everything
    python -m comp_b200.build --ptxas    # also print ptxas register / spill / shared-memory lines
"""

import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcompb200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# IEEE division and square root, no flush-to-zero: the quantizers must reproduce the reference's bytes exactly
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-prec-div=true", "-prec-sqrt=true",
              "-ftz=false", "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    return "nvcc"


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force, ptxas):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not force and not ptxas and not _stale(obj, [src, *headers(), __file__]):
        return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force=False, ptxas=False, jobs=None, log=print):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with concurrent.futures.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, force, ptxas), srcs))
    objs = [o for o, _ in results]
    if ptxas:
        for _, err in results:
            if err.strip():
                log(err.strip())
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
        log(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, ptxas="--ptxas" in sys.argv)
