"""Build the sm_100a shared library ``liborthocache_b200.so`` in-tree.

    python -m orthocache_b200.build        # or: python orthocache_b200/build.py

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links one
shared object next to this file.  Objects go to ``_build/`` (not committed).
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(ROOT, "_build", "obj")
LIB = os.path.join(HERE, "liborthocache_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-I", os.path.join(ROOT, "include"),
]


def _compile(src):
    obj = os.path.join(OBJ, os.path.basename(src).replace(".cu", ".o"))
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs.append(os.path.join(ROOT, "include", "orthocache_b200.h"))
    # sources that include another .cu (oc_score_meta.cu) depend on it
    with open(src) as f:
        text = f.read()
    hdrs += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu") and f'#include "{f}"' in text]
    if os.path.exists(obj):
        t = os.path.getmtime(obj)
        if t >= os.path.getmtime(src) and all(t >= os.path.getmtime(h) for h in hdrs):
            return obj
    cmd = [NVCC] + FLAGS + ["-c", src, "-o", obj]
    if os.environ.get("OC_PTXAS_VERBOSE"):
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if os.environ.get("OC_PTXAS_VERBOSE"):
        sys.stderr.write(r.stderr)
    return obj


def build(verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(_compile, srcs))
    if os.path.exists(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [NVCC, "-shared", "--cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
