"""Per-CTA timeline of the fused decode layer (developer diagnostic).

    python -m orthocache_b200.diag_timeline [evict]      # from the repository root, on a GPU

Builds a second copy of the library with -DOC_TIMING (into _build/timing/,
not the shipped .so), runs the bench workload (configuration 1) as a CUDA
graph of four consecutive layers, and prints, for the last layer, the
distribution over CTAs of the %globaltimer stamps the kernel records: start,
the end of the programmatic-dependent wait, first slab, end of scoring, the
attention's first data and last unit, and the group merges — the breakdown
quoted in the design notes (pipeline fill, streaming, tail).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(ROOT, "_build", "timing")
NSTAMP = 20  # g_sstamp[cta][20] in oc_score.cu

STAMPS = [(0, "start"), (1, "setup done"), (2, "first slab"), (3, "scoring end"), (4, "epilogues end"),
          (15, "first claim"), (11, "attention start"), (12, "attention data"), (13, "attention end"),
          (14, "merged")]


def build_timing_library():
    from . import build
    os.makedirs(OUT, exist_ok=True)
    srcs = sorted(os.path.join(build.CSRC, f) for f in os.listdir(build.CSRC) if f.endswith(".cu"))

    def one(src):
        obj = os.path.join(OUT, os.path.basename(src).replace(".cu", ".o"))
        subprocess.run([build.NVCC] + build.FLAGS + ["-DOC_TIMING", "-c", src, "-o", obj], check=True,
                       capture_output=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(one, srcs))
    lib = os.path.join(OUT, "liborthocache_b200_timing.so")
    subprocess.run([build.NVCC, "-shared", "--cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-o", lib] + objs, check=True, capture_output=True)
    return lib


def main(evict=0.75):
    lib_path = build_timing_library()
    from . import _lib
    _lib.LIB_PATH = lib_path
    sys.path.insert(0, ROOT)
    import torch
    import bench
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    layers = bench.make_layers(0, evict, dev)
    eng = bench.Engine(layers, dev, 1)
    lib = _lib.load()
    for i in range(40):
        eng.step(layers[i % bench.LAYERS])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for L in layers:
            eng.step(L)
    for _ in range(4):
        g.replay()
    torch.cuda.synchronize()
    n = torch.cuda.get_device_properties(dev).multi_processor_count
    buf = (C.c_ulonglong * (n * NSTAMP))()
    lib.oc_probe_read_score_stamps(buf, n)
    s = [[buf[b * NSTAMP + i] for i in range(NSTAMP)] for b in range(n)]
    t0 = min(r[0] for r in s)
    print(f"fused decode layer, configuration 1, eviction {evict}: µs after the first CTA started")
    for i, name in STAMPS:
        v = sorted((r[i] - t0) / 1e3 for r in s)
        print(f"  {name:16s} min {v[0]:7.2f}  median {v[len(v) // 2]:7.2f}  max {v[-1]:7.2f}")


if __name__ == "__main__":
    main(float(sys.argv[1]) if len(sys.argv) > 1 else 0.75)
