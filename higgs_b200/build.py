"""Build libhiggs_cuda.so in-tree for sm_100a (nvcc, no JIT cache).

Usage: python -m higgs_b200.build   (or higgs_b200.build.build())
       python -m higgs_b200.build --timeline   (libhiggs_cuda_timeline.so: the same library
       with per-CTA timestamps in the decode-step kernels, read by higgs_b200.timeline)
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libhiggs_cuda.so")
OBJ_TL = os.path.join(HERE, "_build_timeline")
LIB_TL = os.path.join(HERE, "libhiggs_cuda_timeline.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills", "-DNDEBUG"]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _stale(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(HERE, "..", "include", "higgs_cuda.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src: str, obj_dir: str = OBJ, extra: tuple = ()) -> str:
    obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
    if _stale(src, obj):
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, timeline: bool = False) -> str:
    obj_dir, lib = (OBJ_TL, LIB_TL) if timeline else (OBJ, LIB)
    extra = ("-DHIGGS_TIMELINE",) if timeline else ()
    os.makedirs(obj_dir, exist_ok=True)
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, obj_dir, extra), sources()))
    if not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", *objs, "-o", lib, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(lib)
    return lib


if __name__ == "__main__":
    build(verbose=True, timeline="--timeline" in sys.argv[1:])
