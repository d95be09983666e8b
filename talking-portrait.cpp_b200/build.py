"""Build libtpmd.so (the decoder's C ABI + sm_100a kernels) in place.

nvcc -gencode arch=compute_100a,code=sm_100a for every .cu, the host .cpp
with nvcc too (it includes CUDA headers), static cudart so the library does
not depend on which CUDA runtime the host process (e.g. torch) loaded.
Objects go to _build/ (git-ignored); the .so lands next to this file.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
SO = os.path.join(HERE, "libtpmd.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _compile(src: str) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    deps = [src] + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(HERE, "..", "include", "*.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC] + FLAGS + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC] + FLAGS + ["-x", "cu", "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(_compile, srcs))
    if not os.path.exists(SO) or os.path.getmtime(SO) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", SO] + objs + \
              ["-lpthread", "-ldl", "-Xlinker", "-rpath=/usr/local/cuda/lib64"]
        subprocess.run(cmd, check=True)
    if verbose:
        print(f"built {SO}")
    return SO


if __name__ == "__main__":
    build(verbose=True)
