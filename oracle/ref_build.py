"""Build oracle/_ref/libtpref.so from the reference's own op code.

TEST INFRASTRUCTURE ONLY. The reference cannot be built as a whole (its ggml
submodule is absent), but the ops this decoder depends on are self-contained
inside patches/ggml-tp-ops.patch:

* the ggml CPU forward functions of bilinear_gather, bias_lrelu,
  subpix_lrelu(_cl), upfirdn2x, clsp_mul/lerp and flow_grid (patch:313-657);
* the CUDA kernels bilinear_gather_kernel (patch:688-718), im2col_cf_kernel
  (patch:830-861) and the tp-fused kernels (patch:920-1095).

This script reads those function bodies out of the patch where it lies (it is
never copied into the repository), appends them after oracle/ref_shim.h (which
supplies the few ggml / CUDA names they use) and before oracle/ref_wrap.cpp (C
entry points), and compiles the translation unit as host C++ into
oracle/_ref/, which git ignores. The CUDA kernels run on the host by looping
over every (block, thread) index. Their outputs pin the oracle's op
restatements and generate the golden vectors under tests/golden/.

It also builds oracle/_ref/libtpgraph.so, the graph-level pin: the
reference's own src/motion_dec.cpp, src/motion_enc.cpp and src/gguf_load.cpp,
compiled where they lie against the ggml stand-in in oracle/refgraph/, with
the patch's op constructors (src/ggml.c part of the patch) and CPU forward
functions extracted the same way.

Usage: python oracle/ref_build.py [--reference DIR]
The reference tree is DIR, else $TP_REFERENCE, else BASELINE.json's
"reference_path". Exits 0 without doing anything when it is absent.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
GRAPH_DIR = os.path.join(HERE, "refgraph")

# (file inside the patch, signature marker) for every function to extract
CPU_FUNCS = [
    "void ggml_compute_forward_bilinear_gather(",
    "void ggml_compute_forward_bias_lrelu(",
    "void ggml_compute_forward_subpix_lrelu(",
    "void ggml_compute_forward_subpix_lrelu_cl(",
    "void ggml_compute_forward_upfirdn2x(",
    "void ggml_compute_forward_clsp_mul(",
    "void ggml_compute_forward_clsp_lerp(",
    "void ggml_compute_forward_flow_grid(",
]
# the patch's op constructors (src/ggml.c), needed by the graph-level pin
GRAPH_CTORS = [
    "struct ggml_tensor * ggml_im2col_cf(",
    "struct ggml_tensor * ggml_bilinear_gather(",
    "struct ggml_tensor * ggml_flow_grid(",
    "struct ggml_tensor * ggml_bilinear_gather_planar(",
    "struct ggml_tensor * ggml_bilinear_gather_sp(",
    "struct ggml_tensor * ggml_bias_lrelu(",
    "struct ggml_tensor * ggml_subpix_lrelu(",
    "struct ggml_tensor * ggml_subpix_lrelu_cl(",
    "struct ggml_tensor * ggml_upfirdn2x(",
    "struct ggml_tensor * ggml_clsp_mul(",
    "struct ggml_tensor * ggml_clsp_lerp(",
]
# the reference's own sources compiled for the graph-level pin
GRAPH_SOURCES = ["src/motion_dec.cpp", "src/motion_enc.cpp", "src/gguf_load.cpp"]
CUDA_FUNCS = [
    ("src/ggml-cuda/bilinear-gather.cu", "template <typename T, bool SP>"),
    ("src/ggml-cuda/im2col.cu", "template <typename T, bool IC_POW2>"),
    ("src/ggml-cuda/tp-fused.cu", "static __global__ void bias_lrelu_kernel("),
    ("src/ggml-cuda/tp-fused.cu", "static __global__ void subpix_lrelu_kernel("),
    ("src/ggml-cuda/tp-fused.cu", "static __global__ void subpix_lrelu_cl_kernel("),
    ("src/ggml-cuda/tp-fused.cu", "static __global__ void upfirdn2x_kernel("),
    ("src/ggml-cuda/tp-fused.cu", "template <bool LERP>"),
    ("src/ggml-cuda/tp-fused.cu", "static __global__ void flow_grid_kernel("),
]


def added_lines_by_file(patch_text: str) -> dict[str, list[str]]:
    """Lines a unified diff adds, grouped by target file, '+' stripped."""
    files: dict[str, list[str]] = {}
    cur = None
    for line in patch_text.splitlines():
        if line.startswith("diff --git "):
            cur = line.split(" b/", 1)[1]
            files[cur] = []
        elif cur is not None and line.startswith("+") and not line.startswith("+++"):
            files[cur].append(line[1:])
    return files


def extract_function(lines: list[str], marker: str) -> str:
    """From the line starting with `marker` to the brace that closes it."""
    start = next(i for i, l in enumerate(lines) if l.startswith(marker))
    depth, opened = 0, False
    for i in range(start, len(lines)):
        depth += lines[i].count("{") - lines[i].count("}")
        opened = opened or "{" in lines[i]
        if opened and depth == 0:
            return "\n".join(lines[start:i + 1]) + "\n"
    raise ValueError(f"unterminated function at {marker!r}")


def reference_dir(arg: str | None) -> str | None:
    """--reference, else $TP_REFERENCE, else BASELINE.json's reference_path"""
    if arg:
        return arg
    if os.environ.get("TP_REFERENCE"):
        return os.environ["TP_REFERENCE"]
    bj = os.path.join(os.path.dirname(HERE), "BASELINE.json")
    if os.path.exists(bj):
        import json
        return json.load(open(bj)).get("reference_path")
    return None


def build_graph(ref: str, added: dict[str, list[str]]) -> str:
    """oracle/_ref/libtpgraph.so: the reference's decoder, encoder and loader
    over the stand-in"""
    parts = [f"// GENERATED by oracle/ref_build.py from {ref}/patches; git-ignored.\n",
             '#include "ggml.h"\n#include <cmath>\n']
    for marker in GRAPH_CTORS:
        parts.append(extract_function(added["src/ggml.c"], marker))
    for marker in CPU_FUNCS:
        parts.append(extract_function(added["src/ggml-cpu/ops.cpp"], marker))
    src = os.path.join(OUT_DIR, "patch_graph_ops.cpp")
    with open(src, "w") as f:
        f.write("\n".join(parts))
    so = os.path.join(OUT_DIR, "libtpgraph.so")
    srcs = [os.path.join(GRAPH_DIR, "graph.cpp"), os.path.join(GRAPH_DIR, "wrap.cpp"), src] + \
        [os.path.join(ref, s) for s in GRAPH_SOURCES]
    deps = srcs + [os.path.join(GRAPH_DIR, h) for h in os.listdir(GRAPH_DIR) if h.endswith(".h")]
    if os.path.exists(so) and os.path.getmtime(so) >= max(os.path.getmtime(d) for d in deps):
        return so
    cmd = ["g++", "-O2", "-march=x86-64-v3", "-std=gnu++17", "-fPIC", "-shared", "-fopenmp",
           "-I", GRAPH_DIR, "-I", os.path.join(ref, "src"), "-o", so] + srcs
    subprocess.run(cmd, check=True)
    return so


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    args = ap.parse_args()
    ref = reference_dir(args.reference)
    if not ref:
        print("ref_build: no reference tree named; using any prebuilt oracle/_ref")
        return 0
    args.reference = ref
    patch = os.path.join(args.reference, "patches", "ggml-tp-ops.patch")
    if not os.path.exists(patch):
        print(f"ref_build: {patch} absent; using any prebuilt oracle/_ref")
        return 0
    added = added_lines_by_file(open(patch).read())
    parts = [f"// GENERATED by oracle/ref_build.py from {patch}; git-ignored.\n",
             '#include "../ref_shim.h"\n']
    for marker in CPU_FUNCS:
        parts.append(extract_function(added["src/ggml-cpu/ops.cpp"], marker))
    for fname, marker in CUDA_FUNCS:
        parts.append(extract_function(added[fname], marker))
    parts.append('#include "../ref_wrap.cpp"\n')
    os.makedirs(OUT_DIR, exist_ok=True)
    src = os.path.join(OUT_DIR, "ref_ops.cpp")
    with open(src, "w") as f:
        f.write("\n".join(parts))
    so = os.path.join(OUT_DIR, "libtpref.so")
    # gnu++17 keeps GCC's default floating-point contraction, as a CMake
    # build of ggml (C++ extensions on) would
    cmd = ["g++", "-O2", "-march=x86-64-v3", "-std=gnu++17", "-fPIC", "-shared",
           "-o", so, src]
    subprocess.run(cmd, check=True)
    print(f"ref_build: built {so}")
    print(f"ref_build: built {build_graph(args.reference, added)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
