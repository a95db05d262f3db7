"""Builds libfopt_b200.so in-tree: every .cu / .cpp under csrc/ for sm_100a, linked with the static
CUDA runtime so the library loads wherever the driver is present. NCCL is loaded at run time.

Run as `python furiosa-opt_b200/build.py` (or through `__graft_entry__.build()`).
"""
from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfopt_b200.so")
ROOT = os.path.dirname(HERE)

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
GEN = os.path.join(OBJ, "gen")
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"), "-I", GEN,
          "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


# The GEMM's fused SwiGLU epilogue computes the activation with the same device code as the
# generated elementwise kernels (NVRTC, --fmad=false), so it is compiled without contraction too.
PER_FILE = {"k_gemm.cu": ["--fmad=false"]}


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_digest():
    h = hashlib.sha256()
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".h", ".hpp", ".cuh")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(fh.read())
    return h.hexdigest()[:16]


def _compile(src: str, verbose: bool) -> str:
    base = os.path.splitext(os.path.basename(src))[0]
    obj = os.path.join(OBJ, base + ".o")
    stamp = obj + ".stamp"
    with open(src, "rb") as fh:
        key = hashlib.sha256(fh.read()).hexdigest()[:16] + _headers_digest() + str(PER_FILE.get(os.path.basename(src)))
    if os.path.exists(obj) and os.path.exists(stamp) and open(stamp).read() == key:
        return obj
    cmd = [NVCC, *ARCH, *COMMON, *PER_FILE.get(os.path.basename(src), []), "-c", src, "-o", obj]
    if src.endswith(".cpp"):  # pure host code
        cmd = [NVCC, *COMMON, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, flush=True)
    with open(stamp, "w") as fh:
        fh.write(key)
    return obj


def _generate():
    """ew_ops.cuh as a C++ raw string literal: the prelude handed to NVRTC for generated kernels."""
    os.makedirs(GEN, exist_ok=True)
    with open(os.path.join(CSRC, "ew_ops.cuh")) as fh:
        src = fh.read()
    text = 'R"FOPTSRC(' + src + ')FOPTSRC"\n'
    out = os.path.join(GEN, "ew_ops_src.inc")
    if not os.path.exists(out) or open(out).read() != text:
        with open(out, "w") as fh:
            fh.write(text)


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    _generate()
    srcs = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
