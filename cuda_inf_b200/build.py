"""Build libcuinf.so in-tree for sm_100a (nvcc; no GPU needed to compile).

    python -m cuda_inf_b200.build [--force] [-j N] [--trace]

Objects go to cuda_inf_b200/_build/, the library to cuda_inf_b200/libcuinf.so.
--trace builds the diagnostic variant with the decode kernels' phase
timestamps (-DCUINF_PHASE_TRACE) into _build_trace/ and libcuinf_trace.so;
`python bench.py --phase-trace` loads it.  The product never loads it.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libcuinf.so")
BUILD_TRACE = os.path.join(PKG, "_build_trace")
LIB_TRACE = os.path.join(PKG, "libcuinf_trace.so")
SOURCES = ["ops.cu", "engine.cu", "batch.cu", "tokenizer.cpp"]
HEADERS = sorted(f for f in os.listdir(CSRC) if f.endswith((".cuh", ".h")))

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, extra, build_dir=BUILD):
    obj = os.path.join(build_dir, os.path.splitext(src)[0] + ".o")
    deps = [os.path.join(CSRC, src)] + [os.path.join(CSRC, h) for h in HEADERS] + \
        [os.path.join(ROOT, "include", "cuinf.h")]
    if not _newer(obj, deps):
        return obj, None
    cmd = [NVCC] + ARCH + FLAGS + extra + ["-c", os.path.join(CSRC, src), "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, r.stderr + r.stdout
    return obj, None


def build(force=False, jobs=4, extra=(), trace=False):
    build_dir, lib = (BUILD_TRACE, LIB_TRACE) if trace else (BUILD, LIB)
    if trace:
        extra = list(extra) + ["-DCUINF_PHASE_TRACE"]
    os.makedirs(build_dir, exist_ok=True)
    if force:
        for f in os.listdir(build_dir):
            os.remove(os.path.join(build_dir, f))
    with cf.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, list(extra), build_dir), SOURCES))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if force or _newer(lib, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", lib] + objs + ["-lcudart_static", "-lnccl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr + r.stdout)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=4)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    ap.add_argument("--trace", action="store_true", help="diagnostic build with phase timestamps")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    if a.ptxas_v:
        for s in SOURCES:
            cmd = [NVCC] + ARCH + FLAGS + extra + ["-c", os.path.join(CSRC, s), "-o", os.devnull]
            r = subprocess.run(cmd, capture_output=True, text=True)
            sys.stdout.write(r.stderr)
    print(build(a.force, a.j, trace=a.trace))
