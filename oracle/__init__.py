"""CPU oracle and reference-kernel launchers: TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its
reference arm) may import this package.  The product (cuda_inf_b200) never
imports it.

  pyoracle    ctypes binding of liboracle.so (oracle.c: scalar C restatement
              of src/engine.cu + tools/export_weights.py of g023/cuda_inf)
  refkernels  ctypes binding of _ref/libref.so (the reference's own kernels
              rebuilt for sm_100a, see ref_shim.cu and Makefile)
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_tree():
    """The g023/cuda_inf source tree: $CUINF_REFERENCE, else a checkout named
    `reference` beside this repository; None when neither exists."""
    cand = os.environ.get("CUINF_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(os.path.join(cand, "src")) else None


def build(with_ref=None):
    """Build liboracle.so and libcpubase.so, and _ref/ when the reference
    tree is found (reference_tree())."""
    subprocess.run(["make", "-C", HERE, "liboracle.so", "libcpubase.so"], check=True, capture_output=True)
    ref = reference_tree()
    if with_ref is None:
        with_ref = ref is not None
    if with_ref:
        if ref is None:
            raise RuntimeError("reference tree not found: set CUINF_REFERENCE")
        subprocess.run(["make", "-C", HERE, "ref", f"REF={ref}"], check=True, capture_output=True)


def baseline_library():
    """Path of the timed CPU baseline (oracle.c built with -DORC_BASELINE):
    built for this host's own ISA (-march=native) when gcc is at hand, else
    the prebuilt portable x86-64-v3 library."""
    native = os.path.join(HERE, "_native", "libcpubase.so")
    r = subprocess.run(["make", "-B", "-C", HERE, "native"], capture_output=True)
    if r.returncode == 0 and os.path.exists(native):
        return native
    return os.path.join(HERE, "libcpubase.so")
