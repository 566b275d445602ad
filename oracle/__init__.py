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
REF_TREE = os.environ.get("CUINF_REFERENCE", "/root/reference")


def build(with_ref=None):
    """Build liboracle.so, and _ref/ when the reference tree is present."""
    subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True, capture_output=True)
    if with_ref is None:
        with_ref = os.path.isdir(os.path.join(REF_TREE, "src"))
    if with_ref:
        subprocess.run(["make", "-C", HERE, "ref", f"REF={REF_TREE}"], check=True,
                       capture_output=True)
