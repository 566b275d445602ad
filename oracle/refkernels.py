"""ctypes binding of _ref/libref.so: the reference's own kernels (src/engine.cu of
g023/cuda_inf, rebuilt for sm_100a by oracle/Makefile) behind the launchers of
ref_shim.cu.  TEST INFRASTRUCTURE ONLY.  Dimensions are the reference's
compile-time constants (H=2048, NH=32, NKV=8, HEAD_DIM=64, NSPLIT=16).

Functions take torch CUDA tensors and launch on the current stream.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libref.so")
ENGINE = os.path.join(HERE, "_ref", "ref_engine")
_L = None
P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float

_SIGS = {
    "ref_gemv_int4": [P, P, P, P, I, I, I, P],
    "ref_gemv_fp16": [P, P, P, I, I, I, P],
    "ref_rmsnorm": [P, P, P, I, I, F, P],
    "ref_rmsnorm_head": [P, P, P, I, F, P],
    "ref_rope": [P, P, P, I, P],
    "ref_kv_write_tail": [P, P, P, P, I, I, P],
    "ref_kv_commit_group": [P, P, P, P, P, P, I, I, P],
    "ref_attn_decode": [P, P, P, P, P, P, P, I, I, F, P, P, P, P, P],
    "ref_conv_pre": [P, P, P, I, P],
    "ref_conv_apply": [P, P, P, P, P, I, P],
    "ref_conv_update_state": [P, P, I, P],
    "ref_swiglu": [P, P, P, I, P],
    "ref_acc_scaled": [P, P, F, I, P],
    "ref_add_inplace": [P, P, I, P],
    "ref_add_f32_inplace": [P, P, I, P],
    "ref_f32_to_f16": [P, P, I, P],
    "ref_embed_gather": [P, P, P, I, P],
    "ref_argmax": [P, I, P, P],
    "ref_fp8_roundtrip": [P, P, P, I, P],
    "ref_dims": [P],
}


def available():
    return os.path.exists(LIB)


def lib():
    global _L
    if _L is None:
        L = ctypes.CDLL(LIB)
        for n, a in _SIGS.items():
            f = getattr(L, n)
            f.restype = I
            f.argtypes = a
        _L = L
    return _L


def dims():
    import numpy as np
    d = np.zeros(11, np.int32)
    lib().ref_dims(d.ctypes.data)
    keys = ["H", "NL", "HEAD_DIM", "NH", "NKV", "VOCAB", "NEXP", "TOPK", "MOE_INTER",
            "DENSE_INTER", "NSPLIT"]
    return dict(zip(keys, d.tolist()))


def _s():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def call(name, *args):
    """Launch ref_<name> with tensors/ints/floats; raises on a CUDA error."""
    conv = [(_p(a) if hasattr(a, "data_ptr") else a) for a in args]
    rc = getattr(lib(), "ref_" + name)(*conv, _s())
    if rc != 0:
        raise RuntimeError(f"reference kernel {name} failed with CUDA error {rc}")
