"""ctypes binding of libcuinf.so (include/cuinf.h).

The library is loaded from this package directory only.  There is no
fallback: if the shared library is missing or fails to load, importing the
ops raises.
"""
import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libcuinf.so")

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t
c_int64 = ctypes.c_int64


class CuinfConfig(ctypes.Structure):
    """Mirror of cuinf_config (include/cuinf.h)."""
    _fields_ = [
        ("hidden", ctypes.c_int32), ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("vocab", ctypes.c_int32),
        ("n_dense", ctypes.c_int32), ("n_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("moe_inter", ctypes.c_int32), ("dense_inter", ctypes.c_int32), ("conv_k", ctypes.c_int32),
        ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float),
        ("attn_layer", ctypes.c_uint8 * 64),
    ]


# name -> (restype, argtypes)
_SIGS = {
    "cuinf_last_error": (ctypes.c_char_p, []),
    "cuinf_version": (ctypes.c_char_p, []),
    "cuinf_gemv_int4": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "cuinf_gemm_int4_tc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "cuinf_gemm_fp16_tc": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "cuinf_argmax_key_index": (c_int, [ctypes.c_ulonglong]),
    "cuinf_gemv_fp16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "cuinf_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "cuinf_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_void_p]),
    "cuinf_kv_write_tail": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                    c_void_p]),
    "cuinf_kv_commit_group": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int, c_int, c_int, c_void_p]),
    "cuinf_attn_decode_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "cuinf_attn_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_int, c_int, c_float, c_void_p, c_int, c_int, c_void_p,
                                  c_size_t, c_void_p]),
    "cuinf_attn_decode_static_scratch_bytes": (c_size_t, []),
    "cuinf_attn_decode_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_int, c_int, c_float, c_void_p,
                                          c_int, c_int, c_void_p]),
    "cuinf_conv_pre": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "cuinf_conv_apply": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                 c_void_p]),
    "cuinf_conv_update_state": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "cuinf_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "cuinf_acc_scaled": (c_int, [c_void_p, c_void_p, c_float, c_int, c_void_p]),
    "cuinf_add_inplace": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "cuinf_add_f32_inplace": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "cuinf_f32_to_f16": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "cuinf_embed_gather": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "cuinf_argmax": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "cuinf_moe_route": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
                                c_void_p]),
    "cuinf_moe_ffn_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "cuinf_moe_ffn": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                              c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "cuinf_quantize_int4": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "cuinf_quantize_int4_host": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "cuinf_default_config": (None, [ctypes.POINTER(CuinfConfig)]),
    "cuinf_model_load": (c_int, [ctypes.c_char_p, ctypes.POINTER(CuinfConfig),
                                 ctypes.POINTER(c_void_p)]),
    "cuinf_model_from_device_blob": (c_int, [ctypes.POINTER(CuinfConfig), c_void_p, c_size_t,
                                             c_void_p, c_size_t, ctypes.POINTER(c_void_p)]),
    "cuinf_model_free": (c_int, [c_void_p]),
    "cuinf_session_create": (c_int, [c_void_p, c_int, c_void_p, ctypes.POINTER(c_void_p)]),
    "cuinf_session_free": (c_int, [c_void_p]),
    "cuinf_session_reset": (c_int, [c_void_p]),
    "cuinf_session_pos": (c_int, [c_void_p]),
    "cuinf_session_state_bytes": (c_size_t, [c_void_p]),
    "cuinf_session_save_state": (c_int, [c_void_p, c_void_p, c_size_t]),
    "cuinf_session_load_state": (c_int, [c_void_p, c_void_p, c_size_t]),
    "cuinf_decode_step": (c_int, [c_void_p, c_int, ctypes.POINTER(c_int)]),
    "cuinf_generate": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                               ctypes.POINTER(c_int)]),
    "cuinf_session_keep_logits": (c_int, [c_void_p, c_int]),
    "cuinf_session_set_option": (c_int, [c_void_p, c_int, c_int]),
    "cuinf_session_attn_cluster": (c_int, [c_void_p]),
    "cuinf_prefill": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "cuinf_tokenizer_load": (c_int, [ctypes.c_char_p, c_void_p]),
    "cuinf_tokenizer_free": (c_int, [c_void_p]),
    "cuinf_tokenizer_vocab_size": (c_int, [c_void_p]),
    "cuinf_tokenizer_encode": (c_int, [c_void_p, ctypes.c_char_p, c_size_t, c_void_p, c_int, c_void_p]),
    "cuinf_tokenizer_decode": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "cuinf_chat_prompt": (c_int, [ctypes.c_char_p, c_void_p, c_size_t, c_void_p]),
    "cuinf_session_set_kv_budget": (c_int, [c_void_p, c_int, c_int]),
    "cuinf_session_h2o_state": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "cuinf_batch_create": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "cuinf_batch_free": (c_int, [c_void_p]),
    "cuinf_batch_reset": (c_int, [c_void_p]),
    "cuinf_batch_step": (c_int, [c_void_p, c_void_p, c_void_p]),
    "cuinf_batch_keep_logits": (c_int, [c_void_p, c_int]),
    "cuinf_batch_logits": (c_void_p, [c_void_p]),
    "cuinf_batch_routes": (c_int, [c_void_p, c_void_p]),
    "cuinf_batch_kernels_per_step": (c_int, [c_void_p]),
    "cuinf_batch_fill_synthetic": (c_int, [c_void_p, c_int, ctypes.c_ulonglong]),
    "cuinf_batch_seq_state_bytes": (c_size_t, [c_void_p, c_int]),
    "cuinf_batch_save_seq": (c_int, [c_void_p, c_int, c_void_p, c_size_t]),
    "cuinf_batch_load_seq": (c_int, [c_void_p, c_int, c_void_p, c_size_t]),
    "cuinf_batch_error": (c_int, [c_void_p]),
    "cuinf_batch_profile_step": (c_int, [c_void_p, c_int, c_void_p, ctypes.c_char_p, c_int, c_void_p]),
    "cuinf_batch_create_ep": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "cuinf_ep_unique_id": (c_int, [c_void_p, c_int]),
    "cuinf_ep_unique_id_bytes": (c_int, []),
    "cuinf_batch_sync": (c_int, [c_void_p]),
    "cuinf_ep_plan_host": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "cuinf_batch_abort": (c_int, [c_void_p]),
    "cuinf_batch_set_timeout": (c_int, [c_void_p, c_int]),
    "cuinf_batch_failed": (c_int, [c_void_p]),
    "cuinf_batch_ep_exchange": (c_int, [c_void_p]),
    "cuinf_batch_set_ep_exchange": (c_int, [c_void_p, c_int]),
    "cuinf_device_error": (c_int, [ctypes.POINTER(ctypes.c_uint)]),
    "cuinf_selftest_wait_timeout": (c_int, [ctypes.c_uint, ctypes.POINTER(ctypes.c_uint),
                                            ctypes.POINTER(ctypes.c_ulonglong)]),
    "cuinf_session_uses_megakernel": (c_int, [c_void_p]),
    "cuinf_session_trace": (c_int, [c_void_p, c_void_p, c_int, c_void_p, ctypes.POINTER(c_int),
                                    ctypes.POINTER(c_int)]),
    "cuinf_session_error": (c_int, [c_void_p, c_void_p]),
    "cuinf_session_logits": (c_void_p, [c_void_p]),
    "cuinf_session_hidden": (c_void_p, [c_void_p]),
    "cuinf_session_routes": (c_int, [c_void_p, c_void_p, c_void_p]),
    "cuinf_session_kernels_per_step": (c_int, [c_void_p]),
    "cuinf_session_profile_step": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                           c_int, ctypes.POINTER(c_int)]),
}

EXPORTS = tuple(_SIGS)
_lib = None


def lib():
    """Load libcuinf.so (once).  Raises if it is absent: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m cuda_inf_b200.build` "
                "(there is no CPU fallback)")
        # torch first: its NCCL (libnccl.so.2) is then the one the library's
        # NCCL dependency resolves to, so both share one NCCL in the process
        import torch  # noqa: F401
        import torch.distributed  # noqa: F401
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class CuinfError(RuntimeError):
    pass


def check(rc):
    if rc != 0:
        msg = lib().cuinf_last_error().decode(errors="replace")
        raise CuinfError(f"cuinf error {rc}: {msg}")
    return rc
