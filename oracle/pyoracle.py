"""ctypes binding of liboracle.so (oracle.c).  TEST INFRASTRUCTURE ONLY.

numpy in / numpy out.  fp16 arrays are np.float16 (bit patterns passed
through as uint16); FP8 arrays are np.uint8.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_L = None

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
I64 = ctypes.c_int64


class OrcConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32), ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("vocab", ctypes.c_int32),
        ("n_dense", ctypes.c_int32), ("n_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("moe_inter", ctypes.c_int32), ("dense_inter", ctypes.c_int32), ("conv_k", ctypes.c_int32),
        ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float),
        ("attn_layer", ctypes.c_uint8 * 64),
    ]


_SIGS = {
    "orc_h2f": (F, [ctypes.c_uint16]),
    "orc_f2h": (ctypes.c_uint16, [F]),
    "orc_e4m3_to_f32": (F, [ctypes.c_uint8]),
    "orc_f32_to_e4m3_sat": (ctypes.c_uint8, [F]),
    "orc_quant_int4_group": (None, [P, I64, I64, P, P]),
    "orc_dequant_int4": (None, [P, P, I64, I64, P]),
    "orc_gemv_int4": (None, [P, P, P, P, I, I, I]),
    "orc_gemv_fp16": (None, [P, P, P, I, I, I]),
    "orc_rmsnorm": (None, [P, P, P, I, I, F]),
    "orc_rope": (None, [P, P, P, I, I, I, I, F]),
    "orc_kv_write_tail": (None, [P, P, P, P, I, I, I, I]),
    "orc_kv_commit_group": (None, [P, P, P, P, P, P, I, I, I, I]),
    "orc_attn_decode": (None, [P, P, P, P, P, P, P, I, I, F, P, I, I, I]),
    "orc_conv_pre": (None, [P, P, P, I, I]),
    "orc_conv_apply": (None, [P, P, P, P, P, I, I]),
    "orc_conv_update_state": (None, [P, P, I, I]),
    "orc_swiglu": (None, [P, P, P, I]),
    "orc_acc_scaled": (None, [P, P, F, I]),
    "orc_add_inplace": (None, [P, P, I]),
    "orc_add_f32_inplace": (None, [P, P, I]),
    "orc_f32_to_f16": (None, [P, P, I]),
    "orc_moe_select": (None, [P, P, I, I, P, P]),
    "orc_argmax": (I, [P, I]),
    "orc_model_new": (P, [ctypes.POINTER(OrcConfig), P, ctypes.c_size_t, P, ctypes.c_size_t]),
    "orc_model_free": (None, [P]),
    "orc_state_new": (P, [P, I]),
    "orc_state_free": (None, [P]),
    "orc_state_pos": (I, [P]),
    "orc_state_load": (I, [P, P, P, ctypes.c_size_t]),
    "orc_forward_token": (I, [P, P, I, P, P]),
    "orc_forward_token_ex": (I, [P, P, I, P, P, P, P]),
    "orc_prefill": (I, [P, P, P, I, P]),
    "orc_prefill_ex": (I, [P, P, P, I, P, P, P]),
    "orc_state_route_idx": (P, [P]),
    "orc_state_set_h2o": (I, [P, P, I, I]),
    "orc_state_h2o_own_slots": (P, [P]),
    "orc_state_h2o_used_slots": (P, [P]),
    "orc_state_h2o_attn_sum": (P, [P, I]),
    "orc_state_h2o_slot_pos": (P, [P, I]),
    "orc_state_h2o_n_live": (I, [P, I]),
    "orc_state_force_h2o_slots": (None, [P, P]),
    "orc_state_route_w": (P, [P]),
    "orc_set_threads": (None, [I]),
    "orc_get_threads": (I, []),
}


_PATH = os.path.join(HERE, "liboracle.so")


def use_library(path):
    """Bind this module to another build of oracle.c (the timed CPU baseline,
    libcpubase.so) instead of the checker; only before the first call."""
    global _PATH
    if _L is not None and path != _PATH:
        raise RuntimeError("pyoracle already bound to " + _PATH)
    _PATH = path


def lib():
    global _L
    if _L is None:
        path = _PATH
        if not os.path.exists(path):
            from . import build
            build(with_ref=False)
        L = ctypes.CDLL(path)
        for n, (r, a) in _SIGS.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        _L = L
    return _L


def _ptr(a):
    return None if a is None else a.ctypes.data


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def quant_int4_group(w):
    w = _c(w, np.float32)
    N, K = w.shape
    p = np.empty((N, K // 2), np.uint8)
    s = np.empty((N, K // 128), np.uint16)
    lib().orc_quant_int4_group(_ptr(w), N, K, _ptr(p), _ptr(s))
    return p, s.view(np.float16)


def dequant_int4(packed, scales):
    N = packed.shape[0]
    K = packed.shape[1] * 2
    w = np.empty((N, K), np.float32)
    lib().orc_dequant_int4(_ptr(_c(packed, np.uint8)), _ptr(_c(scales, np.float16)), N, K, _ptr(w))
    return w


def gemv_int4(x, packed, scales):
    x = _c(x, np.float16)
    N, K = packed.shape[0], packed.shape[1] * 2
    M = x.size // K
    y = np.empty((M, N), np.float32)
    lib().orc_gemv_int4(_ptr(x), _ptr(_c(packed, np.uint8)), _ptr(_c(scales, np.float16)), _ptr(y), M, N, K)
    return y.reshape((M, N) if x.ndim > 1 else (N,))


def gemv_fp16(x, W):
    x = _c(x, np.float16)
    N, K = W.shape
    M = x.size // K
    y = np.empty((M, N), np.float32)
    lib().orc_gemv_fp16(_ptr(x), _ptr(_c(W, np.float16)), _ptr(y), M, N, K)
    return y.reshape((M, N) if x.ndim > 1 else (N,))


def rmsnorm(x, w, eps=1e-5):
    x = _c(x, np.float16)
    D = w.size
    out = np.empty_like(x)
    lib().orc_rmsnorm(_ptr(x), _ptr(_c(w, np.float16)), _ptr(out), x.size // D, D, eps)
    return out


def rope(q, k, pos, theta=5e6, head_dim=64):
    q = _c(q, np.float16).copy()
    k = _c(k, np.float16).copy()
    pos = _c(pos, np.int32)
    S = pos.size
    lib().orc_rope(_ptr(q), _ptr(k), _ptr(pos), S, q.size // (S * head_dim), k.size // (S * head_dim),
                   head_dim, theta)
    return q, k


def kv_commit_group(ktail, vtail, kc8, vc8, ksc, vsc, dst_tok_base, grp):
    nkv, hd = ktail.shape[1], ktail.shape[2]
    lib().orc_kv_commit_group(_ptr(_c(ktail, np.float16)), _ptr(_c(vtail, np.float16)), _ptr(kc8),
                              _ptr(vc8), _ptr(ksc), _ptr(vsc), dst_tok_base, grp, nkv, hd)


def attn_decode(q, kc8, vc8, ksc, vsc, ktail, vtail, committed, qpos, scale=0.125):
    q = _c(q, np.float16)
    nkv, hd = ktail.shape[1], ktail.shape[2]
    nh = q.size // hd
    out = np.empty((nh, hd), np.float16)
    lib().orc_attn_decode(_ptr(q), _ptr(_c(kc8, np.uint8)), _ptr(_c(vc8, np.uint8)),
                          _ptr(_c(ksc, np.float16)), _ptr(_c(vsc, np.float16)),
                          _ptr(_c(ktail, np.float16)), _ptr(_c(vtail, np.float16)), committed, qpos,
                          scale, _ptr(out), nh, nkv, hd)
    return out


def conv_pre(inproj, S, H):
    inproj = _c(inproj, np.float32)
    C = np.empty((S, H), np.float16)
    Bx = np.empty((S, H), np.float16)
    lib().orc_conv_pre(_ptr(inproj), _ptr(C), _ptr(Bx), S, H)
    return C, Bx


def conv_apply(Bx, C, w, state, S, H):
    y = np.empty((S, H), np.float16)
    lib().orc_conv_apply(_ptr(_c(Bx, np.float16)), _ptr(_c(C, np.float16)), _ptr(_c(w, np.float16)),
                         _ptr(_c(state, np.float16)), _ptr(y), S, H)
    return y


def conv_update_state(Bx, state, S, H):
    st = _c(state, np.float16).copy()
    lib().orc_conv_update_state(_ptr(_c(Bx, np.float16)), _ptr(st), S, H)
    return st


def swiglu(g, u):
    out = np.empty(g.size, np.float16)
    lib().orc_swiglu(_ptr(_c(g, np.float32)), _ptr(_c(u, np.float32)), _ptr(out), g.size)
    return out


def acc_scaled(dst, src, w):
    d = _c(dst, np.float16).copy()
    lib().orc_acc_scaled(_ptr(d), _ptr(_c(src, np.float32)), w, d.size)
    return d


def add_inplace(a, b):
    d = _c(a, np.float16).copy()
    lib().orc_add_inplace(_ptr(d), _ptr(_c(b, np.float16)), d.size)
    return d


def add_f32_inplace(a, b):
    d = _c(a, np.float16).copy()
    lib().orc_add_f32_inplace(_ptr(d), _ptr(_c(b, np.float32)), d.size)
    return d


def moe_select(logits, bias, topk):
    logits = _c(logits, np.float32)
    bias = _c(bias, np.float32)
    idx = np.empty(topk, np.int32)
    w = np.empty(topk, np.float32)
    lib().orc_moe_select(_ptr(logits), _ptr(bias), logits.size, topk, _ptr(idx), _ptr(w))
    return idx, w


def argmax(logits):
    logits = _c(logits, np.float32)
    return lib().orc_argmax(_ptr(logits), logits.size)


def e4m3_encode(x):
    x = _c(x, np.float32).ravel()
    return np.array([lib().orc_f32_to_e4m3_sat(float(v)) for v in x], np.uint8)


def e4m3_decode(b):
    return np.array([lib().orc_e4m3_to_f32(int(v)) for v in np.asarray(b).ravel()], np.float32)


def set_threads(n):
    lib().orc_set_threads(int(n))


def get_threads():
    return lib().orc_get_threads()


class Model:
    """Whole-model oracle over weights.bin bytes + index.bin bytes."""

    def __init__(self, cfg_dict, blob, index):
        c = OrcConfig()
        for k, v in cfg_dict.items():
            if k == "attn_layer":
                for i, x in enumerate(v):
                    c.attn_layer[i] = int(x)
            elif hasattr(c, k):
                setattr(c, k, v)
        self.cfg = c
        self._blob = np.ascontiguousarray(np.frombuffer(blob, np.uint8)) if not isinstance(blob, np.ndarray) else blob
        self._index = np.frombuffer(bytes(index), np.uint8).copy()
        self._h = lib().orc_model_new(ctypes.byref(c), self._blob.ctypes.data, self._blob.size,
                                      self._index.ctypes.data, self._index.size)
        if not self._h:
            raise RuntimeError("oracle: model tensors missing or out of range")

    def state(self, max_ctx):
        return State(self, max_ctx)

    def __del__(self):
        # at interpreter exit the module globals may already be gone
        if getattr(self, "_h", None) and callable(lib):
            lib().orc_model_free(self._h)
            self._h = None


class State:
    def __init__(self, model, max_ctx):
        self.model = model
        self._h = lib().orc_state_new(model._h, max_ctx)

    def forward(self, token, want_logits=True, want_hidden=False):
        c = self.model.cfg
        lg = np.empty(c.vocab, np.float32) if want_logits else None
        hid = np.empty(c.hidden, np.float16) if want_hidden else None
        nxt = lib().orc_forward_token(self.model._h, self._h, int(token), _ptr(lg), _ptr(hid))
        return nxt, lg, hid

    def prefill(self, tokens, forced_idx=None):
        """Batched prefill of `tokens` (the reference's layer_forward(S));
        returns (argmax, logits of the last row, scores [S, n_moe, E])."""
        c = self.model.cfg
        ids = np.ascontiguousarray(tokens, np.int32)
        n_moe = max(1, c.n_layers - c.n_dense)
        lg = np.empty(c.vocab, np.float32)
        sc = np.empty((ids.size, n_moe, max(1, c.n_experts)), np.float32)
        fi = None if forced_idx is None else np.ascontiguousarray(forced_idx, np.int32)
        nxt = lib().orc_prefill_ex(self.model._h, self._h, ids.ctypes.data, int(ids.size), _ptr(fi),
                                   _ptr(sc), _ptr(lg))
        return nxt, lg, sc

    def forward_ex(self, token, forced_idx=None):
        """Forward with optional forced experts [n_moe*top_k]; returns
        (argmax, logits, hidden, scores [n_moe, E])."""
        c = self.model.cfg
        n_moe = c.n_layers - c.n_dense
        lg = np.empty(c.vocab, np.float32)
        hid = np.empty(c.hidden, np.float16)
        sc = np.empty((max(1, n_moe), max(1, c.n_experts)), np.float32)
        fi = None if forced_idx is None else np.ascontiguousarray(forced_idx, np.int32)
        nxt = lib().orc_forward_token_ex(self.model._h, self._h, int(token), _ptr(fi), _ptr(sc),
                                         _ptr(lg), _ptr(hid))
        return nxt, lg, hid, sc

    def set_h2o(self, budget, window):
        """H2O eviction mode: `budget` per-token FP8 slots per attention layer,
        local window `window` (engine.cu:310-384, 803-828)."""
        if lib().orc_state_set_h2o(self.model._h, self._h, int(budget), int(window)) != 0:
            raise ValueError("bad H2O budget/window (or the state already advanced)")
        self._h2o_budget = int(budget)

    def h2o_slots(self):
        """(own, used): per layer, the slot chosen by this oracle and the slot
        used (forced or own) in the last step; -1 for non-attention layers."""
        nl = self.model.cfg.n_layers
        own = np.ctypeslib.as_array(ctypes.cast(lib().orc_state_h2o_own_slots(self._h),
                                                ctypes.POINTER(ctypes.c_int)), (nl,)).copy()
        used = np.ctypeslib.as_array(ctypes.cast(lib().orc_state_h2o_used_slots(self._h),
                                                 ctypes.POINTER(ctypes.c_int)), (nl,)).copy()
        return own, used

    def h2o_layer(self, layer):
        """(attn_sum float32 [budget], slot_pos int32 [budget], n_live) of layer."""
        b = self._h2o_budget
        a = np.ctypeslib.as_array(ctypes.cast(lib().orc_state_h2o_attn_sum(self._h, layer),
                                              ctypes.POINTER(ctypes.c_float)), (b,)).copy()
        sp = np.ctypeslib.as_array(ctypes.cast(lib().orc_state_h2o_slot_pos(self._h, layer),
                                               ctypes.POINTER(ctypes.c_int)), (b,)).copy()
        return a, sp, lib().orc_state_h2o_n_live(self._h, layer)

    def force_h2o_slots(self, slots):
        """The next decode step uses these slots per layer (None: own choice)."""
        if slots is None:
            lib().orc_state_force_h2o_slots(self._h, None)
        else:
            self._forced = np.ascontiguousarray(slots, np.int32)
            lib().orc_state_force_h2o_slots(self._h, self._forced.ctypes.data)

    def routes(self):
        c = self.model.cfg
        n = max(1, (c.n_layers - c.n_dense) * c.top_k)
        ip = lib().orc_state_route_idx(self._h)
        wp = lib().orc_state_route_w(self._h)
        idx = np.ctypeslib.as_array(ctypes.cast(ip, ctypes.POINTER(ctypes.c_int)), (n,)).copy()
        w = np.ctypeslib.as_array(ctypes.cast(wp, ctypes.POINTER(ctypes.c_float)), (n,)).copy()
        return idx, w

    def load_state(self, snap):
        """Resume from a sequence-state snapshot (bytes in the layout of
        cuinf_session_save_state)."""
        buf = np.frombuffer(snap, np.uint8)
        if lib().orc_state_load(self.model._h, self._h, buf.ctypes.data, buf.size) != 0:
            raise ValueError("state snapshot does not fit this model/state")

    @property
    def pos(self):
        return lib().orc_state_pos(self._h)

    def __del__(self):
        # at interpreter exit the module globals may already be gone
        if getattr(self, "_h", None) and callable(lib):
            lib().orc_state_free(self._h)
            self._h = None
