"""Decode engine handles: Model (one device blob) and Session (KV cache,
conv state, CUDA-graph decode step).  Mirrors main() of src/engine.cu
(load 664-692, decode loop 928-963) over the C ABI."""
import ctypes

import torch

from ._lib import CuinfConfig, check, lib
from .weights import default_config


def device_error():
    """Engine kernels' device error flags (0 = none)."""
    v = ctypes.c_uint(0)
    check(lib().cuinf_device_error(ctypes.byref(v)))
    return v.value


class _DevArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


class Model:
    def __init__(self, handle, cfg, keepalive=None):
        self._h = handle
        self.cfg = cfg
        self._keep = keepalive

    @classmethod
    def load(cls, directory, cfg=None):
        cfg = cfg or default_config()
        h = ctypes.c_void_p()
        check(lib().cuinf_model_load(directory.encode(), ctypes.byref(cfg), ctypes.byref(h)))
        return cls(h, cfg)

    @classmethod
    def from_device_blob(cls, blob, index, cfg=None):
        cfg = cfg or default_config()
        h = ctypes.c_void_p()
        ib = (ctypes.c_uint8 * len(index)).from_buffer_copy(index)
        check(lib().cuinf_model_from_device_blob(ctypes.byref(cfg), ctypes.c_void_p(blob.data_ptr()),
                                                 blob.numel(), ib, len(index), ctypes.byref(h)))
        return cls(h, cfg, keepalive=blob)

    def close(self):
        if self._h:
            lib().cuinf_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    def __init__(self, model, max_ctx, stream=None):
        self.model = model
        self.max_ctx = max_ctx
        h = ctypes.c_void_p()
        st = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
        check(lib().cuinf_session_create(model._h, max_ctx, st, ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().cuinf_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self):
        return lib().cuinf_session_pos(self._h)

    def reset(self):
        check(lib().cuinf_session_reset(self._h))

    def save_state(self):
        """Snapshot of the KV cache and conv state at the current position
        (bytes, the layout of cuinf_session_save_state)."""
        import numpy as np
        n = lib().cuinf_session_state_bytes(self._h)
        buf = np.empty(n, np.uint8)
        check(lib().cuinf_session_save_state(self._h, buf.ctypes.data, n))
        return buf.tobytes()

    def load_state(self, snap):
        """Resume from a snapshot: the session moves to its position; the
        next step() must pass a token."""
        import numpy as np
        buf = np.frombuffer(snap, np.uint8)
        check(lib().cuinf_session_load_state(self._h, buf.ctypes.data, buf.size))

    def step(self, token=-1, want=True):
        """One decode step; token < 0 feeds back the previous argmax on the
        device.  Returns the argmax (synchronizes) when want is true."""
        out = ctypes.c_int(-1)
        check(lib().cuinf_decode_step(self._h, int(token), ctypes.byref(out) if want else None))
        return out.value if want else None

    def prefill(self, ids, routes=False):
        """Batched prompt processing (the reference's prefill): returns the
        argmax after the last id, and with routes=True also the expert ids
        each token chose, int32 [S, n_moe_layers, top_k]."""
        import numpy as np
        S = len(ids)
        p = (ctypes.c_int * S)(*[int(t) for t in ids])
        out = ctypes.c_int(-1)
        c = self.model.cfg
        r = np.zeros((S, max(1, c.n_layers - c.n_dense), c.top_k), np.int32) if routes else None
        check(lib().cuinf_prefill(self._h, p, S, ctypes.byref(out),
                                  r.ctypes.data if routes else None))
        return (out.value, r) if routes else out.value

    def set_kv_budget(self, budget, window=0):
        """H2O eviction mode: `budget` FP8 slots per attention layer, local
        window (0: budget/2); before the first token."""
        check(lib().cuinf_session_set_kv_budget(self._h, int(budget), int(window)))
        self._kv_budget = int(budget)

    def h2o_state(self, layer):
        """(slot_pos int32 [budget], attn_sum float32 [budget], n_live, last slot)."""
        import numpy as np
        b = self._kv_budget
        sp = np.zeros(b, np.int32)
        a = np.zeros(b, np.float32)
        n = ctypes.c_int(0)
        last = ctypes.c_int(-1)
        check(lib().cuinf_session_h2o_state(self._h, int(layer), sp.ctypes.data, a.ctypes.data,
                                            ctypes.byref(n), ctypes.byref(last)))
        return sp, a, n.value, last.value

    def generate(self, prompt, n_new, eos=-1):
        p = (ctypes.c_int * len(prompt))(*prompt)
        o = (ctypes.c_int * n_new)()
        n = ctypes.c_int(0)
        check(lib().cuinf_generate(self._h, p, len(prompt), n_new, eos, o, ctypes.byref(n)))
        return list(o[:n.value])

    (OPT_PREFETCH, OPT_PDL, OPT_MEGAKERNEL, OPT_TRACE, OPT_PREFILL, OPT_ATTN_CLUSTER,
     OPT_PREFETCH_MB, OPT_PREFETCH_AHEAD) = 1, 2, 3, 4, 5, 6, 7, 8
    STAGE_KINDS = ("conv_in", "residual", "qkv", "attention", "dense_up", "moe_up", "moe_down",
                   "lm_head")

    def trace(self):
        """Per-stage timestamps of the last traced megakernel step: returns
        (kinds [S], t [S, G, 16]): %globaltimer ns at start, prologue end and
        end (0, 1, 3), slab-wait SM cycles (2); SM cycles since the stage start for
        pre-slab ready (4), the first item's slab ready, dot done and
        epilogue done (5-7), MoE-up norm, router dots and selection done
        (8-10); %clock64 at the stage start (11); producer %clock64 at the
        pre-slab issue (12), first item ready to place (13) and issued (14);
        SM cycles from the stage start to the prologue end (15).
        0 = no such point."""
        import numpy as np
        c = self.model.cfg
        max_stages = 5 * c.n_layers + 1
        cap = max_stages * 1024 * 16
        buf = np.zeros(cap, np.uint64)
        kinds = np.zeros(max_stages, np.int32)
        ns, ng = ctypes.c_int(0), ctypes.c_int(0)
        check(lib().cuinf_session_trace(self._h, buf.ctypes.data, cap, kinds.ctypes.data,
                                        ctypes.byref(ns), ctypes.byref(ng)))
        t = buf[:ns.value * ng.value * 16].reshape(ns.value, ng.value, 16)
        return [self.STAGE_KINDS[k] for k in kinds[:ns.value]], t

    @property
    def uses_megakernel(self):
        return bool(lib().cuinf_session_uses_megakernel(self._h))

    def error(self, detail=False):
        """Megakernel error flags (0 = none); synchronizes the session stream.
        detail=True returns (flags, stage, cta, slab) of the first failure."""
        v = (ctypes.c_uint * 4)()
        check(lib().cuinf_session_error(self._h, v))
        return tuple(v) if detail else v[0]

    def set_option(self, option, value):
        """OPT_PREFETCH: L2 prefetch of upcoming weights; OPT_PDL: programmatic
        dependent launch between the step's kernels (both default on)."""
        check(lib().cuinf_session_set_option(self._h, int(option), int(value)))


    @property
    def attn_cluster(self):
        """True if decode attention can merge its splits over a cluster."""
        return bool(lib().cuinf_session_attn_cluster(self._h))
    def keep_logits(self, on=True):
        check(lib().cuinf_session_keep_logits(self._h, 1 if on else 0))

    def logits(self):
        """Device view (fp32 [vocab]) of the last step's logits (keep_logits on)."""
        ptr = lib().cuinf_session_logits(self._h)
        return torch.as_tensor(_DevArray(ptr, (self.model.cfg.vocab,), "<f4"), device="cuda")

    def hidden(self):
        """Device view (fp16 [hidden]) of the last step's final pre-norm hidden state."""
        ptr = lib().cuinf_session_hidden(self._h)
        return torch.as_tensor(_DevArray(ptr, (self.model.cfg.hidden,), "<f2"), device="cuda")

    def routes(self):
        c = self.model.cfg
        n_moe = c.n_layers - c.n_dense
        n = max(1, n_moe * c.top_k)
        idx = (ctypes.c_int * n)()
        w = (ctypes.c_float * n)()
        check(lib().cuinf_session_routes(self._h, idx, w))
        return list(idx), list(w)

    @property
    def kernels_per_step(self):
        return lib().cuinf_session_kernels_per_step(self._h)

    def profile_step(self, token=-1):
        """One step launched kernel by kernel with events: list of
        (name, ms, algorithmic bytes) per kernel."""
        cap, nl = 1024, 32
        ms = (ctypes.c_float * cap)()
        by = (ctypes.c_double * cap)()
        names = ctypes.create_string_buffer(cap * nl)
        n = ctypes.c_int(0)
        check(lib().cuinf_session_profile_step(self._h, int(token), cap, ms, by, names, nl,
                                               ctypes.byref(n)))
        return [(names.raw[i * nl:(i + 1) * nl].split(b"\0")[0].decode(), ms[i], by[i])
                for i in range(n.value)]


class Batch:
    """Sequence-batched decode (cuinf_batch_*): n_seqs independent sequences
    advance one token per step, all matmuls on the tensor-core GEMMs."""

    def __init__(self, model, n_seqs, max_ctx, stream=None, ep=None):
        """ep = (nccl_id bytes, rank, world) for expert parallelism."""
        self.model = model
        self.n = n_seqs
        h = ctypes.c_void_p()
        st = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
        if ep is None:
            check(lib().cuinf_batch_create(model._h, n_seqs, max_ctx, st, ctypes.byref(h)))
        else:
            uid, rank, world = ep
            buf = (ctypes.c_ubyte * len(uid)).from_buffer_copy(bytes(uid))
            check(lib().cuinf_batch_create_ep(model._h, n_seqs, max_ctx, st, buf, rank, world, ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().cuinf_batch_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        check(lib().cuinf_batch_reset(self._h))

    def step(self, tokens=None, want=True):
        """One step for every sequence; tokens None feeds back each one's
        previous argmax.  Returns the new argmax per sequence when want."""
        t = (ctypes.c_int * self.n)(*[int(x) for x in tokens]) if tokens is not None else None
        o = (ctypes.c_int * self.n)() if want else None
        check(lib().cuinf_batch_step(self._h, t, o))
        return list(o) if want else None

    def keep_logits(self, on=True):
        check(lib().cuinf_batch_keep_logits(self._h, int(on)))

    def sync(self):
        """Wait for the queued steps (expert parallel: polling NCCL errors
        under the batch's time limit)."""
        check(lib().cuinf_batch_sync(self._h))

    def abort(self):
        """Abort the expert-parallel communicator (a peer failed); the batch
        takes no more steps."""
        check(lib().cuinf_batch_abort(self._h))

    def set_timeout(self, ms):
        check(lib().cuinf_batch_set_timeout(self._h, int(ms)))

    @property
    def failed(self):
        return bool(lib().cuinf_batch_failed(self._h))

    @property
    def exchange(self):
        """Expert-parallel row exchange: "peer_memory", "nccl", or None (one GPU)."""
        v = lib().cuinf_batch_ep_exchange(self._h)
        return None if v < 0 else ("peer_memory" if v == 1 else "nccl")

    def set_exchange(self, kind):
        """Select the expert-parallel exchange ("peer_memory" or "nccl"); every
        rank must make the same choice between the same two steps."""
        check(lib().cuinf_batch_set_ep_exchange(self._h, 1 if kind == "peer_memory" else 0))

    def logits(self):
        ptr = lib().cuinf_batch_logits(self._h)
        return torch.as_tensor(_DevArray(ptr, (self.n, self.model.cfg.vocab), "<f4"), device="cuda")

    def routes(self):
        """Experts of the last step, int32 [n_moe_layers, n_seqs, top_k]."""
        import numpy as np
        c = self.model.cfg
        r = np.zeros((max(1, c.n_layers - c.n_dense), self.n, c.top_k), np.int32)
        check(lib().cuinf_batch_routes(self._h, r.ctypes.data))
        return r

    def fill_synthetic(self, ctx, seed=1):
        check(lib().cuinf_batch_fill_synthetic(self._h, int(ctx), int(seed)))

    def save_seq(self, seq):
        """State snapshot of sequence seq (the session snapshot layout)."""
        import numpy as np
        n = lib().cuinf_batch_seq_state_bytes(self._h, int(seq))
        if n == 0:
            raise ValueError("bad sequence index or device error")
        buf = np.empty(n, np.uint8)
        check(lib().cuinf_batch_save_seq(self._h, int(seq), buf.ctypes.data, n))
        return buf.tobytes()

    def load_seq(self, seq, snap):
        """Put sequence seq at a snapshot's state and position."""
        import numpy as np
        buf = np.frombuffer(snap, np.uint8)
        check(lib().cuinf_batch_load_seq(self._h, int(seq), buf.ctypes.data, buf.size))

    @property
    def kernels_per_step(self):
        return lib().cuinf_batch_kernels_per_step(self._h)

    @staticmethod
    def error(detail=False):
        """Tensor-core kernel error flags (0 = none); detail=True returns
        (flags, barrier code, block, stage counter) of the first failure."""
        v = (ctypes.c_uint * 4)()
        check(lib().cuinf_batch_error(v))
        return tuple(v) if detail else v[0]

    def profile_step(self, max_kernels=4096, name_len=32):
        """Eager step with per-launch CUDA-event timing: [(name, ms)]."""
        ms = (ctypes.c_float * max_kernels)()
        names = ctypes.create_string_buffer(max_kernels * name_len)
        n = ctypes.c_int(0)
        check(lib().cuinf_batch_profile_step(self._h, max_kernels, ms, names, name_len, ctypes.byref(n)))
        raw = names.raw
        return [(raw[i * name_len:(i + 1) * name_len].split(b"\0")[0].decode(), ms[i]) for i in range(n.value)]


def ep_unique_id():
    """A fresh NCCL unique id (bytes) for cuinf_batch_create_ep."""
    n = lib().cuinf_ep_unique_id_bytes()
    buf = (ctypes.c_ubyte * n)()
    check(lib().cuinf_ep_unique_id(buf, n))
    return bytes(buf)


def ep_unique_id_shared(group=None):
    """Rank 0's NCCL id broadcast over torch.distributed (any backend)."""
    import torch.distributed as dist
    n = lib().cuinf_ep_unique_id_bytes()
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.zeros(n, dtype=torch.uint8, device=dev)
    if dist.get_rank(group) == 0:
        t.copy_(torch.frombuffer(bytearray(ep_unique_id()), dtype=torch.uint8))
    dist.broadcast(t, src=0, group=group)
    return bytes(t.cpu().numpy().tobytes())
