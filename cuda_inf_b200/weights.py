"""The reference's on-disk weight format: weights.bin + index.bin.

Writer side of tools/export_weights.py (tensor order 96-129, INT4 G=128
quantizer 64-79, fp16 for everything else) and tools/make_index.py (index
record layout 3-11, 21-36), plus seeded synthetic models written straight
into a device blob with the same layout (random init: no checkpoint exists
on this machine).
"""
import ctypes
import hashlib
import os
import struct
import zlib
from dataclasses import dataclass

import numpy as np

from ._lib import CuinfConfig, check, lib

FP16, INT4G = 0, 1


@dataclass
class Entry:
    name: str
    kind: int          # 0 fp16, 1 int4g
    shape: tuple       # logical shape as exported (conv kernel stored [H,3])
    offset: int = 0
    packed: int = 0    # fp16: data bytes; int4g: N*K/2
    scales: int = 0    # int4g: N*(K/128)*2

    @property
    def nbytes(self):
        return self.packed + self.scales


def default_config():
    c = CuinfConfig()
    lib().cuinf_default_config(ctypes.byref(c))
    return c


def make_config(hidden=2048, n_layers=24, n_heads=32, n_kv_heads=8, vocab=128000, n_dense=2,
                n_experts=32, top_k=4, moe_inter=1792, dense_inter=7168,
                attn_layers=(2, 6, 10, 14, 18, 21), rope_theta=5e6, norm_eps=1e-5):
    c = CuinfConfig()
    c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim = hidden, n_layers, n_heads, n_kv_heads, 64
    c.vocab, c.n_dense, c.n_experts, c.top_k = vocab, n_dense, n_experts, top_k
    c.moe_inter, c.dense_inter, c.conv_k = moe_inter, dense_inter, 3
    c.rope_theta, c.norm_eps = rope_theta, norm_eps
    for i in attn_layers:
        c.attn_layer[i] = 1
    return c


def config_dict(c):
    return {f: (list(getattr(c, f)) if f == "attn_layer" else getattr(c, f)) for f, _ in c._fields_}


def layout(c):
    """Tensors in export order (tools/export_weights.py:96-129) with offsets."""
    H, hd = c.hidden, c.head_dim
    ents = [Entry("model.embed_tokens.weight", FP16, (c.vocab, H)),
            Entry("model.embedding_norm.weight", FP16, (H,))]
    for L in range(c.n_layers):
        p = f"model.layers.{L}."
        ents += [Entry(p + "operator_norm.weight", FP16, (H,)), Entry(p + "ffn_norm.weight", FP16, (H,))]
        if c.attn_layer[L]:
            ents += [Entry(p + "self_attn.q_proj.weight", INT4G, (c.n_heads * hd, H)),
                     Entry(p + "self_attn.k_proj.weight", INT4G, (c.n_kv_heads * hd, H)),
                     Entry(p + "self_attn.v_proj.weight", INT4G, (c.n_kv_heads * hd, H)),
                     Entry(p + "self_attn.out_proj.weight", INT4G, (H, c.n_heads * hd)),
                     Entry(p + "self_attn.q_layernorm.weight", FP16, (hd,)),
                     Entry(p + "self_attn.k_layernorm.weight", FP16, (hd,))]
        else:
            ents += [Entry(p + "conv.in_proj.weight", INT4G, (3 * H, H)),
                     Entry(p + "conv.out_proj.weight", INT4G, (H, H)),
                     Entry(p + "conv.conv.weight", FP16, (H, 3))]
        if L < c.n_dense:
            ents += [Entry(p + "feed_forward.w1.weight", INT4G, (c.dense_inter, H)),
                     Entry(p + "feed_forward.w3.weight", INT4G, (c.dense_inter, H)),
                     Entry(p + "feed_forward.w2.weight", INT4G, (H, c.dense_inter))]
        else:
            ents += [Entry(p + "feed_forward.gate.weight", FP16, (c.n_experts, H)),
                     Entry(p + "feed_forward.expert_bias", FP16, (c.n_experts,))]
            for e in range(c.n_experts):
                ep = p + f"feed_forward.experts.{e}."
                ents += [Entry(ep + "w1.weight", INT4G, (c.moe_inter, H)),
                         Entry(ep + "w3.weight", INT4G, (c.moe_inter, H)),
                         Entry(ep + "w2.weight", INT4G, (H, c.moe_inter))]
    off = 0
    for e in ents:
        if e.kind == FP16:
            e.packed, e.scales = int(np.prod(e.shape)) * 2, 0
        else:
            N, K = e.shape
            e.packed, e.scales = N * K // 2, N * (K // 128) * 2
        e.offset = off
        off += e.nbytes
    return ents


def index_bytes(ents):
    """index.bin (tools/make_index.py:3-11): u32 n; per tensor u8 len, name,
    u8 kind, u64 offset, u64 packed, u64 scales, i64 d0, i64 d1."""
    out = [struct.pack("<I", len(ents))]
    for e in ents:
        nb = e.name.encode()
        d0 = e.shape[0]
        d1 = e.shape[1] if len(e.shape) > 1 else 0
        out += [struct.pack("<B", len(nb)), nb, struct.pack("<B", e.kind),
                struct.pack("<QQQ", e.offset, e.packed, e.scales), struct.pack("<qq", d0, d1)]
    return b"".join(out)


def quantize_int4_host(w):
    """Bit-exact host copy of the export quantizer (libcuinf, no GPU needed)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    packed = np.empty((N, K // 2), np.uint8)
    scales = np.empty((N, K // 128), np.uint16)
    check(lib().cuinf_quantize_int4_host(w.ctypes.data, N, K, packed.ctypes.data, scales.ctypes.data))
    return packed, scales


def write_model(out_dir, c, get_tensor):
    """Write weights.bin + index.bin from float32 tensors get_tensor(name,
    shape) (shape as stored; the conv kernel may come as [H,1,3] like the
    checkpoint).  Returns the sha256 of weights.bin."""
    os.makedirs(out_dir, exist_ok=True)
    ents = layout(c)
    h = hashlib.sha256()
    with open(os.path.join(out_dir, "weights.bin"), "wb") as f:
        for e in ents:
            w = np.asarray(get_tensor(e.name, e.shape), dtype=np.float32)
            if e.kind == FP16:
                b = w.reshape(e.shape).astype(np.float16).tobytes()
            else:
                p, s = quantize_int4_host(w.reshape(e.shape))
                b = p.tobytes() + s.tobytes()
            assert len(b) == e.nbytes, e.name
            f.write(b)
            h.update(b)
    with open(os.path.join(out_dir, "index.bin"), "wb") as f:
        f.write(index_bytes(ents))
    return h.hexdigest()


# ---------------------------------------------------------------------------
# seeded random-init models on the device
# ---------------------------------------------------------------------------
def init_kind(name):
    """HF-style random init: Linear/Embedding N(0, 0.02), RMSNorm weights
    1 + N(0, 0.02), depthwise conv U(-1/sqrt(3), 1/sqrt(3)) (Conv1d default
    with fan_in 3), expert bias N(0, 0.1)."""
    if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
        return "norm"
    if name.endswith("expert_bias"):
        return "bias"
    if name.endswith("conv.conv.weight"):
        return "conv"
    return "linear"


def synth_tensor_torch(name, shape, seed, device):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed((zlib.crc32(name.encode()) + seed) & 0x7FFFFFFF)
    k = init_kind(name)
    if k == "conv":
        b = 1.0 / np.sqrt(3.0)
        return (torch.rand(shape, generator=g, device=device, dtype=torch.float32) * 2 - 1) * b
    t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if k == "norm":
        return 1.0 + 0.02 * t
    if k == "bias":
        return 0.1 * t
    return 0.02 * t


def synth_device_blob(c, seed=1234, device="cuda"):
    """Random-init model quantized on the GPU into one device blob laid out
    exactly like weights.bin.  Returns (blob uint8 tensor, index bytes)."""
    import torch
    from . import ops
    ents = layout(c)
    total = ents[-1].offset + ents[-1].nbytes
    blob = torch.empty(total, dtype=torch.uint8, device=device)
    for e in ents:
        w = synth_tensor_torch(e.name, e.shape, seed, device)
        dst = blob[e.offset:e.offset + e.nbytes]
        if e.kind == FP16:
            dst.view(torch.float16).copy_(w.reshape(-1).to(torch.float16))
        else:
            N, K = e.shape
            p, s = ops.quantize_int4(w.contiguous())
            dst[:e.packed].copy_(p.reshape(-1))
            dst[e.packed:].view(torch.float16).copy_(s.reshape(-1))
        del w
    torch.cuda.synchronize()
    return blob, index_bytes(ents)


def save_blob(blob, idx, out_dir):
    """Write a device blob + index as weights.bin/index.bin (for the reference
    engine, which reads files)."""
    os.makedirs(out_dir, exist_ok=True)
    host = blob.cpu().numpy()
    with open(os.path.join(out_dir, "weights.bin"), "wb") as f:
        f.write(host.tobytes())
    with open(os.path.join(out_dir, "index.bin"), "wb") as f:
        f.write(idx)
