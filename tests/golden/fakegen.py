"""Deterministic synthetic tensors for format fixtures (test infrastructure).

Every tensor is a function of its name only, so the golden script (which feeds
them to the reference's own exporter) and the tests (which feed them to this
library's writer) see identical float32 inputs without storing them.
"""
import zlib

import numpy as np

# Small dims for format fixtures: the reference exporter hard-codes 24 layers,
# 32 experts and attention at {2,6,10,14,18,21}; shapes come from the tensors.
SMALL = dict(hidden=128, n_heads=2, n_kv_heads=1, head_dim=64, vocab=384,
             dense_inter=256, moe_inter=128, n_experts=32, n_layers=24, n_dense=2,
             attn_layers=(2, 6, 10, 14, 18, 21))


def shape_of(name, c=SMALL):
    H, hd = c["hidden"], c["head_dim"]
    if name == "model.embed_tokens.weight":
        return (c["vocab"], H)
    if name.endswith(("norm.weight",)) and "layernorm" not in name:
        return (H,)
    if name.endswith(("q_layernorm.weight", "k_layernorm.weight")):
        return (hd,)
    if name.endswith("q_proj.weight"):
        return (c["n_heads"] * hd, H)
    if name.endswith(("k_proj.weight", "v_proj.weight")):
        return (c["n_kv_heads"] * hd, H)
    if name.endswith("out_proj.weight") and "self_attn" in name:
        return (H, c["n_heads"] * hd)
    if name.endswith("conv.in_proj.weight"):
        return (3 * H, H)
    if name.endswith("conv.out_proj.weight"):
        return (H, H)
    if name.endswith("conv.conv.weight"):
        return (H, 1, 3)
    if name.endswith("feed_forward.gate.weight"):
        return (c["n_experts"], H)
    if name.endswith("feed_forward.expert_bias"):
        return (c["n_experts"],)
    if ".experts." in name:
        if name.endswith("w2.weight"):
            return (H, c["moe_inter"])
        return (c["moe_inter"], H)
    if name.endswith("feed_forward.w2.weight"):
        return (H, c["dense_inter"])
    if name.endswith(("feed_forward.w1.weight", "feed_forward.w3.weight")):
        return (c["dense_inter"], H)
    raise KeyError(name)


def fake_tensor(name, stored_shape=None, c=SMALL, base_seed=20261201):
    """stored_shape (as the writer stores it) is accepted and ignored: the
    checkpoint shape comes from the name."""
    shape = shape_of(name, c)
    rng = np.random.default_rng((zlib.crc32(name.encode()) + base_seed) & 0xFFFFFFFF)
    if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
        return (1.0 + 0.02 * rng.standard_normal(shape)).astype(np.float32)
    if name.endswith("expert_bias"):
        return (0.1 * rng.standard_normal(shape)).astype(np.float32)
    if name.endswith("conv.conv.weight"):
        b = 1.0 / np.sqrt(3.0)
        return rng.uniform(-b, b, shape).astype(np.float32)
    return (0.02 * rng.standard_normal(shape)).astype(np.float32)
