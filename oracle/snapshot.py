"""Random sequence-state snapshots (the layout of cuinf_session_save_state).
TEST INFRASTRUCTURE: used by tests/ and by bench.py's CPU baseline to start
the engine and the oracle at a long context without a long prompt: every attention layer gets committed FP8 groups quantized from
N(0,1) keys/values by the reference's commit rule (scale = absmax/448 +
1e-12 per (group, kv head), codes = e4m3(x / scale); engine.cu:202-228) and
an fp16 tail, every short-conv layer a random fp16 state."""
import struct

import numpy as np
import torch

MAGIC, VERSION = 0x54534943, 1


def _fp8_group_codes(x):
    """x float32 [G, 64, nkv, 64] -> (codes u8 same shape, scales fp16 [G, nkv])."""
    amax = np.abs(x).max(axis=(1, 3))                     # [G, nkv]
    sc32 = (amax / np.float32(448.0) + np.float32(1e-12)).astype(np.float32)
    q = x / sc32[:, None, :, None]
    codes = torch.from_numpy(np.ascontiguousarray(q)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return codes, sc32.astype(np.float16)


def random_snapshot(cfg, pos, seed):
    """bytes of a snapshot at position pos with seeded random contents."""
    rng = np.random.default_rng(seed)
    nkv, H = cfg.n_kv_heads, cfg.hidden
    C = (pos // 64) * 64
    out = [struct.pack("<IIiiiiii", MAGIC, VERSION, pos, cfg.n_layers, H, nkv, 0, 0)]
    for l in range(cfg.n_layers):
        if cfg.attn_layer[l]:
            parts = []
            for _ in range(2):  # K then V
                x = rng.standard_normal((C // 64, 64, nkv, 64), dtype=np.float32)
                codes, sc = _fp8_group_codes(x)
                parts.append((codes.tobytes(), sc.tobytes()))
            tails = []
            for _ in range(2):
                t = np.zeros((64, nkv, 64), np.float16)
                t[:pos - C] = rng.standard_normal((pos - C, nkv, 64)).astype(np.float16)
                tails.append(t.tobytes())
            out += [parts[0][0], parts[1][0], parts[0][1], parts[1][1], tails[0], tails[1]]
        else:
            out.append((0.8 * rng.standard_normal((2, H))).astype(np.float16).tobytes())
    return b"".join(out)
