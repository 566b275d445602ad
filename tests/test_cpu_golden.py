"""CPU tests: pin the oracle (and the product's host-side format code) to
golden vectors produced by the reference's own code (tests/golden/make_golden.py
runs tools/export_weights.py and tools/make_index.py of g023/cuda_inf)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import pyoracle
from cuda_inf_b200 import weights

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _quant_cases():
    z = np.load(os.path.join(GOLDEN, "quant_int4.npz"))
    names = sorted({k.rsplit("_", 1)[0] for k in z.files})
    return [(n, z[n + "_w"], z[n + "_packed"], z[n + "_scales"]) for n in names]


@pytest.mark.parametrize("case", _quant_cases(), ids=lambda c: c[0])
def test_oracle_quantizer_matches_reference(case):
    """orc_quant_int4_group == quant_int4_group (export_weights.py:64-79), bit-exact."""
    _, w, packed, scales = case
    p, s = pyoracle.quant_int4_group(w)
    assert np.array_equal(p, packed)
    assert np.array_equal(s.view(np.uint16), scales)


@pytest.mark.parametrize("case", _quant_cases(), ids=lambda c: c[0])
def test_product_host_quantizer_matches_reference(case):
    """libcuinf's host quantizer (format writer) is bit-exact too."""
    _, w, packed, scales = case
    p, s = weights.quantize_int4_host(w)
    assert np.array_equal(p, packed)
    assert np.array_equal(s, scales)


def test_format_writer_matches_reference_exporter(tmp_path):
    """weights.bin/index.bin written by this library are byte-identical to
    the ones tools/export_weights.py + tools/make_index.py wrote for the same
    float inputs (small dims, full 24-layer / 32-expert structure)."""
    import fakegen
    info = json.load(open(os.path.join(GOLDEN, "format_small.json")))
    c = info["config"]
    cfg = weights.make_config(hidden=c["hidden"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                              vocab=c["vocab"], dense_inter=c["dense_inter"],
                              moe_inter=c["moe_inter"], n_experts=c["n_experts"],
                              n_layers=c["n_layers"], n_dense=c["n_dense"],
                              attn_layers=c["attn_layers"])
    sha = weights.write_model(str(tmp_path), cfg, fakegen.fake_tensor)
    assert os.path.getsize(tmp_path / "weights.bin") == info["weights_bytes"]
    assert sha == info["weights_sha256"]
    ib = open(tmp_path / "index.bin", "rb").read()
    assert ib == open(os.path.join(GOLDEN, "index_small.bin"), "rb").read()
    assert len(weights.layout(cfg)) == info["n_tensors"]


def test_default_layout_size():
    """The full LFM2.5-8B-A1B layout is 4,757,814,144 bytes (README ~4.76 GB)."""
    ents = weights.layout(weights.make_config())
    assert ents[-1].offset + ents[-1].nbytes == 4_757_814_144
    assert all(e.offset % 16 == 0 for e in ents)


def test_fp8_decode_all_codes_vs_torch():
    """E4M3 decode of all 256 codes equals torch.float8_e4m3fn (OCP E4M3)."""
    codes = np.arange(256, dtype=np.uint8)
    ours = pyoracle.e4m3_decode(codes)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan], ref[~nan])


def test_fp8_encode_vs_torch_in_range():
    """RNE encode equals torch's float -> e4m3fn cast inside the finite range;
    beyond 448 the reference's SATFINITE clamps (torch gives NaN there)."""
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(4000) * 50, rng.uniform(-448, 448, 2000),
                        np.array([0.0, -0.0, 2 ** -9, 2 ** -10, 3 * 2 ** -11, 447.9, -447.9, 464.0 - 1e-3])])
    x = x.astype(np.float32)
    ours = pyoracle.e4m3_encode(x)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)
    big = np.array([449.0, 1e6, -1e6, np.inf, -np.inf], np.float32)
    assert list(pyoracle.e4m3_encode(big)) == [0x7E, 0x7E, 0xFE, 0x7E, 0xFE]


def test_oracle_gemv_int4_vs_numpy():
    rng = np.random.default_rng(1)
    w = (0.02 * rng.standard_normal((48, 384))).astype(np.float32)
    p, s = pyoracle.quant_int4_group(w)
    x = rng.standard_normal((2, 384)).astype(np.float16)
    deq = pyoracle.dequant_int4(p, s).astype(np.float64)
    ref = x.astype(np.float64) @ deq.T
    y = pyoracle.gemv_int4(x, p, s)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)


def _argmax_ref_kernel(v):
    """Direct restatement of argmax_kernel (engine.cu:562-572) with 256 threads."""
    bv, bi = [], []
    for tid in range(256):
        best, bidx = np.float32(-1e30), 0
        for i in range(tid, len(v), 256):
            if v[i] > best:
                best, bidx = v[i], i
        bv.append(best)
        bi.append(bidx)
    s = 128
    while s > 0:
        for t in range(s):
            if bv[t + s] > bv[t]:
                bv[t], bi[t] = bv[t + s], bi[t + s]
        s >>= 1
    return bi[0]


def test_oracle_argmax_tie_rule():
    rng = np.random.default_rng(2)
    v = rng.standard_normal(3000).astype(np.float32)
    v[[5, 261, 1000, 2000]] = 9.0  # ties: winner has the smallest index mod 256
    assert pyoracle.argmax(v) == _argmax_ref_kernel(v)
    for _ in range(5):
        v = rng.integers(0, 4, 1000).astype(np.float32)
        assert pyoracle.argmax(v) == _argmax_ref_kernel(v)


def _select_ref(logits, bias, topk):
    """numpy-float32 restatement of engine.cu:883-892."""
    f = np.float32
    sig = [f(1.0) / (f(1.0) + np.exp(f(-z), dtype=np.float32)) for z in logits]
    score = [f(s + b) for s, b in zip(sig, bias)]
    used = [False] * len(logits)
    sel, w = [], []
    for _ in range(topk):
        best, bv = -1, f(-1e30)
        for e in range(len(logits)):
            if not used[e] and score[e] > bv:
                bv, best = score[e], e
        used[best] = True
        sel.append(best)
        w.append(sig[best])
    ws = f(0)
    for x in w:
        ws = f(ws + x)
    return sel, [f(x / f(ws + f(1e-6))) for x in w]


def test_oracle_moe_select():
    rng = np.random.default_rng(3)
    for t in range(20):
        lg = rng.standard_normal(32).astype(np.float32)
        b = rng.standard_normal(32).astype(np.float16).astype(np.float32) * np.float32(0.1)
        if t % 4 == 0:
            lg[7] = lg[3]
            b[7] = b[3]  # exact tie: lower index first
        idx, w = pyoracle.moe_select(lg, b, 4)
        sel, ww = _select_ref(lg, b, 4)
        assert list(idx) == sel
        np.testing.assert_allclose(w, ww, rtol=2e-7)


def test_argmax_key_rule_matches_reference_tree():
    """The device argmax encodes ties as 'smallest bit-reversed index mod 256,
    then smallest index' (argmax_key in csrc/common.cuh); that rule equals the
    result of argmax_kernel's tree reduction on heavy-tie inputs."""
    def brev8(r):
        return int("{:08b}".format(r)[::-1], 2)

    def key_argmax(v):
        best = None
        for i, x in enumerate(v):
            if x > -1e30:
                k = (float(x), -((brev8(i & 255) << 23) | (i >> 8)))
                if best is None or k > best[0]:
                    best = (k, i)
        return best[1] if best else 0

    rng = np.random.default_rng(4)
    for _ in range(60):
        n = int(rng.integers(1, 3000))
        v = rng.integers(0, int(rng.integers(1, 6)), n).astype(np.float32)
        assert key_argmax(v) == _argmax_ref_kernel(v)


def test_oracle_prefill_semantics(tmp_path):
    """The oracle's batched prefill (engine.cu:784-917) equals decoding the
    same ids one by one while no KV group commits inside it (every key is
    then read from the fp16 tail in both), and differs once one does (the
    prefill's queries then read their own group's keys as FP8)."""
    import zlib
    cfg = weights.make_config(hidden=128, n_layers=3, n_heads=2, n_kv_heads=1, vocab=300, n_dense=1,
                              n_experts=8, top_k=2, moe_inter=128, dense_inter=128, attn_layers=(1, 2))

    def tensor(name, shape):
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        k = weights.init_kind(name)
        if k == "norm":
            return (1 + 0.02 * rng.standard_normal(shape)).astype(np.float32)
        if k == "conv":
            return rng.uniform(-0.577, 0.577, shape).astype(np.float32)
        return (0.05 * rng.standard_normal(shape)).astype(np.float32)

    weights.write_model(str(tmp_path), cfg, tensor)
    om = pyoracle.Model(weights.config_dict(cfg), np.fromfile(tmp_path / "weights.bin", np.uint8),
                        open(tmp_path / "index.bin", "rb").read())
    toks = np.random.default_rng(3).integers(0, cfg.vocab, 80)
    a, b = om.state(128), om.state(128)
    for t in toks[:20]:
        a.forward(int(t), want_logits=False)
        b.forward(int(t), want_logits=False)
    n1, lg1, sc = a.prefill(toks[20:40])  # positions 20..39: no commit
    for t in toks[20:40]:
        n2, lg2, _, _ = b.forward_ex(int(t))
    assert n1 == n2 and np.array_equal(lg1, lg2) and a.pos == b.pos == 40
    assert sc.shape == (20, 2, 8)  # [S, moe layers, experts]
    n1, lg1, _ = a.prefill(toks[40:80])  # commits group 0 at position 64
    for t in toks[40:80]:
        n2, lg2, _, _ = b.forward_ex(int(t))
    assert not np.array_equal(lg1, lg2)
    assert np.abs(lg1 - lg2).max() < 0.1 * np.abs(lg2).max()


def test_oracle_h2o_policy(tmp_path):
    """The oracle's H2O slot choice (engine.cu:808-823): append while there is
    room, then the least cumulative attention outside the local window (first
    minimum), else the least overall; the chosen slot's mass restarts at 0 and
    its position becomes the token's.  Without eviction a prefill equals
    decoding the same ids."""
    import zlib
    cfg = weights.make_config(hidden=128, n_layers=3, n_heads=2, n_kv_heads=1, vocab=300, n_dense=1,
                              n_experts=8, top_k=2, moe_inter=128, dense_inter=128, attn_layers=(1, 2))

    def tensor(name, shape):
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        k = weights.init_kind(name)
        if k == "norm":
            return (1 + 0.02 * rng.standard_normal(shape)).astype(np.float32)
        if k == "conv":
            return rng.uniform(-0.577, 0.577, shape).astype(np.float32)
        return (0.05 * rng.standard_normal(shape)).astype(np.float32)

    weights.write_model(str(tmp_path), cfg, tensor)
    om = pyoracle.Model(weights.config_dict(cfg), np.fromfile(tmp_path / "weights.bin", np.uint8),
                        open(tmp_path / "index.bin", "rb").read())
    C, W = 8, 3
    st = om.state(64)
    st.set_h2o(C, W)
    toks = np.random.default_rng(9).integers(0, cfg.vocab, 30)
    for pos, t in enumerate(toks):
        a, sp, n = st.h2o_layer(1)
        if n < C:
            want = n
        else:
            elig = [i for i in range(C) if sp[i] <= pos - W]
            pool = elig if elig else list(range(C))
            want = min(pool, key=lambda i: (a[i], i))
        st.forward_ex(int(t))
        own, used = st.h2o_slots()
        assert own[1] == used[1] == want, (pos, own[1], want)
        a2, sp2, n2 = st.h2o_layer(1)
        assert sp2[want] == pos and n2 == min(pos + 1, C)
    # prefill == decode while nothing is evicted
    s1, s2 = om.state(64), om.state(64)
    s1.set_h2o(16, 8)
    s2.set_h2o(16, 8)
    n1, lg1, _ = s1.prefill(toks[:12])
    for t in toks[:12]:
        n2, lg2, _, _ = s2.forward_ex(int(t))
    assert n1 == n2 and np.array_equal(lg1, lg2)
