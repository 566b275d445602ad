"""GPU parity of every operator of the C ABI against the CPU oracle.

Tolerances (stated by the path's contract): GEMV outputs within 1e-3 relative
(max-abs error / max-abs reference), attention within 2e-3; fp16 elementwise
results within one fp16 ulp; integer/byte results (FP8 codes, scales,
quantizer, routing indices, argmax, unpacked INT4 weights) bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import pyoracle as orc
from cuda_inf_b200 import ops

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3
ATTN_TOL = 2e-3


def relerr(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def ulp_diff_f16(a, b):
    ai = np.asarray(a, np.float16).view(np.int16).astype(np.int32)
    bi = np.asarray(b, np.float16).view(np.int16).astype(np.int32)
    ai = np.where(ai < 0, -32768 - ai, ai)
    bi = np.where(bi < 0, -32768 - bi, bi)
    return int(np.max(np.abs(ai - bi))) if ai.size else 0


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def int4_weights(rng, N, K):
    """Config-1 distribution: nibbles uniform 0..15, fp16 scales log-uniform
    in [0.005, 0.05]."""
    packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    scales = np.exp(rng.uniform(np.log(0.005), np.log(0.05), (N, K // 128))).astype(np.float16)
    return packed, scales


@pytest.mark.parametrize("N,K,M", [(7168, 2048, 1), (512, 2048, 1), (2048, 7168, 1),
                                   (2048, 1792, 2), (1792, 2048, 1), (6144, 2048, 1),
                                   (40, 256, 3), (16, 128, 1)])
def test_gemv_int4(cuda, N, K, M):
    rng = np.random.default_rng(N * 7 + K + M)
    packed, scales = int4_weights(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float16)
    ref = orc.gemv_int4(x, packed, scales)
    y = ops.gemv_int4(T(x, cuda), T(packed, cuda), T(scales, cuda))
    assert relerr(y.cpu().numpy(), ref) < GEMV_TOL


def test_gemv_int4_unpacked_weights_bit_exact(cuda):
    """One-hot inputs read the dequantized weights (nib-8)*scale out of the
    GEMV exactly: they must equal the reference dequant bit for bit."""
    rng = np.random.default_rng(11)
    N, K = 48, 256
    packed, scales = int4_weights(rng, N, K)
    x = np.eye(K, dtype=np.float16)
    y = ops.gemv_int4(T(x, cuda), T(packed, cuda), T(scales, cuda)).cpu().numpy()  # [K, N]
    ref = orc.dequant_int4(packed, scales).T
    assert np.array_equal(y.view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_gemv_int4_quantized_normal(cuda):
    rng = np.random.default_rng(5)
    w = (0.02 * rng.standard_normal((2048, 2048))).astype(np.float32)
    p, s = orc.quant_int4_group(w)
    x = rng.standard_normal(2048).astype(np.float16)
    ref = orc.gemv_int4(x, p, s)
    y = ops.gemv_int4(T(x, cuda), T(p, cuda), T(s, cuda))
    assert relerr(y.cpu().numpy(), ref) < GEMV_TOL


@pytest.mark.parametrize("N,K,M", [(4096, 2048, 1), (32, 2048, 1), (1000, 256, 2)])
def test_gemv_fp16(cuda, N, K, M):
    rng = np.random.default_rng(N + K)
    W = (0.02 * rng.standard_normal((N, K))).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    ref = orc.gemv_fp16(x, W)
    y = ops.gemv_fp16(T(x, cuda), T(W, cuda))
    assert relerr(y.cpu().numpy(), ref) < GEMV_TOL


@pytest.mark.parametrize("M,D", [(3, 2048), (40, 64)])
def test_rmsnorm(cuda, M, D):
    rng = np.random.default_rng(M + D)
    x = (rng.standard_normal((M, D)) * 3).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    ref = orc.rmsnorm(x, w)
    out = ops.rmsnorm(T(x, cuda), T(w, cuda)).cpu().numpy()
    assert ulp_diff_f16(out, ref) <= 1


def test_rope(cuda):
    rng = np.random.default_rng(9)
    pos = np.array([0, 1, 4095, 32767], np.int32)
    q = rng.standard_normal((4, 32, 64)).astype(np.float16)
    k = rng.standard_normal((4, 8, 64)).astype(np.float16)
    rq, rk = orc.rope(q, k, pos)
    tq, tk = T(q, cuda), T(k, cuda)
    ops.rope(tq, tk, T(pos, cuda))
    np.testing.assert_allclose(tq.cpu().numpy().astype(np.float32), rq.astype(np.float32), atol=4e-3)
    np.testing.assert_allclose(tk.cpu().numpy().astype(np.float32), rk.astype(np.float32), atol=4e-3)


def _kv_cache(rng, n_tok, nkv=8, zero_head=False):
    """Tokens [0, n_tok) committed to FP8 by the oracle in 64-token groups,
    the remainder kept as the fp16 tail (kv placement, engine.cu:831-845)."""
    K = rng.standard_normal((n_tok, nkv, 64)).astype(np.float16)
    V = rng.standard_normal((n_tok, nkv, 64)).astype(np.float16)
    if zero_head:
        K[:, 1] = 0
        V[:, 2] = 0
    committed = (n_tok // 64) * 64
    T_ = max(committed, 64)
    kc8 = np.zeros((T_, nkv, 64), np.uint8)
    vc8 = np.zeros_like(kc8)
    ksc = np.zeros((T_ // 64 + 1, nkv), np.float16)
    vsc = np.zeros_like(ksc)
    for g in range(committed // 64):
        orc.kv_commit_group(K[g * 64:(g + 1) * 64], V[g * 64:(g + 1) * 64], kc8, vc8, ksc, vsc, g * 64, g)
    ktail = np.zeros((64, nkv, 64), np.float16)
    vtail = np.zeros_like(ktail)
    tl = n_tok - committed
    ktail[:tl] = K[committed:]
    vtail[:tl] = V[committed:]
    return K, V, kc8, vc8, ksc, vsc, ktail, vtail, committed


def test_kv_commit_group_bit_exact(cuda):
    rng = np.random.default_rng(21)
    for zero in (False, True):
        K = (rng.standard_normal((64, 8, 64)) * rng.uniform(0.01, 30)).astype(np.float16)
        V = (rng.standard_normal((64, 8, 64)) * rng.uniform(0.01, 30)).astype(np.float16)
        if zero:
            K[:, 3] = 0
        kc8 = np.zeros((128, 8, 64), np.uint8)
        vc8 = np.zeros_like(kc8)
        ksc = np.zeros((3, 8), np.float16)
        vsc = np.zeros_like(ksc)
        orc.kv_commit_group(K, V, kc8, vc8, ksc, vsc, 64, 1)
        g = [T(a, cuda) for a in (K, V, np.zeros_like(kc8), np.zeros_like(vc8), np.zeros_like(ksc),
                                   np.zeros_like(vsc))]
        ops.kv_commit_group(*g, 64, 1)
        for a, b in zip(g[2:], (kc8, vc8, ksc, vsc)):
            assert np.array_equal(a.cpu().numpy().view(np.uint8), b.view(np.uint8))


def test_kv_write_tail(cuda):
    rng = np.random.default_rng(22)
    k = rng.standard_normal((3, 8, 64)).astype(np.float16)
    v = rng.standard_normal((3, 8, 64)).astype(np.float16)
    kt = torch.zeros((64, 8, 64), dtype=torch.float16, device=cuda)
    vt = torch.zeros_like(kt)
    ops.kv_write_tail(T(k, cuda), T(v, cuda), kt, vt, 10, 3)
    assert np.array_equal(kt[10:13].cpu().numpy(), k) and np.array_equal(vt[10:13].cpu().numpy(), v)
    assert kt[:10].abs().sum().item() == 0 and kt[13:].abs().sum().item() == 0


@pytest.mark.parametrize("n_tok", [1, 5, 63, 64, 65, 127, 128, 200, 2048, 4113, 8192, 32768])
def test_attn_decode(cuda, n_tok):
    rng = np.random.default_rng(n_tok)
    K, V, kc8, vc8, ksc, vsc, ktail, vtail, committed = _kv_cache(rng, n_tok, zero_head=n_tok == 200)
    q = rng.standard_normal((32, 64)).astype(np.float16)
    qpos = n_tok - 1
    ref = orc.attn_decode(q, kc8, vc8, ksc, vsc, ktail, vtail, committed, qpos)
    out = ops.attn_decode(*(T(a, cuda) for a in (q, kc8, vc8, ksc, vsc, ktail, vtail)), committed, qpos)
    assert relerr(out.cpu().numpy(), ref) < ATTN_TOL


def test_attn_decode_full_tail(cuda):
    """Tail of exactly 64 fp16 tokens (committed lags by a full group)."""
    rng = np.random.default_rng(77)
    K, V, kc8, vc8, ksc, vsc, ktail, vtail, committed = _kv_cache(rng, 128)
    ktail[:] = K[64:128]
    vtail[:] = V[64:128]
    q = rng.standard_normal((32, 64)).astype(np.float16)
    ref = orc.attn_decode(q, kc8, vc8, ksc, vsc, ktail, vtail, 64, 127)
    out = ops.attn_decode(*(T(a, cuda) for a in (q, kc8, vc8, ksc, vsc, ktail, vtail)), 64, 127)
    assert relerr(out.cpu().numpy(), ref) < ATTN_TOL


@pytest.mark.parametrize("S", [1, 4])
def test_shortconv(cuda, S):
    H = 2048
    rng = np.random.default_rng(S)
    inproj = rng.standard_normal((S, 3 * H)).astype(np.float32)
    w = rng.uniform(-0.577, 0.577, (H, 3)).astype(np.float16)
    state = rng.standard_normal((2, H)).astype(np.float16)
    C, Bx = orc.conv_pre(inproj, S, H)
    y = orc.conv_apply(Bx, C, w, state, S, H)
    st2 = orc.conv_update_state(Bx, state, S, H)
    tC = torch.empty((S, H), dtype=torch.float16, device=cuda)
    tB = torch.empty_like(tC)
    ops.conv_pre(T(inproj, cuda), tC, tB, S, H)
    assert np.array_equal(tC.cpu().numpy(), C) and np.array_equal(tB.cpu().numpy(), Bx)
    ty = torch.empty_like(tC)
    tst = T(state, cuda)
    ops.conv_apply(tB, tC, T(w, cuda), tst, ty, S, H)
    assert ulp_diff_f16(ty.cpu().numpy(), y) <= 1
    ops.conv_update_state(tB, tst, S, H)
    assert np.array_equal(tst.cpu().numpy(), st2)


def test_elementwise(cuda):
    rng = np.random.default_rng(31)
    n = 7168
    g = rng.standard_normal(n).astype(np.float32) * 3
    u = rng.standard_normal(n).astype(np.float32)
    out = torch.empty(n, dtype=torch.float16, device=cuda)
    ops.swiglu(T(g, cuda), T(u, cuda), out)
    ref = orc.swiglu(g, u)
    np.testing.assert_allclose(out.cpu().numpy().astype(np.float32), ref.astype(np.float32),
                               rtol=2e-3, atol=1e-4)
    a = rng.standard_normal(n).astype(np.float16)
    b = rng.standard_normal(n).astype(np.float16)
    f = rng.standard_normal(n).astype(np.float32)
    ta = T(a, cuda)
    ops.add_inplace(ta, T(b, cuda))
    assert np.array_equal(ta.cpu().numpy(), orc.add_inplace(a, b))
    ta = T(a, cuda)
    ops.add_f32_inplace(ta, T(f, cuda))
    assert np.array_equal(ta.cpu().numpy(), orc.add_f32_inplace(a, f))
    ta = T(a, cuda)
    ops.acc_scaled(ta, T(f, cuda), 0.37)
    assert ulp_diff_f16(ta.cpu().numpy(), orc.acc_scaled(a, f, 0.37)) <= 1
    th = torch.empty(n, dtype=torch.float16, device=cuda)
    ops.f32_to_f16(T(f, cuda), th)
    assert np.array_equal(th.cpu().numpy(), f.astype(np.float16))
    emb = rng.standard_normal((50, 256)).astype(np.float16)
    ids = np.array([3, 49, 0], np.int32)
    o = torch.empty((3, 256), dtype=torch.float16, device=cuda)
    ops.embed_gather(T(emb, cuda), T(ids, cuda), o)
    assert np.array_equal(o.cpu().numpy(), emb[ids])


def test_argmax_tie_rule(cuda):
    rng = np.random.default_rng(41)
    for trial in range(6):
        n = [128000, 1000, 3000, 5, 257, 128000][trial]
        v = rng.standard_normal(n).astype(np.float32)
        if trial % 2 == 0 and n > 600:
            v[[7, 263, 519]] = 11.0  # tie: same value at indices 7, 263 (=7 mod 256), 519
            v[300] = 11.0            # and at 300 (44 mod 256)
        if trial == 5:
            v = rng.integers(0, 3, n).astype(np.float32)
        out = ops.argmax(T(v, cuda)).item()
        assert out == orc.argmax(v)


def test_moe_route_bit_exact(cuda):
    """Given identical router logits the selected experts equal the
    reference's host selection (engine.cu:883-892) bit for bit."""
    rng = np.random.default_rng(51)
    S, E, K = 512, 32, 4
    logits = rng.standard_normal((S, E)).astype(np.float32) * 2
    bias = (0.1 * rng.standard_normal(E)).astype(np.float16)
    logits[::7, 9] = logits[::7, 4]  # exact score ties on some tokens
    idx, w = ops.moe_route(T(logits, cuda), T(bias, cuda), K)
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    exact_w = 0
    for s in range(S):
        ri, rw = orc.moe_select(logits[s], bias.astype(np.float32), K)
        assert list(idx[s]) == list(ri)
        np.testing.assert_allclose(w[s], rw, rtol=1e-6)
        exact_w += int(np.array_equal(w[s].view(np.uint32), rw.view(np.uint32)))
    assert exact_w >= S * 0.99  # weights: bit-exact except for 1-ulp expf differences


def test_quantize_int4_device_bit_exact(cuda):
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_int4.npz"))
    for name in ("normal", "wide", "ties", "tiny", "big"):
        p, s = ops.quantize_int4(T(z[name + "_w"], cuda))
        assert np.array_equal(p.cpu().numpy(), z[name + "_packed"]), name
        assert np.array_equal(s.cpu().numpy().view(np.uint16), z[name + "_scales"]), name


def test_moe_ffn_fused(cuda):
    """Fused router + top-k + experts + fp16 weighted accumulate + residual
    against the oracle's composition of the reference kernels."""
    rng = np.random.default_rng(61)
    H, I, E, K = 2048, 1792, 32, 4
    xn = rng.standard_normal(H).astype(np.float16)
    gate = (0.02 * rng.standard_normal((E, H))).astype(np.float16)
    bias = (0.1 * rng.standard_normal(E)).astype(np.float16)
    h = rng.standard_normal(H).astype(np.float16)
    ex = []
    for e in range(E):
        ex.append([int4_weights(rng, I, H), int4_weights(rng, I, H), int4_weights(rng, H, I)])
    # oracle
    logits = orc.gemv_fp16(xn, gate)
    ri, rw = orc.moe_select(logits, bias.astype(np.float32), K)
    acc = np.zeros(H, np.float16)
    for t in range(K):
        (p1, s1), (p3, s3), (p2, s2) = ex[ri[t]]
        g = orc.gemv_int4(xn, p1, s1)
        u = orc.gemv_int4(xn, p3, s3)
        mid = orc.swiglu(g, u)
        o = orc.gemv_int4(mid, p2, s2)
        acc = orc.acc_scaled(acc, o, float(rw[t]))
    href = orc.add_inplace(h, acc)
    # device
    dev_ex = [[T(a, cuda) for pair in e for a in pair] for e in ex]
    table = ops.expert_table(dev_ex)
    th = T(h, cuda)
    idx = torch.empty(K, dtype=torch.int32, device=cuda)
    w = torch.empty(K, dtype=torch.float32, device=cuda)
    ops.moe_ffn(T(xn, cuda), T(gate, cuda), T(bias, cuda), table, th, K, I, idx, w)
    assert list(idx.cpu().numpy()) == list(ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-5)
    assert relerr(th.cpu().numpy().astype(np.float32) - h.astype(np.float32),
                  href.astype(np.float32) - h.astype(np.float32)) < 5e-3
