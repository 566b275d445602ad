"""GPU: this library's kernels against the reference's own kernels run live
(src/engine.cu rebuilt for sm_100a in oracle/_ref/libref.so) on identical
inputs at the reference's dimensions.  Same tolerances as test_gpu_ops."""
import numpy as np
import pytest
import torch

from oracle import refkernels as rk
from cuda_inf_b200 import ops

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not rk.available(), reason="oracle/_ref/libref.so not built")]


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


@pytest.mark.parametrize("N,K", [(7168, 2048), (2048, 7168), (2048, 1792), (512, 2048)])
def test_gemv_int4_vs_reference_kernel(cuda, N, K):
    rng = np.random.default_rng(N + K)
    packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    scales = np.exp(rng.uniform(np.log(0.005), np.log(0.05), (N, K // 128))).astype(np.float16)
    x = rng.standard_normal(K).astype(np.float16)
    yr = torch.empty(N, dtype=torch.float32, device=cuda)
    rk.call("gemv_int4", T(x), T(packed), T(scales), yr, 1, N, K)
    y = ops.gemv_int4(T(x), T(packed), T(scales))
    assert rel(y.cpu().numpy(), yr.cpu().numpy()) < 1e-3


def test_kv_and_attention_vs_reference_kernels(cuda):
    d = rk.dims()
    NH, NKV = d["NH"], d["NKV"]
    rng = np.random.default_rng(5)
    n_tok = 1000
    K = rng.standard_normal((n_tok, NKV, 64)).astype(np.float16)
    V = rng.standard_normal((n_tok, NKV, 64)).astype(np.float16)
    bufs = {}
    for side in ("ref", "ours"):
        kc8 = torch.zeros((1024, NKV, 64), dtype=torch.uint8, device=cuda)
        vc8 = torch.zeros_like(kc8)
        ksc = torch.zeros((17, NKV), dtype=torch.float16, device=cuda)
        vsc = torch.zeros_like(ksc)
        kt = torch.zeros((64, NKV, 64), dtype=torch.float16, device=cuda)
        vt = torch.zeros_like(kt)
        committed = 0
        for t in range(n_tok):
            slot = t - committed
            if side == "ref":
                rk.call("kv_write_tail", T(K[t]), T(V[t]), kt, vt, slot, 1)
            else:
                ops.kv_write_tail(T(K[t]), T(V[t]), kt, vt, slot, 1)
            if slot + 1 == 64:
                if side == "ref":
                    rk.call("kv_commit_group", kt, vt, kc8, vc8, ksc, vsc, committed, committed // 64)
                else:
                    ops.kv_commit_group(kt, vt, kc8, vc8, ksc, vsc, committed, committed // 64)
                committed += 64
        bufs[side] = (kc8, vc8, ksc, vsc, kt, vt, committed)
    for a, b in zip(bufs["ref"][:6], bufs["ours"][:6]):
        assert torch.equal(a, b)  # FP8 codes, scales and tails bit-exact
    kc8, vc8, ksc, vsc, kt, vt, committed = bufs["ref"]
    q = T(rng.standard_normal((NH, 64)).astype(np.float16))
    pm = torch.empty(NH * d["NSPLIT"], dtype=torch.float32, device=cuda)
    pl = torch.empty_like(pm)
    po = torch.empty(NH * d["NSPLIT"] * 64, dtype=torch.float32, device=cuda)
    outr = torch.empty((NH, 64), dtype=torch.float16, device=cuda)
    rk.call("attn_decode", q, kc8, vc8, ksc, vsc, kt, vt, committed, n_tok - 1, 0.125, pm, pl, po, outr)
    out = ops.attn_decode(q, kc8, vc8, ksc, vsc, kt, vt, committed, n_tok - 1)
    assert rel(out.cpu().numpy(), outr.cpu().numpy()) < 2e-3


def test_argmax_vs_reference_kernel(cuda):
    rng = np.random.default_rng(8)
    v = rng.standard_normal(128000).astype(np.float32)
    v[[100, 356, 1000]] = 6.0
    r = torch.empty(1, dtype=torch.int32, device=cuda)
    rk.call("argmax", T(v), v.size, r)
    assert ops.argmax(T(v)).item() == r.item()
