"""Golden vectors from the reference's own kernels (src/engine.cu of
g023/cuda_inf rebuilt for sm_100a into oracle/_ref/libref.so) on seeded
inputs.  Needs a GPU; run on the B200 box:

    python tests/golden/make_ref_kernel_golden.py [--out tests/golden/ref_kernels.npz]

The CPU suite then pins the oracle to these outputs (test_cpu_ref_golden.py).
Dimensions are the reference's compile-time ones (H=2048, NH=32, NKV=8).
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import refkernels as rk  # noqa: E402
from oracle import pyoracle as orc  # noqa: E402


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make(out):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    d = rk.dims()
    H, NH, NKV = d["H"], d["NH"], d["NKV"]
    rng = np.random.default_rng(2026)
    z = {}
    # gemv_int4 (config-1 value distribution), two rows of x
    N, K = 96, 2048
    packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    scales = np.exp(rng.uniform(np.log(0.005), np.log(0.05), (N, K // 128))).astype(np.float16)
    x = rng.standard_normal((2, K)).astype(np.float16)
    y = torch.empty((2, N), dtype=torch.float32, device=dev)
    rk.call("gemv_int4", T(x), T(packed), T(scales), y, 2, N, K)
    z.update(gemv_x=x, gemv_packed=packed, gemv_scales=scales, gemv_y=y.cpu().numpy())
    # gemv_fp16 (router shape)
    W = (0.02 * rng.standard_normal((32, H))).astype(np.float16)
    xf = rng.standard_normal(H).astype(np.float16)
    yf = torch.empty(32, dtype=torch.float32, device=dev)
    rk.call("gemv_fp16", T(xf), T(W), yf, 1, 32, H)
    z.update(gemvf_x=xf, gemvf_W=W, gemvf_y=yf.cpu().numpy())
    # rmsnorm / rmsnorm_head
    xr = (3 * rng.standard_normal((3, H))).astype(np.float16)
    wr = (1 + 0.1 * rng.standard_normal(H)).astype(np.float16)
    o = torch.empty_like(T(xr))
    rk.call("rmsnorm", T(xr), T(wr), o, 3, H, 1e-5)
    z.update(rms_x=xr, rms_w=wr, rms_y=o.cpu().numpy())
    xh = rng.standard_normal((40, 64)).astype(np.float16)
    wh = (1 + 0.1 * rng.standard_normal(64)).astype(np.float16)
    oh = torch.empty_like(T(xh))
    rk.call("rmsnorm_head", T(xh), T(wh), oh, 40, 1e-5)
    z.update(rmsh_x=xh, rmsh_w=wh, rmsh_y=oh.cpu().numpy())
    # rope at small and large positions
    pos = np.array([0, 5, 4095, 32767], np.int32)
    q = rng.standard_normal((4, NH, 64)).astype(np.float16)
    k = rng.standard_normal((4, NKV, 64)).astype(np.float16)
    tq, tk = T(q), T(k)
    rk.call("rope", tq, tk, T(pos), 4)
    z.update(rope_pos=pos, rope_q=q, rope_k=k, rope_qo=tq.cpu().numpy(), rope_ko=tk.cpu().numpy())
    # FP8 E4M3 round trip through f2e4m3 / e4m3f
    xs = np.concatenate([rng.standard_normal(6000) * 60, rng.uniform(-500, 500, 3000),
                         np.exp(rng.uniform(-14, 7, 3000)) * rng.choice([-1, 1], 3000),
                         [0.0, -0.0, 448.0, 464.0, 480.0, -1e9, 1e9, 2 ** -9, 2 ** -10, 1.5 * 2 ** -9]])
    xs = xs.astype(np.float32)
    enc = torch.empty(xs.size, dtype=torch.uint8, device=dev)
    dec = torch.empty(xs.size, dtype=torch.float32, device=dev)
    rk.call("fp8_roundtrip", T(xs), enc, dec, xs.size)
    z.update(fp8_x=xs, fp8_enc=enc.cpu().numpy(), fp8_dec=dec.cpu().numpy())
    # KV: tail writes of 200 tokens with commits at 64/128/192, then attention
    n_tok = 200
    Kv = rng.standard_normal((n_tok, NKV, 64)).astype(np.float16)
    Vv = rng.standard_normal((n_tok, NKV, 64)).astype(np.float16)
    Kv[:, 3] *= 20
    Vv[:, 5] *= 0.01
    kc8 = torch.zeros((256, NKV, 64), dtype=torch.uint8, device=dev)
    vc8 = torch.zeros_like(kc8)
    ksc = torch.zeros((6, NKV), dtype=torch.float16, device=dev)
    vsc = torch.zeros_like(ksc)
    kt = torch.zeros((64, NKV, 64), dtype=torch.float16, device=dev)
    vt = torch.zeros_like(kt)
    committed = 0
    for t in range(n_tok):
        slot = t - committed
        rk.call("kv_write_tail", T(Kv[t]), T(Vv[t]), kt, vt, slot, 1)
        if slot + 1 == 64:
            rk.call("kv_commit_group", kt, vt, kc8, vc8, ksc, vsc, committed, committed // 64)
            committed += 64
    qa = rng.standard_normal((NH, 64)).astype(np.float16)
    pm = torch.empty(NH * d["NSPLIT"], dtype=torch.float32, device=dev)
    pl = torch.empty_like(pm)
    po = torch.empty(NH * d["NSPLIT"] * 64, dtype=torch.float32, device=dev)
    ao = torch.empty((NH, 64), dtype=torch.float16, device=dev)
    rk.call("attn_decode", T(qa), kc8, vc8, ksc, vsc, kt, vt, committed, n_tok - 1, 0.125, pm, pl, po, ao)
    z.update(kv_K=Kv, kv_V=Vv, kv_kc8=kc8.cpu().numpy(), kv_vc8=vc8.cpu().numpy(),
             kv_ksc=ksc.cpu().numpy(), kv_vsc=vsc.cpu().numpy(), kv_ktail=kt.cpu().numpy(),
             kv_vtail=vt.cpu().numpy(), kv_committed=np.int32(committed), attn_q=qa,
             attn_out=ao.cpu().numpy())
    # short conv, S = 1 and S = 3
    for S in (1, 3):
        inproj = rng.standard_normal((S, 3 * H)).astype(np.float32)
        w = rng.uniform(-0.577, 0.577, (H, 3)).astype(np.float16)
        state = rng.standard_normal((2, H)).astype(np.float16)
        C = torch.empty((S, H), dtype=torch.float16, device=dev)
        Bx = torch.empty_like(C)
        yy = torch.empty_like(C)
        ts = T(state)
        rk.call("conv_pre", T(inproj), C, Bx, S)
        rk.call("conv_apply", Bx, C, T(w), ts, yy, S)
        rk.call("conv_update_state", Bx, ts, S)
        z.update({f"conv{S}_inproj": inproj, f"conv{S}_w": w, f"conv{S}_state": state,
                  f"conv{S}_C": C.cpu().numpy(), f"conv{S}_Bx": Bx.cpu().numpy(),
                  f"conv{S}_y": yy.cpu().numpy(), f"conv{S}_state_out": ts.cpu().numpy()})
    # elementwise
    n = 4096
    g = (3 * rng.standard_normal(n)).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    sw = torch.empty(n, dtype=torch.float16, device=dev)
    rk.call("swiglu", T(g), T(u), sw, n)
    a16 = rng.standard_normal(n).astype(np.float16)
    src = rng.standard_normal(n).astype(np.float32)
    ta = T(a16)
    rk.call("acc_scaled", ta, T(src), 0.3125, n)
    z.update(ew_g=g, ew_u=u, ew_swiglu=sw.cpu().numpy(), ew_a=a16, ew_src=src,
             ew_acc=ta.cpu().numpy())
    # argmax with ties
    v = rng.standard_normal(5000).astype(np.float32)
    v[[9, 265, 777, 4000]] = 7.5
    am = torch.empty(1, dtype=torch.int32, device=dev)
    rk.call("argmax", T(v), 5000, am)
    z.update(argmax_v=v, argmax_i=am.cpu().numpy())
    torch.cuda.synchronize()
    np.savez_compressed(out, **z)
    print("wrote", out, sum(a.nbytes for a in z.values()), "bytes raw")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "ref_kernels.npz"))
    a = ap.parse_args()
    make(a.out)
