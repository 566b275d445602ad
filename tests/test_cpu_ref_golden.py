"""CPU: pin the oracle to golden outputs of the reference's own kernels
(tests/golden/ref_kernels.npz, made on a B200 by make_ref_kernel_golden.py
from src/engine.cu rebuilt for sm_100a).

Bit-exact where the reference's arithmetic is exact or a single IEEE
rounding (FP8 encode/decode, kv commit, conv_pre, state update, argmax);
otherwise within the fp32-reduction-order tolerance stated per test."""
import os

import numpy as np
import pytest

from oracle import pyoracle as orc

PATH = os.path.join(os.path.dirname(__file__), "golden", "ref_kernels.npz")
pytestmark = pytest.mark.skipif(not os.path.exists(PATH), reason="ref_kernels.npz not generated yet")


@pytest.fixture(scope="module")
def z():
    return np.load(PATH)


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


def ulp16(a, b):
    ai = np.asarray(a, np.float16).view(np.int16).astype(np.int32)
    bi = np.asarray(b, np.float16).view(np.int16).astype(np.int32)
    ai = np.where(ai < 0, -32768 - ai, ai)
    bi = np.where(bi < 0, -32768 - bi, bi)
    return int(np.max(np.abs(ai - bi)))


def test_fp8_roundtrip_bit_exact(z):
    assert np.array_equal(orc.e4m3_encode(z["fp8_x"]), z["fp8_enc"])
    d = orc.e4m3_decode(z["fp8_enc"])
    assert np.array_equal(d.view(np.uint32), z["fp8_dec"].view(np.uint32))


def test_gemv_int4(z):
    assert rel(orc.gemv_int4(z["gemv_x"], z["gemv_packed"], z["gemv_scales"]), z["gemv_y"]) < 1e-5


def test_gemv_fp16(z):
    assert rel(orc.gemv_fp16(z["gemvf_x"], z["gemvf_W"]), z["gemvf_y"]) < 1e-5


def test_rmsnorm(z):
    assert ulp16(orc.rmsnorm(z["rms_x"], z["rms_w"]), z["rms_y"]) <= 1
    assert ulp16(orc.rmsnorm(z["rmsh_x"], z["rmsh_w"]), z["rmsh_y"]) <= 1


def test_rope(z):
    """The angle pos * theta^(-2d/64) is fp32 on both sides; libm and CUDA
    powf/cosf differ by an ulp, which at pos 32767 moves the angle by up to
    ~1e-3 rad: |diff| <= 4e-3 for inputs ~N(0,1); exact at small positions."""
    q, k = orc.rope(z["rope_q"], z["rope_k"], z["rope_pos"])
    for a, b in ((q, z["rope_qo"]), (k, z["rope_ko"])):
        d = np.abs(a.astype(np.float64) - b.astype(np.float64))
        assert d.max() <= 4e-3
        assert d[:2].max() == 0.0


def test_kv_commit_bit_exact(z):
    K, V = z["kv_K"], z["kv_V"]
    kc8 = np.zeros_like(z["kv_kc8"])
    vc8 = np.zeros_like(kc8)
    ksc = np.zeros_like(z["kv_ksc"])
    vsc = np.zeros_like(ksc)
    committed = int(z["kv_committed"])
    for g in range(committed // 64):
        orc.kv_commit_group(K[g * 64:(g + 1) * 64], V[g * 64:(g + 1) * 64], kc8, vc8, ksc, vsc, g * 64, g)
    assert np.array_equal(kc8, z["kv_kc8"]) and np.array_equal(vc8, z["kv_vc8"])
    assert np.array_equal(ksc.view(np.uint16), z["kv_ksc"].view(np.uint16))
    assert np.array_equal(vsc.view(np.uint16), z["kv_vsc"].view(np.uint16))
    tl = K.shape[0] - committed
    assert np.array_equal(z["kv_ktail"][:tl], K[committed:])


def test_attention(z):
    out = orc.attn_decode(z["attn_q"], z["kv_kc8"], z["kv_vc8"], z["kv_ksc"], z["kv_vsc"],
                          z["kv_ktail"], z["kv_vtail"], int(z["kv_committed"]), z["kv_K"].shape[0] - 1)
    assert rel(out, z["attn_out"]) < 2e-3


@pytest.mark.parametrize("S", [1, 3])
def test_shortconv(z, S):
    H = z[f"conv{S}_w"].shape[0]
    C, Bx = orc.conv_pre(z[f"conv{S}_inproj"], S, H)
    assert np.array_equal(C, z[f"conv{S}_C"]) and np.array_equal(Bx, z[f"conv{S}_Bx"])
    y = orc.conv_apply(Bx, C, z[f"conv{S}_w"], z[f"conv{S}_state"], S, H)
    assert ulp16(y, z[f"conv{S}_y"]) <= 1
    st = orc.conv_update_state(Bx, z[f"conv{S}_state"], S, H)
    assert np.array_equal(st, z[f"conv{S}_state_out"])


def test_elementwise(z):
    sw = orc.swiglu(z["ew_g"], z["ew_u"])
    np.testing.assert_allclose(sw.astype(np.float32), z["ew_swiglu"].astype(np.float32), rtol=2e-3, atol=1e-4)
    acc = orc.acc_scaled(z["ew_a"], z["ew_src"], 0.3125)
    assert ulp16(acc, z["ew_acc"]) <= 1


def test_argmax(z):
    assert orc.argmax(z["argmax_v"]) == int(z["argmax_i"][0])
