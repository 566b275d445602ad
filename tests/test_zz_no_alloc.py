"""cuinf_attn_decode_noalloc: attention with the library's static scratch.

Checks the allocation-free entry point against the workspace entry point
(cuinf_attn_decode) and the CPU oracle on the same inputs, two calls in a
row, and that a shape whose split-K scratch exceeds the static array is
rejected before any launch.  The file is named to be collected last so that
it runs both after the other GPU tests and alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import pyoracle as orc
from cuda_inf_b200 import ops
from cuda_inf_b200._lib import lib

pytestmark = pytest.mark.gpu

ATTN_TOL = 2e-3  # relative max-abs error, same bar as cuinf_attn_decode


def _relerr(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _cache(rng, n_tok, nkv):
    """Tokens [0, n_tok): full 64-token groups committed to FP8 by the oracle,
    the rest in the fp16 tail."""
    K = rng.standard_normal((n_tok, nkv, 64)).astype(np.float16)
    V = rng.standard_normal((n_tok, nkv, 64)).astype(np.float16)
    committed = (n_tok // 64) * 64
    T_ = max(committed, 64)
    kc8 = np.zeros((T_, nkv, 64), np.uint8)
    vc8 = np.zeros_like(kc8)
    ksc = np.zeros((T_ // 64 + 1, nkv), np.float16)
    vsc = np.zeros_like(ksc)
    for g in range(committed // 64):
        sl = slice(g * 64, (g + 1) * 64)
        orc.kv_commit_group(K[sl], V[sl], kc8, vc8, ksc, vsc, g * 64, g)
    ktail = np.zeros((64, nkv, 64), np.float16)
    vtail = np.zeros_like(ktail)
    ktail[:n_tok - committed] = K[committed:]
    vtail[:n_tok - committed] = V[committed:]
    return kc8, vc8, ksc, vsc, ktail, vtail, committed


def _dev(arrs, dev):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in arrs]


def test_static_scratch_size():
    assert lib().cuinf_attn_decode_static_scratch_bytes() == 512 * 1024


@pytest.mark.parametrize("n_tok", [1, 100, 4096, 8192])
def test_noalloc_matches_workspace_entry(cuda, n_tok):
    rng = np.random.default_rng(1000 + n_tok)
    kc8, vc8, ksc, vsc, ktail, vtail, committed = _cache(rng, n_tok, 8)
    qpos = n_tok - 1
    for _ in range(2):  # two calls in a row, fresh queries each time
        q = rng.standard_normal((32, 64)).astype(np.float16)
        g = _dev((q, kc8, vc8, ksc, vsc, ktail, vtail), cuda)
        ref_dev = ops.attn_decode(*g, committed, qpos)
        out = torch.full_like(g[0], float("nan"))
        ops.attn_decode_noalloc(*g, committed, qpos, out=out)
        torch.cuda.synchronize()
        ref_cpu = orc.attn_decode(q, kc8, vc8, ksc, vsc, ktail, vtail, committed, qpos)
        o = out.cpu().numpy()
        assert np.all(np.isfinite(o))
        assert _relerr(o, ref_dev.cpu().numpy()) < ATTN_TOL
        assert _relerr(o, ref_cpu) < ATTN_TOL


def test_noalloc_rejects_oversized_scratch(cuda):
    """8 kv heads x 8 query heads at 2048 tokens need 32 splits x 8 x 8
    partials = 0.53 MiB of scratch: rejected with CUINF_ERR_ARG, no launch."""
    rng = np.random.default_rng(7)
    kc8, vc8, ksc, vsc, ktail, vtail, committed = _cache(rng, 2048, 8)
    q = rng.standard_normal((64, 64)).astype(np.float16)
    g = _dev((q, kc8, vc8, ksc, vsc, ktail, vtail), cuda)
    out = torch.zeros_like(g[0])
    p = [ctypes.c_void_p(t.data_ptr()) for t in g]
    rc = lib().cuinf_attn_decode_noalloc(*p, committed, 2047, ctypes.c_float(0.125),
                                          ctypes.c_void_p(out.data_ptr()), 64, 8,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1
    assert b"512 KiB" in lib().cuinf_last_error()
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0
