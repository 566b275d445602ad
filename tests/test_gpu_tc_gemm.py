"""Tensor-core (tcgen05) GEMMs against a plain PyTorch fp32 reference of the
same op: the INT4 dequant-GEMM y = x . ((nib-8)*scale)^T (gemv_int4,
engine.cu:83-109, at M activation rows) and the fp16 lm_head GEMM with its
fused argmax (gemv_fp16 + argmax_kernel, engine.cu:112-128, 562-572).

Tolerance: max-abs error / max-abs reference < 1e-3 (the contract); the
INT4 path is in fact exact up to fp32 summation order (the MMA sums exact
products (nib-8)*x per 128-K group and the fp32 scale is applied per group),
which the tests hold to 2e-5.  Split-K reduces in a fixed order, so repeated
runs are bit-identical.  Shapes with more than 148 tiles give a CTA several
work items and more than 8 K stages per item (the packed ring wraps).
"""
import numpy as np
import pytest
import torch

from oracle import pyoracle as orc
from cuda_inf_b200 import ops
from cuda_inf_b200.engine import Batch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def relerr(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def int4_case(seed, M, N, K, dev):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    scales = torch.exp(torch.empty(N, K // 128).uniform_(np.log(0.005), np.log(0.05), generator=g)).half()
    x = torch.randn(M, K, generator=g).half()
    return packed.to(dev), scales.to(dev), x.to(dev)


def dequant_f32(packed, scales):
    lo = (packed & 15).float()
    hi = (packed >> 4).float()
    q = torch.stack([lo, hi], dim=-1).reshape(packed.shape[0], -1) - 8.0
    return q * scales.float().repeat_interleave(128, dim=1)


@pytest.mark.parametrize("M,N,K", [(1, 7168, 2048), (64, 6144, 2048), (64, 2048, 7168), (37, 1000, 256),
                                   (128, 512, 2048), (200, 1792, 2048), (16, 128, 128), (8, 2048, 1792),
                                   (64, 20480, 2048), (24, 19200, 1536)])
def test_gemm_int4_tc_vs_torch_fp32(cuda, M, N, K):
    packed, scales, x = int4_case(M * 1000 + N + K, M, N, K, cuda)
    ref = x.float() @ dequant_f32(packed, scales).t()
    y = ops.gemm_int4_tc(x, packed, scales)
    torch.cuda.synchronize()
    e = relerr(y, ref)
    print(f"M={M} N={N} K={K}: rel err {e:.2e}")
    assert e < TOL and e < 2e-5
    y2 = ops.gemm_int4_tc(x, packed, scales)
    assert torch.equal(y, y2)  # deterministic split-K
    assert Batch.error() == 0


def test_gemm_int4_tc_vs_oracle(cuda):
    """Pinned to the CPU oracle (orc.gemv_int4) on a small case too."""
    packed, scales, x = int4_case(7, 5, 384, 512, cuda)
    ref = orc.gemv_int4(x.cpu().numpy(), packed.cpu().numpy(), scales.cpu().numpy())
    y = ops.gemm_int4_tc(x, packed, scales).cpu()
    assert relerr(y, torch.from_numpy(np.asarray(ref))) < TOL


@pytest.mark.parametrize("M,N,K", [(64, 4196, 2048), (3, 1000, 256), (128, 640, 128), (64, 25600, 2048),
                                   (64, 64000, 2048)])
def test_gemm_fp16_tc_argmax(cuda, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    W = (0.02 * torch.randn(N, K, generator=g)).half().to(cuda)
    x = torch.randn(M, K, generator=g).half().to(cuda)
    ref = x.float() @ W.float().t()
    y, idx = ops.gemm_fp16_tc(x, W)
    torch.cuda.synchronize()
    assert relerr(y, ref) < TOL
    assert idx == torch.argmax(y, dim=1).tolist()  # the argmax of its own logits
    _, idx2 = ops.gemm_fp16_tc(x, W, want_logits=False)
    assert idx2 == idx
    assert Batch.error() == 0
