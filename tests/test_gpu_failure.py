"""Failure paths on the GPU, without faulting it: a bounded device wait whose
barrier never completes gives up after its limit, reports the failure in its
error word, and the context stays usable (the next kernels run and match the
oracle).  Peer failures of the expert-parallel group are covered on CPU by
test_cpu_ep_host.py."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import pyoracle as orc
from cuda_inf_b200 import ops
from cuda_inf_b200._lib import check, lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("limit_us", [2000, 50000])
def test_bounded_wait_gives_up_and_context_survives(cuda, limit_us):
    flags = ctypes.c_uint(0)
    waited = ctypes.c_ulonglong(0)
    check(lib().cuinf_selftest_wait_timeout(limit_us, ctypes.byref(flags), ctypes.byref(waited)))
    assert flags.value == 1, flags.value          # gave up; the barrier never completed
    assert limit_us * 1000 <= waited.value < limit_us * 1000 + 200_000_000, waited.value
    # the device still runs kernels correctly
    rng = np.random.default_rng(limit_us)
    N, K = 256, 512
    packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    scales = rng.uniform(0.005, 0.05, (N, K // 128)).astype(np.float16)
    x = rng.standard_normal(K).astype(np.float16)
    y = ops.gemv_int4(torch.from_numpy(x).to(cuda), torch.from_numpy(packed).to(cuda),
                      torch.from_numpy(scales).to(cuda)).cpu().numpy()
    ref = orc.gemv_int4(x, packed, scales)
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 1e-3
