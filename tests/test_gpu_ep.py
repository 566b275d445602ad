"""Expert-parallel batched decode on 2 GPUs (one process per GPU; rows
exchanged through peer memory, and by NCCL send/recv in a second batch):
each rank's sequences must follow the CPU oracle.  Skipped with fewer than 2
GPUs.  The host-side NCCL id exchange is covered on CPU by
test_cpu_ep_id.py."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("n_local,steps", [(3, 70), (32, 4)])
def test_ep_two_ranks_match_oracle(n_local, steps):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29617",
           os.path.join(ROOT, "tests", "ep_worker.py"), str(n_local), str(steps)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    out = r.stdout + r.stderr
    print("\n".join(l for l in out.splitlines() if l.startswith("EP rank")))
    assert r.returncode == 0, out[-3000:]
    assert out.count("EP rank") == 2
