"""One rank of the expert-parallel batched-decode parity run (launched by
tests/test_gpu_ep.py through torch.distributed.run, one process per GPU).

Each rank decodes its own sequences with experts sharded across the ranks
(cuinf_batch_create_ep, rows exchanged through peer memory) and checks every
one of them against the CPU oracle, teacher-forced, exactly as the
single-GPU batch test does; a second batch with the vocabulary-sharded
lm_head and the NCCL send/recv exchange must produce the same tokens.
Prints one line "EP rank R: ..." and exits non-zero on a mismatch."""
import datetime
import os
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import pyoracle as orc  # noqa: E402
from cuda_inf_b200 import weights  # noqa: E402
from cuda_inf_b200.engine import Batch, Model, ep_unique_id_shared  # noqa: E402
from enginecheck import TINY, check_logits, check_routes, tiny_tensor  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    n_local, steps = int(sys.argv[1]), int(sys.argv[2])
    cfg = weights.make_config(**TINY)
    with tempfile.TemporaryDirectory() as d:
        weights.write_model(d, cfg, tiny_tensor)
        blob = np.fromfile(os.path.join(d, "weights.bin"), np.uint8)
        index = open(os.path.join(d, "index.bin"), "rb").read()
        om = orc.Model(weights.config_dict(cfg), blob, index)
        gm = Model.load(d, cfg)
    uid = ep_unique_id_shared()
    bt = Batch(gm, n_local, max_ctx=160, ep=(uid, rank, world))
    bt.keep_logits(True)
    # every rank draws the global token matrix, then takes its own columns
    toks = np.random.default_rng(4242).integers(0, cfg.vocab, (steps, n_local * world))
    mine = toks[:, rank * n_local:(rank + 1) * n_local]
    states = [om.state(160) for _ in range(n_local)]
    # a second batch on the same tokens without kept logits: its lm_head is
    # sharded by vocabulary over the ranks (argmax keys max-reduced), and its
    # tokens must equal the replicated lm_head's bit for bit
    bt2 = Batch(gm, n_local, max_ctx=160, ep=(ep_unique_id_shared(), rank, world))  # its own communicator
    assert bt.exchange == "peer_memory", bt.exchange
    bt2.set_exchange("nccl")
    assert bt2.exchange == "nccl"
    worst, checked, near = 0.0, 0, 0
    for i in range(steps):
        got = bt.step(mine[i])
        got2 = bt2.step(mine[i])
        assert got2 == got, (rank, i, got, got2)
        routes = bt.routes()
        glog = bt.logits().cpu().numpy()
        for b in range(n_local):
            gi = routes[:, b, :]
            ref, lg, _, sc = states[b].forward_ex(int(mine[i, b]), forced_idx=gi.ravel())
            c, n = check_routes(gi, sc, cfg.top_k, 1e-3, (rank, i, b))
            checked += c
            near += n
            worst = max(worst, check_logits(glog[b], lg, got[b], ref, 1e-2, (rank, i, b)))
    assert checked > 0.9 * (checked + near), (checked, near)
    assert Batch.error() == 0
    print(f"EP rank {rank}/{world}: {n_local} sequences x {steps} steps, worst logits rel err {worst:.2e}, "
          f"routing checked {checked}, near-ties {near}; peer-memory and NCCL exchanges agree", flush=True)
    bt.close()  # the step graph holds NCCL calls: release it before the process group
    bt2.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
