"""Host side of expert parallelism on CPU: rank 0's NCCL unique id reaches
every rank intact through torch.distributed (gloo, world size 2)."""
import os

import torch.multiprocessing as mp


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from cuda_inf_b200.engine import ep_unique_id_shared
    from cuda_inf_b200._lib import lib
    uid = ep_unique_id_shared()
    q.put((rank, uid, lib().cuinf_ep_unique_id_bytes()))
    dist.barrier()
    dist.destroy_process_group()


def test_ep_unique_id_broadcast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, 29631, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ids = {r: u for r, u, _ in got}
    assert ids[0] == ids[1] and len(ids[0]) == got[0][2] == 128
