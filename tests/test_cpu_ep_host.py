"""Host side of expert parallelism on CPU, as gloo ranks (no GPU):

  * the dispatch plan (cuinf_ep_plan_host, the index math the device runs in
    k_ep_plan) with the exchange and the slot-ordered combine, at world
    sizes 2 and 4: every token's result equals a direct computation
    bit-for-bit;
  * failure detection between steps (StepGuard / GuardedBatch): a rank whose
    step raises, or that leaves, or whose process exits, makes the other
    ranks' next step raise PeerFailure (within the guard's timeout) and abort
    their batch, instead of hanging in a collective.
"""
import os
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

H, E, TOPK, B = 16, 8, 2, 5


def _collect(q, procs, n, limit_s):
    """n results from the workers' queue; fails fast if a worker died first."""
    import queue
    out, t0 = [], time.time()
    while len(out) < n:
        try:
            out.append(q.get(timeout=1.0))
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead and time.time() - t0 < limit_s, ("workers failed or hung", dead, out)
    return out


def _half_chain(h, outs, w):
    """acc = half(acc + w_t * o_t) in slot order, then h = half(h + acc)."""
    acc = np.zeros(H, np.float16)
    for o, wt in zip(outs, w):
        acc = (acc.astype(np.float32) + np.float32(wt) * o).astype(np.float16)
    return (h.astype(np.float32) + acc.astype(np.float32)).astype(np.float16)


def _plan_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from cuda_inf_b200.ep import ep_plan
    e_loc, cap = E // world, B * TOPK
    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((B, H)).astype(np.float16)
    h = rng.standard_normal((B, H)).astype(np.float16)
    ridx = np.stack([rng.choice(E, TOPK, replace=False) for _ in range(B)]).astype(np.int32)  # [B, K]
    w = rng.uniform(0.1, 0.6, (B, TOPK)).astype(np.float32)
    dest, meta = ep_plan(ridx.ravel(), e_loc, world, cap)
    # pack, exchange rows and their local expert ids
    send_x = np.zeros((world * cap, H), np.float16)
    for j in range(B * TOPK):
        send_x[dest[j]] = x[j // TOPK]
    recv_x = torch.zeros(world * cap, H, dtype=torch.float16)
    recv_m = torch.zeros(world * cap, dtype=torch.int32)
    dist.all_to_all_single(recv_x, torch.from_numpy(send_x))
    dist.all_to_all_single(recv_m, torch.from_numpy(meta))
    # this rank's "experts": out = x * (global expert id + 1), in fp32
    rx, rm = recv_x.numpy(), recv_m.numpy()
    out = np.zeros((world * cap, H), np.float32)
    for i in range(world * cap):
        if rm[i] >= 0:
            out[i] = rx[i].astype(np.float32) * np.float32(rank * e_loc + rm[i] + 1)
    back = torch.zeros(world * cap, H, dtype=torch.float32)
    dist.all_to_all_single(back, torch.from_numpy(out))
    back = back.numpy()
    ok = True
    for b in range(B):
        got = _half_chain(h[b], [back[dest[b * TOPK + t]] for t in range(TOPK)], w[b])
        want = _half_chain(h[b], [x[b].astype(np.float32) * np.float32(ridx[b, t] + 1) for t in range(TOPK)], w[b])
        ok = ok and np.array_equal(got.view(np.uint16), want.view(np.uint16))
    q.put((rank, ok, int((meta >= 0).sum())))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,port", [(2, 29641), (4, 29643)])
def test_dispatch_plan_exchange_and_combine(world, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_plan_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(q, procs, world, 180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in got), got
    # every rank sent every one of its B*TOPK rows exactly once
    assert sum(n for _, _, n in got) == world * B * TOPK


class _FakeBatch:
    """Stands in for an expert-parallel Batch on CPU: records steps and aborts."""

    def __init__(self, fail_at=None):
        self.steps, self.aborted, self.fail_at = 0, False, fail_at

    def step(self, tokens=None, want=True):
        self.steps += 1
        if self.fail_at is not None and self.steps == self.fail_at:
            raise RuntimeError("injected step failure")
        return [0]

    def abort(self):
        self.aborted = True


def _guard_worker(rank, world, port, mode, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from cuda_inf_b200.ep import GuardedBatch, PeerFailure, StepGuard
    guard = StepGuard(timeout_s=5.0)
    fb = _FakeBatch(fail_at=3 if (rank == 1 and mode == "raise") else None)
    gb = GuardedBatch(fb, guard)
    t0 = time.time()
    result = "ran"
    for i in range(6):
        if rank == 1 and mode == "leave" and i == 3:
            gb.leave()
            result = "left"
            break
        if rank == 1 and mode == "exit" and i == 3:
            q.put((rank, "exited", fb.steps, fb.aborted, time.time() - t0))
            q.close()
            q.join_thread()  # the result reaches the parent before the process vanishes
            os._exit(0)  # the process disappears between steps
        try:
            gb.step([1])
        except PeerFailure:
            result = "peer_failure"
            break
        except RuntimeError:
            result = "own_failure"
            # tell the others at their next check, as a failing rank does
            try:
                guard.check(False)
            except PeerFailure:
                pass
            break
    q.put((rank, result, fb.steps, fb.aborted, time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("mode,port", [("raise", 29651), ("leave", 29653), ("exit", 29655)])
def test_peer_failure_between_steps(mode, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_guard_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for r, result, steps, aborted, dt in _collect(q, procs, 2, 120):
        got[r] = (result, steps, aborted, dt)
    for p in procs:
        p.join(timeout=60)
    r0 = got[0]
    # rank 0 noticed at its next check, aborted its batch, and did not hang
    assert r0[0] == "peer_failure", got
    assert r0[2] is True, got
    assert r0[3] < 60, got
    assert r0[1] == 3, got  # it stepped 3 times; the 4th check failed
