"""Host side of expert-parallel batched decode across processes (one per
GPU): the per-layer dispatch plan on the host, and a liveness check between
steps.  The reference runs on one GPU (src/engine.cu:2) and has neither.

The device step (cuinf_batch_create_ep) exchanges rows with NCCL inside its
CUDA graph; a peer that fails mid-step is caught there (NCCL's asynchronous
error state and a time limit, then the communicator is aborted).  StepGuard
catches a peer that failed *between* steps before any rank launches the next
one: before each step every rank contributes its status to a MIN all-reduce
on a CPU (gloo) process group with a short timeout.  A rank that raised,
reported an error or left makes every other rank's next check raise
PeerFailure; GuardedBatch then aborts its batch's communicator, so no rank
is left with kernels or collectives waiting for a peer that will not come.
"""
import ctypes
import datetime

import numpy as np

from ._lib import check, lib


class PeerFailure(RuntimeError):
    """A rank of the expert-parallel group failed or left."""


def ep_plan(ridx, e_loc, world, cap):
    """The dispatch plan of one MoE layer (cuinf_ep_plan_host): ridx int
    [n] experts of the (token, slot) entries; returns (dest_pos [n],
    meta [world*cap]: local expert index per send position, -1 unused)."""
    r = np.ascontiguousarray(ridx, np.int32).ravel()
    dest = np.empty(r.size, np.int32)
    meta = np.empty(world * cap, np.int32)
    check(lib().cuinf_ep_plan_host(r.ctypes.data_as(ctypes.c_void_p), int(r.size), int(e_loc), int(world), int(cap),
                                   dest.ctypes.data_as(ctypes.c_void_p), meta.ctypes.data_as(ctypes.c_void_p)))
    return dest, meta


class StepGuard:
    """Liveness check of the ranks of one expert-parallel group between
    steps, on its own gloo process group with a short timeout."""

    def __init__(self, timeout_s=10.0, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group or dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=timeout_s))
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()

    def check(self, ok=True):
        """All ranks must call this before each step.  Raises PeerFailure if
        any rank reported ok=False or did not take part within the timeout;
        raises it on this rank too when ok is False."""
        import torch
        t = torch.tensor([1 if ok else 0], dtype=torch.int32)
        try:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN, group=self.group)
        except Exception as e:  # a peer left: its connection closed or the timeout ran out
            raise PeerFailure(f"rank {self.rank}: a peer left the expert-parallel group ({type(e).__name__})") from e
        if not ok:
            raise PeerFailure(f"rank {self.rank} reported a failure to the group")
        if int(t.item()) != 1:
            raise PeerFailure(f"rank {self.rank}: a peer reported a failure")


class GuardedBatch:
    """An expert-parallel Batch (or anything with step/abort) whose steps
    are preceded by a StepGuard check; on any failure the batch is aborted
    and PeerFailure (or the step's own error) propagates."""

    def __init__(self, batch, guard):
        self.batch = batch
        self.guard = guard
        self.failed = False

    def step(self, tokens=None, want=True):
        if self.failed:
            raise PeerFailure("the batch was aborted after an earlier failure")
        try:
            self.guard.check(True)
        except PeerFailure:
            self._abort()
            raise
        try:
            return self.batch.step(tokens, want)
        except Exception:
            self._abort()
            raise

    def leave(self):
        """Stop this rank between steps: the other ranks learn it at their
        next check."""
        try:
            self.guard.check(False)
        except PeerFailure:
            pass
        self._abort()

    def _abort(self):
        self.failed = True
        try:
            self.batch.abort()
        except Exception:
            pass
