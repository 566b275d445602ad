"""Parity at the context lengths and sizes the benchmark configurations name,
against the whole-model CPU oracle, teacher-forced on the engine's expert
choices (enginecheck.run_compare: routing outside near-ties, logits within
LOGIT_TOL = 1e-2 relative, argmax outside logit near-ties).

  * config 4 (full 24-layer model, batch 1, context 4096) and config 3
    (attention at context 32768, through the engine's fused q/k/v kernel:
    QK-norm, RoPE at position 32767, tail append and the FP8 group commit at
    32768): both the engine and the oracle resume from the same random state
    snapshot (cuinf_session_load_state / orc_state_load) a few tokens before
    the commit, then decode 12 teacher-forced tokens across it;
  * config 5b (prefill of 4,090 tokens, so the grouped expert GEMMs run over
    16 chunks of 256 tokens and the prefill attention over 64 FP8 groups) on
    a 3-layer model of the full width (hidden 2048, 32/8 heads, 32 experts
    top-4 of 1792, dense 7168, vocab 128000), then 10 decode steps across
    the commit at 4096;
  * config 5a (64 sequences at context 2048): a batch whose sequences resume
    from snapshots at positions 2040..2055, 10 steps, 8 of the sequences
    followed by their own oracle state.
"""
import os

import numpy as np
import pytest
import torch

from oracle import pyoracle as orc
from cuda_inf_b200 import weights
from cuda_inf_b200.engine import Batch, Model, Session, device_error
from enginecheck import check_logits, check_routes, run_compare
from oracle.snapshot import random_snapshot

pytestmark = pytest.mark.gpu

ROUTE_MARGIN_FULL = 5e-3  # full width: see test_gpu_engine_full.py


@pytest.fixture(scope="module")
def full(cuda):
    cfg = weights.default_config()
    blob, index = weights.synth_device_blob(cfg, seed=2024, device=cuda)
    host = blob.cpu().numpy()
    orc.set_threads(os.cpu_count() or 1)
    om = orc.Model(weights.config_dict(cfg), host, index)
    gm = Model.from_device_blob(blob, index, cfg)
    yield cfg, om, gm
    gm.close()
    del blob
    torch.cuda.empty_cache()


@pytest.mark.parametrize("start,max_ctx", [(4090, 4200), (32760, 32800)], ids=["ctx4096", "ctx32768"])
def test_full_model_at_long_context(full, start, max_ctx):
    cfg, om, gm = full
    snap = random_snapshot(cfg, start, seed=start)
    s = Session(gm, max_ctx=max_ctx)
    s.keep_logits(True)
    s.load_state(snap)
    assert s.pos == start
    st = om.state(max_ctx)
    st.load_state(snap)
    toks = np.random.default_rng(start + 1).integers(0, cfg.vocab, 12)
    worst, near, checked, _ = run_compare(cfg, om, s, toks, max_ctx, route_margin=ROUTE_MARGIN_FULL, st=st)
    print(f"full model from position {start}: worst logits rel err {worst:.2e}; routing checked {checked}, "
          f"near-ties {near}")
    assert s.pos == start + 12 and st.pos == start + 12
    assert checked > 0.8 * (checked + near)
    assert device_error() == 0
    # the state written across the commit equals a snapshot taken now
    snap2 = s.save_state()
    assert len(snap2) == len(random_snapshot(cfg, start + 12, seed=0))
    s.close()


def test_session_snapshot_round_trip(full):
    """save -> load into a fresh session -> identical logits step for step."""
    cfg, om, gm = full
    a = Session(gm, max_ctx=256)
    a.keep_logits(True)
    toks = np.random.default_rng(8).integers(0, cfg.vocab, 70)
    for t in toks[:60]:
        a.step(int(t))
    snap = a.save_state()
    b = Session(gm, max_ctx=256)
    b.keep_logits(True)
    b.load_state(snap)
    assert b.pos == 60 and b.save_state() == snap
    for t in toks[60:]:
        assert a.step(int(t)) == b.step(int(t))
        assert np.array_equal(a.logits().cpu().numpy(), b.logits().cpu().numpy())
    a.close()
    b.close()


@pytest.fixture(scope="module")
def wide3(cuda):
    """3 layers at the full width: conv + dense FFN, attention + MoE, conv + MoE."""
    cfg = weights.make_config(n_layers=3, n_dense=1, attn_layers=(1,))
    blob, index = weights.synth_device_blob(cfg, seed=77, device=cuda)
    host = blob.cpu().numpy()
    orc.set_threads(os.cpu_count() or 1)
    om = orc.Model(weights.config_dict(cfg), host, index)
    gm = Model.from_device_blob(blob, index, cfg)
    yield cfg, om, gm
    gm.close()
    del blob
    torch.cuda.empty_cache()


def test_prefill_4090_then_decode(wide3):
    cfg, om, gm = wide3
    S = 4090
    rng = np.random.default_rng(4090)
    ids = rng.integers(0, cfg.vocab, S)
    s = Session(gm, max_ctx=4160)
    s.keep_logits(True)
    st = om.state(4160)
    got, gi = s.prefill(ids, routes=True)
    ref, lg, sc = st.prefill(ids, forced_idx=gi)
    checked = near = 0
    for i in range(S):
        c, n = check_routes(gi[i], sc[i], cfg.top_k, ROUTE_MARGIN_FULL, ("prefill row", i))
        checked += c
        near += n
    e = check_logits(s.logits().cpu().numpy(), lg, got, ref, 1e-2, "prefill")
    print(f"prefill {S}: last-row logits rel err {e:.2e}; routing checked {checked}, near-ties {near}")
    assert checked > 0.8 * (checked + near)
    assert s.pos == S and st.pos == S
    tail = rng.integers(0, cfg.vocab, 9)
    worst, near, checked, _ = run_compare(cfg, om, s, [got] + list(tail), 4160, route_margin=ROUTE_MARGIN_FULL,
                                          st=st)
    print(f"decode 4090..4099: worst logits rel err {worst:.2e}")
    assert device_error() == 0
    s.close()


def test_batched_decode_at_context_2048(full):
    cfg, om, gm = full
    B, steps, max_ctx = 64, 10, 2112
    snaps = [random_snapshot(cfg, 2040 + j, seed=500 + j) for j in range(16)]
    bt = Batch(gm, B, max_ctx=max_ctx)
    bt.keep_logits(True)
    for b in range(B):
        bt.load_seq(b, snaps[b % 16])
    assert bt.save_seq(5) == snaps[5]
    follow = list(range(0, B, 9))  # 8 sequences: 0, 9, ..., 63
    states = {}
    for b in follow:
        states[b] = om.state(max_ctx)
        states[b].load_state(snaps[b % 16])
    toks = np.random.default_rng(2048).integers(0, cfg.vocab, (steps, B))
    worst, checked, near = 0.0, 0, 0
    for i in range(steps):
        got = bt.step(toks[i])
        routes = bt.routes()
        glog = bt.logits().cpu().numpy()
        for b in follow:
            gi = routes[:, b, :]
            ref, lg, _, sc = states[b].forward_ex(int(toks[i, b]), forced_idx=gi.ravel())
            c, n = check_routes(gi, sc, cfg.top_k, ROUTE_MARGIN_FULL, (i, b))
            checked += c
            near += n
            worst = max(worst, check_logits(glog[b], lg, got[b], ref, 1e-2, (i, b)))
    print(f"batched B={B} at 2040..2064: worst logits rel err {worst:.2e}; routing checked {checked}, "
          f"near-ties {near}")
    assert checked > 0.8 * (checked + near)
    assert Batch.error() == 0
    bt.close()
