"""H2O eviction mode (the reference's --kv-budget, engine.cu:310-384,
803-828) against the CPU oracle's restatement, teacher-forced on the small
model with a budget of 40 slots and a window of 20, so eviction starts at
token 40 and runs for 100 more steps.

Each step the oracle runs on the engine's experts and on the engine's slot
choices (forced), and records its own choice.  The engine's cumulative
attention must follow the oracle's within ATTN_TOL (relative to the largest
mass; these are running sums of probabilities, so fp16-level differences in
q and k accumulate).  Where the two slot choices differ, the oracle's masses
of the two slots must be a near-tie: closer than twice the engine-oracle mass
difference seen at the previous step.  Logits within 1e-2 relative."""
import numpy as np
import pytest

from cuda_inf_b200.engine import Session, device_error
from enginecheck import check_logits, check_routes

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-2


def test_h2o_decode_matches_oracle(tiny):
    cfg, om, gm = tiny
    budget, window = 40, 20
    s = Session(gm, max_ctx=200)
    s.set_kv_budget(budget, window)
    s.keep_logits(True)
    st = om.state(200)
    st.set_h2o(budget, window)
    attn_layers = [l for l in range(cfg.n_layers) if l in (1, 4)]
    toks = np.random.default_rng(77).integers(0, cfg.vocab, 140)
    differ = checked_slots = 0
    worst = 0.0
    mass_err = {l: 0.0 for l in attn_layers}
    for i, t in enumerate(toks):
        got = s.step(int(t))
        gi, _ = s.routes()
        gi = np.array(gi, np.int32).reshape(-1, cfg.top_k)
        eng_slots = np.full(cfg.n_layers, -1, np.int32)
        for l in attn_layers:
            eng_slots[l] = s.h2o_state(l)[3]
        # the oracle's own choice comes from its state before this token
        pre = {l: st.h2o_layer(l)[0] for l in attn_layers}
        st.force_h2o_slots(eng_slots)
        ref, lg, _, sc = st.forward_ex(int(t), forced_idx=gi.ravel())
        own, used = st.h2o_slots()
        for l in attn_layers:
            assert used[l] == eng_slots[l]
            if own[l] != eng_slots[l]:  # only an eviction near-tie may differ
                differ += 1
                a = pre[l]
                assert i >= budget, (i, l, own[l], eng_slots[l])
                assert abs(float(a[own[l]]) - float(a[eng_slots[l]])) <= 2 * mass_err[l] + 1e-6, \
                    (i, l, own[l], eng_slots[l], a[own[l]], a[eng_slots[l]], mass_err[l])
            checked_slots += 1
        for l in attn_layers:
            sp_e, a_e, n_e, _ = s.h2o_state(l)
            a_o, sp_o, n_o = st.h2o_layer(l)
            assert n_e == n_o == min(i + 1, budget)
            assert np.array_equal(sp_e[:n_e], sp_o[:n_o]), (i, l)
            mass_err[l] = float(np.max(np.abs(a_e[:n_e] - a_o[:n_o])))
            rel = mass_err[l] / max(1.0, float(np.max(np.abs(a_o[:n_o]))))
            assert rel < ATTN_TOL, (i, l, rel)
        check_routes(gi, sc, cfg.top_k, 1e-3, i)
        worst = max(worst, check_logits(s.logits().cpu().numpy(), lg, got, ref, 1e-2, i))
    print(f"H2O: worst logits rel err {worst:.2e}; slot choices differing at near-ties {differ}/{checked_slots}")
    assert differ <= 0.05 * checked_slots
    assert device_error() == 0
    s.close()


def test_h2o_prefill_then_decode(tiny):
    """A prompt prefilled into the slots (no eviction inside it), then decode
    steps that evict, against the oracle's prefill and decode."""
    cfg, om, gm = tiny
    budget, window = 48, 16
    s = Session(gm, max_ctx=160)
    s.set_kv_budget(budget, window)
    s.keep_logits(True)
    st = om.state(160)
    st.set_h2o(budget, window)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, cfg.vocab, 40)
    got, routes = s.prefill(prompt, routes=True)
    ref, lg, _ = st.prefill(prompt, forced_idx=routes)
    check_logits(s.logits().cpu().numpy(), lg, got, ref, 1e-2, "prefill")
    for l in (1, 4):
        sp_e, a_e, n_e, _ = s.h2o_state(l)
        a_o, sp_o, n_o = st.h2o_layer(l)
        assert n_e == n_o == 40 and np.array_equal(sp_e[:40], sp_o[:40])
        assert float(np.max(np.abs(a_e[:40] - a_o[:40]))) < ATTN_TOL * max(1.0, float(np.max(a_o)))
    feed = [got] + list(rng.integers(0, cfg.vocab, 30))
    for i, t in enumerate(feed):
        g = s.step(int(t))
        gi, _ = s.routes()
        gi = np.array(gi, np.int32).reshape(-1, cfg.top_k)
        slots = np.full(cfg.n_layers, -1, np.int32)
        for l in (1, 4):
            slots[l] = s.h2o_state(l)[3]
        st.force_h2o_slots(slots)
        r, lg, _, _ = st.forward_ex(int(t), forced_idx=gi.ravel())
        check_logits(s.logits().cpu().numpy(), lg, g, r, 1e-2, ("decode", i))
    s.close()
