"""Teacher-forced comparison of a decode Session with the whole-model CPU
oracle, shared by the engine GPU tests.

Each step runs the oracle with the engine's expert choices and asserts the
engine chose the oracle's own top-k set whenever the oracle's k-th vs (k+1)-th
score margin exceeds ROUTE_MARGIN, in the oracle's order up to swaps of
scores within that margin; logits agree within LOGIT_TOL (max-abs
error / max-abs logit) and the argmax agrees outside TIE_MARGIN near-ties.
"""
import zlib

import numpy as np

LOGIT_TOL = 1e-2
TIE_MARGIN = 1e-3
ROUTE_MARGIN = 1e-3


def own_topk(scores, k):
    """The reference's selection on given scores (strict '>', lowest index)."""
    order = sorted(range(len(scores)), key=lambda e: (-scores[e], e))
    return order[:k], (scores[order[k - 1]] - scores[order[k]]) if len(scores) > k else np.inf


def check_routes(gi, sc, k, route_margin, where):
    """gi [n_moe, k] the engine's experts, sc [n_moe, E] the oracle's scores
    on the same inputs; returns (checked, near_ties)."""
    checked = near = 0
    for l in range(gi.shape[0]):
        sel, margin = own_topk(sc[l], k)
        if margin > route_margin:
            # same expert set; each slot holds an expert whose score is
            # within route_margin of the oracle's expert for that slot
            # (the order is descending score, so near-equal scores may swap)
            assert sorted(gi[l].tolist()) == sorted(sel), (where, l, list(gi[l]), sel, margin)
            for j, e in enumerate(gi[l]):
                assert abs(sc[l][e] - sc[l][sel[j]]) <= route_margin, (where, l, j, list(gi[l]), sel)
            checked += 1
        else:
            near += 1
    return checked, near


def check_logits(glog, lg, got, ref, logit_tol, where):
    """Relative max-abs logit error below logit_tol; the engine's token is
    the argmax of its own logits; it equals the oracle's argmax unless the
    oracle's top-2 margin is a near-tie: below TIE_MARGIN of the top logit or
    below twice the observed max-abs logit error (within which the two
    computations may rank the top two either way).  Returns the error."""
    err = float(np.max(np.abs(glog - lg)))
    e = err / float(np.max(np.abs(lg)))
    assert e < logit_tol, (where, e)
    assert glog[got] == np.max(glog), (where, got, int(np.argmax(glog)))
    top = np.sort(lg)[::-1]
    if top[0] - top[1] > max(TIE_MARGIN * max(1.0, abs(top[0])), 2 * err):
        assert got == ref, (where, got, ref)
    return e


def run_compare(cfg, om, s, tokens, max_ctx, logit_tol=LOGIT_TOL, route_margin=ROUTE_MARGIN, st=None):
    """Teacher-forced decode steps; st continues an existing oracle state."""
    st = om.state(max_ctx) if st is None else st
    worst, near_ties, checked = 0.0, 0, 0
    got_tokens = []
    for i, t in enumerate(tokens):
        got = s.step(int(t))
        got_tokens.append(got)
        gi, _ = s.routes()
        gi = np.array(gi, np.int32).reshape(-1, cfg.top_k)
        ref, lg, _, sc = st.forward_ex(int(t), forced_idx=gi.ravel())
        c, n = check_routes(gi, sc, cfg.top_k, route_margin, i)
        checked += c
        near_ties += n
        worst = max(worst, check_logits(s.logits().cpu().numpy(), lg, got, ref, logit_tol, i))
    return worst, near_ties, checked, got_tokens


# A small model that exercises every layer kind (conv, attention with GQA 4,
# dense and MoE FFN), FP8 KV commits, and a vocab not a multiple of 16.
TINY = dict(hidden=256, n_layers=6, n_heads=4, n_kv_heads=1, vocab=1000, n_dense=1, n_experts=8,
            top_k=2, moe_inter=256, dense_inter=384, attn_layers=(1, 4))


def tiny_tensor(name, shape):
    from cuda_inf_b200 import weights
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    k = weights.init_kind(name)
    if k == "norm":
        return (1 + 0.02 * rng.standard_normal(shape)).astype(np.float32)
    if k == "bias":
        return (0.1 * rng.standard_normal(shape)).astype(np.float32)
    if k == "conv":
        return rng.uniform(-0.577, 0.577, shape).astype(np.float32)
    return (0.05 * rng.standard_normal(shape)).astype(np.float32)
