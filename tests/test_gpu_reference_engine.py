"""Greedy tokens against the reference engine itself (src/engine.cu of
g023/cuda_inf, built unmodified for sm_100a by oracle/Makefile into
oracle/_ref/ref_engine), on the same random-init full-size weights.

Both engines consume the prompt with a batched prefill (layer_forward with
S = prompt length, engine.cu:784-917): every attention layer first places all
the prompt's keys/values, FP8-committing each full 64-token group, then every
prompt query attends over them (attention_fused, 236-308); this engine's
cuinf_prefill does the same.  Prompts of 1 and 64 tokens are run; the
64-token prompt commits its group inside the prefill, so its queries read
their own group's keys as FP8.  Then 80 tokens are generated, crossing the
next commit.

Two models are run.  On the plain random-init model (expert bias
N(0, 0.1)) routing near-ties occur at most positions, so the comparison
walks the trajectories up to their first parting and requires it to sit on
a near-tie.  On the same model with a spaced router bias (each MoE layer's
expert bias set to 1.0 x a random permutation of 0..31, so the 4th vs 5th
expert score margin is at least 1.0 - 0.7: sigmoid values of these logits
stay inside (0.15, 0.85)) no routing decision is near a tie, and the greedy
tokens must be identical to the reference engine's for the first
MIN_PREFIX tokens.

The CPU oracle, teacher-forced along the reference's tokens, gives at every
position the top-2 logit margin and the margin between the 4th and 5th
expert scores of each MoE layer (of every prompt row for the prefill).  Two
faithful implementations differ by fp16 ulps in the residual stream, which
moves router scores by up to ~1.5e-3; a flipped expert then changes the
logits by far more than any rounding, so the two greedy trajectories can
part at such a routing near-tie.  The test walks the reference's tokens:
this engine's tokens must equal them up to the first difference, that
difference must sit on a near-tie (logit margin below TIE_MARGIN of the top
logit, or a routing margin below ROUTE_MARGIN in some layer), and at every
clear position the reference's token must be the oracle's argmax.  The
matched prefix is printed.
"""
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest
import torch

from oracle import pyoracle as orc
from cuda_inf_b200 import weights
from cuda_inf_b200.engine import Model, Session

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "ref_engine")
N_NEW = 80
MIN_PREFIX = 32
TIE_MARGIN = 1e-2  # relative top-2 logit margin below which a greedy pick is a near-tie
ROUTE_MARGIN = 2e-3  # 4th-vs-5th expert score margin below which routing is a near-tie


def space_router_bias(blob, cfg, seed):
    """Overwrite every MoE layer's expert bias in the device blob with
    1.0 x a random permutation of 0..E-1 (fp16, exact)."""
    rng = np.random.default_rng(seed)
    for e in weights.layout(cfg):
        if e.name.endswith("feed_forward.expert_bias"):
            b = rng.permutation(cfg.n_experts).astype(np.float16)
            blob[e.offset:e.offset + e.nbytes].copy_(torch.from_numpy(b.view(np.uint8)).to(blob.device))


@pytest.mark.skipif(not os.path.exists(REF_ENGINE), reason="reference engine not built (oracle/_ref)")
@pytest.mark.parametrize("spaced", [False, True], ids=["plain", "spaced_bias"])
@pytest.mark.parametrize("n_prompt", [1, 64])
def test_greedy_matches_reference_engine(cuda, n_prompt, spaced):
    cfg = weights.default_config()
    blob, index = weights.synth_device_blob(cfg, seed=97, device=cuda)
    if spaced:
        space_router_bias(blob, cfg, seed=11)
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, cfg.vocab, n_prompt)]
    base = "/dev/shm" if shutil.disk_usage("/dev/shm").free > 6e9 else None
    with tempfile.TemporaryDirectory(dir=base) as d:
        weights.save_blob(blob, index, d)
        np.array(prompt, np.int32).tofile(os.path.join(d, "ids.i32"))
        os.makedirs(os.path.join(d, "scratch"), exist_ok=True)
        r = subprocess.run([REF_ENGINE, "--dir", d, "--ids", os.path.join(d, "ids.i32"), "--n", str(N_NEW),
                            "--no-stream"], cwd=d, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-500:]
        ref = np.fromfile(os.path.join(d, "scratch", "engine_out_ids.i32"), np.int32).tolist()
        host = np.fromfile(os.path.join(d, "weights.bin"), np.uint8)
    assert 1 <= len(ref) <= N_NEW

    gm = Model.from_device_blob(blob, index, cfg)
    s = Session(gm, max_ctx=n_prompt + N_NEW + 8)
    ours = s.generate(prompt, len(ref))  # prompt through cuinf_prefill
    s.close()
    gm.close()
    del blob
    torch.cuda.empty_cache()

    orc.set_threads(os.cpu_count() or 1)
    om = orc.Model(weights.config_dict(cfg), host, index)
    st = om.state(n_prompt + N_NEW + 8)
    matched = 0
    min_route_margin = np.inf
    for i, tok in enumerate(ref):
        if i == 0:
            nxt, lg, sc = st.prefill(prompt)  # sc [S, n_moe, E]
        else:
            nxt, lg, _, sc = st.forward_ex(ref[i - 1])
        top = np.sort(lg)[::-1]
        srt = -np.sort(-sc, axis=-1)
        route_margin = float(np.min(srt[..., cfg.top_k - 1] - srt[..., cfg.top_k]))
        min_route_margin = min(min_route_margin, route_margin)
        logit_tie = top[0] - top[1] <= TIE_MARGIN * max(1.0, abs(float(top[0])))
        near_tie = logit_tie or route_margin <= ROUTE_MARGIN
        if ours[i] != tok:
            assert near_tie, (i, float(top[0] - top[1]), route_margin, ours[: i + 1], ref[: i + 1])
            break
        if not near_tie:
            assert tok == nxt, (i, tok, nxt)
        matched += 1
    print(f"prompt {n_prompt} ({'spaced' if spaced else 'plain'} bias): greedy tokens equal to the reference "
          f"engine's: first {matched} of {len(ref)}; ours {ours[:matched + 1]}, reference {ref[:matched + 1]}")
    if spaced:
        assert min_route_margin > 0.1
        assert matched >= min(MIN_PREFIX, len(ref))
    elif n_prompt == 1:
        assert matched >= 1
