"""The roofline numerators bench.py reports, for the config-4 model:
algorithmic bytes of one decode step (every weight read once, the KV cache
of the 6 attention layers, activations) and the linear layers' work per
token (the prefill and batched tensor-pipe fractions)."""
import bench
from cuda_inf_b200 import weights


def test_step_bytes_match_the_per_token_budget():
    # 733,151,232 INT4 + 2,883,584 router + 524,288,000 lm_head + 424,832
    # norms/conv/bias + 25,178,112 KV + 4,096 embedding row at context 4096;
    # step_bytes also counts the activation reads (< 0.02 % more)
    b = bench.step_bytes(weights.default_config(), 4096)
    assert 1_285_929_856 <= b <= 1_285_929_856 * 1.0002, b


def test_linear_flops_per_token():
    c = weights.default_config()
    macs = bench.linear_macs_per_token(c)
    # 6 attention (q,k,v,o) + 18 conv (in 3H, out H) + 2 dense (3 x 7168) +
    # 22 MoE (router + 4 experts x 3 x 1792), all over H = 2048
    H = 2048
    want = 6 * ((32 + 16) * 64 * H + H * 2048) + 18 * 4 * H * H + 2 * 3 * 7168 * H + \
        22 * (32 * H + 4 * 3 * 1792 * H)
    assert macs == want
    assert abs(2 * macs * 4096 / 1e12 - 11.66) < 0.01
