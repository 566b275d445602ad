import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
for _d in (os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")):
    if _d not in sys.path:
        sys.path.insert(0, _d)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def tiny(tmp_path_factory, cuda):
    """(config, CPU oracle model, GPU model) of the TINY test model."""
    import numpy as np
    from enginecheck import TINY, tiny_tensor
    from oracle import pyoracle as orc
    from cuda_inf_b200 import weights
    from cuda_inf_b200.engine import Model
    d = tmp_path_factory.mktemp("tiny")
    cfg = weights.make_config(**TINY)
    weights.write_model(str(d), cfg, tiny_tensor)
    blob = np.fromfile(d / "weights.bin", np.uint8)
    index = open(d / "index.bin", "rb").read()
    om = orc.Model(weights.config_dict(cfg), blob, index)
    gm = Model.load(str(d), cfg)
    return cfg, om, gm
