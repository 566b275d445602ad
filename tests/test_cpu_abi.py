"""CPU tests of the C-ABI boundary: the library loads, exports every symbol
include/cuinf.h declares, rejects bad arguments without touching a GPU, and
the product never imports the oracle."""
import ctypes
import os
import re

import pytest

from cuda_inf_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    hdr = open(os.path.join(ROOT, "include", "cuinf.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(cuinf_[a-z0-9_]+)\s*\(", hdr)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = _declared()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_bindings_cover_header():
    assert set(_declared()) <= set(_lib.EXPORTS)


def test_argument_errors_without_gpu():
    L = _lib.lib()
    rc = L.cuinf_gemv_int4(None, None, None, None, 1, 16, 128, None)
    assert rc == 1
    assert b"null pointer" in L.cuinf_last_error()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    rc = L.cuinf_gemv_int4(p, p, p, p, 1, 16, 100, None)
    assert rc == 1 and b"multiple of 128" in L.cuinf_last_error()
    rc = L.cuinf_attn_decode(p, p, p, p, p, p, p, 60, 100, 0.125, p, 32, 8, None, 0, None)
    assert rc == 1 and b"committed" in L.cuinf_last_error()
    rc = L.cuinf_attn_decode(p, p, p, p, p, p, p, 0, 100, 0.125, p, 32, 8, None, 0, None)
    assert rc == 1 and b"tail length" in L.cuinf_last_error()


def test_config_default_matches_reference_defines():
    from cuda_inf_b200 import weights
    c = weights.default_config()
    assert (c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.vocab) == \
        (2048, 24, 32, 8, 64, 128000)
    assert (c.n_dense, c.n_experts, c.top_k, c.moe_inter, c.dense_inter) == (2, 32, 4, 1792, 7168)
    assert [i for i in range(24) if c.attn_layer[i]] == [2, 6, 10, 14, 18, 21]
    assert c.rope_theta == pytest.approx(5e6) and c.norm_eps == pytest.approx(1e-5)


def test_product_does_not_use_oracle():
    pkg = os.path.join(ROOT, "cuda_inf_b200")
    for dp, _, fs in os.walk(pkg):
        for f in fs:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                src = open(os.path.join(dp, f)).read()
                assert "oracle" not in src.replace("oracle/", ""), f
                assert "import oracle" not in src and "liboracle" not in src, f


def test_session_option_constants_match_header():
    """The Python mirror's option numbers are the header's CUINF_OPT_* values."""
    from cuda_inf_b200.engine import Session
    hdr = open(os.path.join(ROOT, "include", "cuinf.h")).read()
    defs = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define CUINF_(OPT_[A-Z_]+)\s+(\d+)", hdr)}
    assert len(defs) >= 8
    for name, value in defs.items():
        assert getattr(Session, name) == value, name
    assert len(set(defs.values())) == len(defs)  # no two options share a number
