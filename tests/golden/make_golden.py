"""Generate CPU golden fixtures by running the reference's own Python code.

Run here (where the reference tree is mounted), not on the GPU box:

    python tests/golden/make_golden.py [--ref <g023/cuda_inf source tree>]

Writes:
  quant_int4.npz    inputs/outputs of quant_int4_group (tools/export_weights.py:64-79),
                    executed from the reference source, on seeded and edge-case inputs
  format_small.json + index_small.bin
                    the reference exporter (tools/export_weights.py, whole script) and
                    index writer (tools/make_index.py) run on fakegen.SMALL-shaped
                    synthetic tensors: sha256 of weights.bin, index.bin bytes and the
                    tensor list, which this library's writer must reproduce byte for byte.
"""
import argparse
import ast
import hashlib
import json
import os
import runpy
import sys
import tempfile
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import fakegen  # noqa: E402


def load_quantizer(ref):
    """Extract quant_int4_group from the reference exporter and compile it alone
    (the script's module level opens the real checkpoint, so it cannot be imported)."""
    src = open(os.path.join(ref, "tools", "export_weights.py")).read()
    tree = ast.parse(src)
    fn = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "quant_int4_group"][0]
    mod = ast.Module(body=[fn], type_ignores=[])
    ns = {"np": np, "G": 128, "name": "golden"}
    exec(compile(mod, "export_weights.py:quant_int4_group", "exec"), ns)
    return ns["quant_int4_group"]


def quant_cases():
    rng = np.random.default_rng(7)
    cases = {}
    cases["normal"] = (0.02 * rng.standard_normal((16, 256))).astype(np.float32)
    cases["wide"] = (rng.standard_normal((8, 512)) * np.exp(rng.uniform(-6, 2, (8, 1)))).astype(np.float32)
    # exact half-way points: amax 7 -> scale 1, values k + 0.5 round to even
    t = np.zeros((4, 128), np.float32)
    t[:, 0] = 7.0
    halves = np.arange(-6.5, 7.0, 1.0, dtype=np.float32)
    t[:, 1:1 + halves.size] = halves
    t[1] *= -1.0
    t[2, 0] = -7.0
    t[3] = 0.0  # all-zero group: scale 0, nibble 8
    cases["ties"] = t
    tiny = (1e-9 * rng.standard_normal((2, 128))).astype(np.float32)  # fp16 scale underflow
    cases["tiny"] = tiny
    big = (1e6 * rng.standard_normal((2, 128))).astype(np.float32)    # fp16 scale overflow
    cases["big"] = big
    return cases


def make_quant(ref, out):
    q = load_quantizer(ref)
    arrays = {}
    with np.errstate(over="ignore"):
        for k, w in quant_cases().items():
            packed, scales = q(w)
            arrays[k + "_w"] = w
            arrays[k + "_packed"] = packed
            arrays[k + "_scales"] = scales.view(np.uint16)
    np.savez_compressed(os.path.join(out, "quant_int4.npz"), **arrays)
    print("quant_int4.npz:", sorted(arrays))


class _FakeSafeOpen:
    def __init__(self, path, framework="pt"):
        self.path = path

    def keys(self):
        return []

    def get_tensor(self, name):
        import torch
        return torch.from_numpy(fakegen.fake_tensor(name))


def make_format(ref, out):
    with tempfile.TemporaryDirectory() as root:
        os.makedirs(os.path.join(root, "scratch", "LFM2.5-8B-A1B"), exist_ok=True)
        fake = types.ModuleType("safetensors")
        fake.safe_open = _FakeSafeOpen
        saved = sys.modules.get("safetensors")
        sys.modules["safetensors"] = fake
        os.environ["SPINT4_ROOT"] = root
        try:
            runpy.run_path(os.path.join(ref, "tools", "export_weights.py"), run_name="__main__")
            runpy.run_path(os.path.join(ref, "tools", "make_index.py"), run_name="__main__")
        finally:
            if saved is not None:
                sys.modules["safetensors"] = saved
            else:
                del sys.modules["safetensors"]
            del os.environ["SPINT4_ROOT"]
        wdir = os.path.join(root, "scratch", "engine_weights")
        wb = open(os.path.join(wdir, "weights.bin"), "rb").read()
        ib = open(os.path.join(wdir, "index.bin"), "rb").read()
        man = json.load(open(os.path.join(wdir, "manifest.json")))
    meta = {k: v for k, v in man.items() if k != "tensors"}
    info = {
        "config": fakegen.SMALL,
        "weights_bytes": len(wb),
        "weights_sha256": hashlib.sha256(wb).hexdigest(),
        "index_sha256": hashlib.sha256(ib).hexdigest(),
        "n_tensors": len(man["tensors"]),
        "manifest_meta": meta,
        "first_tensors": [[t["name"], t["kind"], t["offset"]] for t in man["tensors"][:8]],
    }
    with open(os.path.join(out, "index_small.bin"), "wb") as f:
        f.write(ib)
    with open(os.path.join(out, "format_small.json"), "w") as f:
        json.dump(info, f, indent=1)
    print("format_small.json:", info["weights_bytes"], "bytes,", info["n_tensors"], "tensors")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import reference_tree
    ap.add_argument("--ref", default=reference_tree(),
                    help="the g023/cuda_inf source tree (default: $CUINF_REFERENCE or ../reference)")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    make_quant(a.ref, a.out)
    make_format(a.ref, a.out)
