"""The Python layers against the reference's own patchers, on the CPU.

The fixtures of ``tests/golden/make_dropin.py`` hold every SC matmul call the
reference's unmodified ``patch_model`` / ``SCLinear`` / ``SCMatMul`` made on
small cases, with the oracle's answers, and their final outputs.  Here the
oracle stands in for the engine (a test-only substitute for ``sc_matmul``)
and this package's modules run the same cases: the routing, mixed-precision
bucketing, pool creation order and FP glue must give the reference's outputs
bit for bit.  ``tests/test_dropin_gpu.py`` runs the same cases on the engine.
"""
import json
import os
import random
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200 import mp_linear

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import dropin_cases  # noqa: E402
from dropin_cases import oracle_sc_matmul  # noqa: E402

META = json.loads((GOLDEN / "dropin.json").read_text())
FIX = np.load(GOLDEN / "dropin.npz")
REF = os.environ.get("SCMP_REFERENCE_DIR")


def _t(name):
    return torch.from_numpy(np.array(FIX[name]))


def _bit_equal(got, want, what):
    got = np.ascontiguousarray(got, dtype=np.float32)
    assert got.shape == want.shape, what
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{what}: max |diff| {np.abs(got - want).max()}"


def test_fixture_calls_replay_on_the_oracle():
    for i, c in enumerate(META["calls"]):
        cfg = ch.config_from_table(np.array(FIX[c["pool"]]), c["sc_prec"])
        y = oracle_sc_matmul(_t(c["a"]), _t(c["b"]), granularity=c["granularity"],
                             mode=c["mode"], sc_prec=c["sc_prec"], config=cfg,
                             group_a=c["group_a"], group_b=c["group_b"], chunk_d=c["chunk_d"],
                             stoc_len=c["stoc_len"])
        _bit_equal(y.numpy(), np.array(FIX[c["out"]]), f"call {i} ({c['case']})")


@pytest.fixture()
def engine_is_oracle(monkeypatch):
    from scmp_vit_b200 import attention, sc_linear
    monkeypatch.setattr(attention, "sc_matmul", oracle_sc_matmul)
    monkeypatch.setattr(sc_linear, "sc_matmul", oracle_sc_matmul)
    monkeypatch.setattr(sc_linear, "USE_NOISE_MODEL", False)


@pytest.mark.parametrize("name", [n for n, *_ in dropin_cases.det_cases()])
def test_det_scmatmul_layer_matches_reference(engine_is_oracle, name):
    from scmp_vit_b200 import attention
    case = META["cases"][name]
    seed, kw = {n: (s, k) for n, s, k, *_ in dropin_cases.det_cases()}[name]
    kw = dict(kw)
    if "op" in kw:
        kw["mp_cfg"] = dropin_cases.det_mp(mp_linear)
    attention._DET_CFG_CACHE.clear()
    random.seed(seed)
    y = attention.SCMatMul(**kw)(_t(case["A"]), _t(case["B"]))
    _bit_equal(y.numpy(), np.array(FIX[case["out"]]), name)


@pytest.mark.parametrize("name", [n for n, *_ in dropin_cases.linear_cases(mp_linear)])
def test_sc_linear_layer_matches_reference(engine_is_oracle, name):
    from scmp_vit_b200 import sc_linear as scl
    case = META["cases"][name]
    seed, kw = {n: (s, k) for n, s, k, *_ in dropin_cases.linear_cases(mp_linear)}[name]
    lin = torch.nn.Linear(case["in"], case["out_features"])
    with torch.no_grad():
        lin.weight.copy_(_t(case["weight"]))
        lin.bias.copy_(_t(case["bias"]))
    scl._CFG_CACHE.clear()
    random.seed(seed)
    with torch.no_grad():
        y = scl.SCLinear(lin, **kw)(_t(case["x"]))
    _bit_equal(y.numpy(), np.array(FIX[case["out"]]), name)


@pytest.mark.parametrize("name", [n for n, *_ in dropin_cases.cls_cases(mp_linear)])
def test_cls_forward_layers_match_reference_patch_model(name):
    """In a child process: the pinned CPU glue needs its environment before
    torch loads."""
    res = subprocess.run([sys.executable, str(GOLDEN / "dropin_forward.py"), name, "oracle"],
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    got = np.array(out["bits"], dtype=np.uint32).view(np.float32).reshape(out["shape"])
    _bit_equal(got, np.array(FIX[META["cases"][name]["logits"]]), f"{name} logits")


@pytest.mark.skipif(not REF, reason="SCMP_REFERENCE_DIR not set (the reference tree)")
def test_reference_regenerates_the_fixture():
    with tempfile.TemporaryDirectory() as tmp:
        res = subprocess.run([sys.executable, str(GOLDEN / "make_dropin.py"), REF, tmp],
                             capture_output=True, text=True, timeout=600)
        assert res.returncode == 0, res.stderr[-3000:]
        meta = json.loads((Path(tmp) / "dropin.json").read_text())
        arrays = np.load(Path(tmp) / "dropin.npz")
        assert meta == META
        assert sorted(arrays.files) == sorted(FIX.files)
        for k in FIX.files:
            assert np.array_equal(arrays[k], FIX[k]), k
