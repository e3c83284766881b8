"""The reference's own patchers against this engine, through their fixtures.

``tests/golden/make_dropin.py`` ran the reference's unmodified
``cls/sc_attention_patch.py`` (``patch_model`` and its attention forward),
``sc_integration/sc_linear.py`` (``SCLinear``: chunked, range x row MP) and
``det/sc_patch/sc_matmul.py`` (``SCMatMul``: uniform, stoc_len, per-head and
per-row MP) on the CPU, each SC matmul answered by the oracle, and recorded
every call.  Here, on the GPU:

1. every recorded call runs through ``sc_matmul`` (the function the shim
   serves as ``scmp_kernels.sc.sc_matmul``) with the same operands, keyword
   arguments and pool, and matches the oracle's answer;
2. this package's ``SCMatMul`` and ``SCLinear`` run the det and linear cases
   from the same inputs and random state and match the reference's outputs;
3. this package's modules, installed where ``patch_model`` installs the
   reference's, run the cls forwards (CPU glue pinned as in the fixture run,
   every SC matmul on the engine) and give the reference's logits.

Tolerance: the north star's 1e-5 relative for rescaled outputs; the engine
reproduces the oracle's fp32 sequence, so the results are in practice equal
bit for bit, which the tests also count.
"""
import json
import os
import random
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from scmp_vit_b200 import _lib
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200 import mp_linear, sc_matmul

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import dropin_cases  # noqa: E402

RTOL = 1e-5
META = json.loads((GOLDEN / "dropin.json").read_text())
FIX = np.load(GOLDEN / "dropin.npz")


def _t(name):
    return torch.from_numpy(np.array(FIX[name]))


def _check(got: np.ndarray, want: np.ndarray, what: str):
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=1e-30, err_msg=what)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"{what}: not bit-equal"


@pytest.fixture(autouse=True)
def _no_noise_surrogate(monkeypatch):
    from scmp_vit_b200 import sc_linear
    monkeypatch.setattr(sc_linear, "USE_NOISE_MODEL", False)


@pytest.mark.parametrize("i", range(len(META["calls"])))
def test_recorded_reference_call_on_the_engine(cuda_device, i):
    c = META["calls"][i]
    dev = cuda_device
    pool = np.array(FIX[c["pool"]])
    cfg = ch.config_from_table(pool, c["sc_prec"])
    y = sc_matmul(_t(c["a"]).to(dev), _t(c["b"]).to(dev), granularity=c["granularity"],
                  mode=c["mode"], sc_prec=c["sc_prec"], config=cfg, group_a=c["group_a"],
                  group_b=c["group_b"], chunk_d=c["chunk_d"], stoc_len=c["stoc_len"])
    torch.cuda.synchronize()
    assert _lib.engine_status() == 0
    _check(y.cpu().numpy(), np.array(FIX[c["out"]]), f"call {i} of {c['case']}")


@pytest.mark.parametrize("name", [n for n, *_ in dropin_cases.det_cases()])
def test_det_scmatmul_matches_reference(cuda_device, name):
    from scmp_vit_b200 import attention
    case = META["cases"][name]
    spec = {n: (seed, kw) for n, seed, kw, *_ in dropin_cases.det_cases()}
    seed, kw = spec[name]
    kw = dict(kw)
    if "op" in kw:
        kw["mp_cfg"] = dropin_cases.det_mp(mp_linear)
    attention._DET_CFG_CACHE.clear()
    random.seed(seed)
    y = attention.SCMatMul(**kw)(_t(case["A"]).to(cuda_device), _t(case["B"]).to(cuda_device))
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), np.array(FIX[case["out"]]), name)


@pytest.mark.parametrize("name", [n for n, *_ in dropin_cases.linear_cases(mp_linear)])
def test_sc_linear_matches_reference(cuda_device, name):
    from scmp_vit_b200 import sc_linear as scl
    case = META["cases"][name]
    spec = {n: (seed, kw) for n, seed, kw, *_ in dropin_cases.linear_cases(mp_linear)}
    seed, kw = spec[name]
    dev = cuda_device
    lin = torch.nn.Linear(case["in"], case["out_features"]).to(dev)
    with torch.no_grad():
        lin.weight.copy_(_t(case["weight"]))
        lin.bias.copy_(_t(case["bias"]))
    scl._CFG_CACHE.clear()
    random.seed(seed)
    with torch.no_grad():
        y = scl.SCLinear(lin, **kw)(_t(case["x"]).to(dev))
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), np.array(FIX[case["out"]]), name)


@pytest.mark.parametrize("name", [n for n, *_ in dropin_cases.cls_cases(mp_linear)])
def test_cls_forward_matches_reference_patch_model(name):
    """Whole forwards in a child process (the pinned CPU glue needs its
    environment before torch loads)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    env = dict(os.environ)
    res = subprocess.run([sys.executable, str(GOLDEN / "dropin_forward.py"), name],
                         capture_output=True, text=True, env=env, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    got = np.array(out["bits"], dtype=np.uint32).view(np.float32).reshape(out["shape"])
    want = np.array(FIX[META["cases"][name]["logits"]])
    _check(got, want, f"{name} logits")
