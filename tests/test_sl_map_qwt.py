"""sl_map ingestion and QwT block compensation (host side, CPU).

The sl_map rules follow ``cls/experiments/mp_budget_swap_search.py``:
entries are ints or per-row bins, levels longest first with their shares,
non-positive levels dropped and the rest renormalised, JSON bare or under
"sl_map". The compensation follows ``docs/SC_COMP_ALGORITHM.md``: ridge fit
with an unregularised bias, cross-seed cosine gate, ``block(x) + comp(x)``.
Models run on the noise surrogate here (the engine itself needs a GPU).
"""
import importlib
import json
import math
import os
import sys
from pathlib import Path

import pytest
import torch
import torch.nn as nn

from scmp_vit_b200 import qwt, sl_map
from scmp_vit_b200 import sc_linear as scl
from scmp_vit_b200 import vit
from scmp_vit_b200.mp import MPConfig


def test_entry_rules():
    assert sl_map.entry_bins(128) == [128]
    assert sl_map.entry_bins([256, 128, 128, 0]) == [256, 128, 128, 0]
    levels, fracs = sl_map.entry_levels_fractions([128, 256, 128, 64])
    assert levels == [256, 128, 64] and fracs == [0.25, 0.5, 0.25]
    assert sl_map.entry_avg_sl([256, 128]) == 192.0
    assert sl_map.entry_to_mpconfig(0) is None
    assert sl_map.entry_to_mpconfig([0, 0]) is None
    cfg = sl_map.entry_to_mpconfig([256, 0, 128, 128])  # the 0 bin is dropped
    assert cfg.stoc_len_levels == [256, 128]
    assert cfg.level_fractions == pytest.approx([1 / 3, 2 / 3])
    one = sl_map.entry_to_mpconfig(192)
    assert one.stoc_len_levels == [192] and one.level_fractions == [1.0]
    assert sl_map.make_entry(128, 1) == 128 and sl_map.make_entry(64, 3) == [64, 64, 64]


def test_json_round_trip_and_validation(tmp_path):
    m = {op: [128, [256, 128], 0] for op in sl_map.SC_OP_NAMES}
    p = tmp_path / "sl.json"
    sl_map.save_sl_map_json(str(p), m, budget=160)
    assert json.loads(p.read_text())["budget"] == 160
    assert sl_map.load_sl_map_json(str(p)) == m
    bare = tmp_path / "bare.json"
    bare.write_text(json.dumps(m))
    assert sl_map.load_sl_map_json(str(bare)) == m
    bad = dict(m)
    bad["qk"] = [128]
    (tmp_path / "bad.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="block counts"):
        sl_map.load_sl_map_json(str(tmp_path / "bad.json"))
    (tmp_path / "short.json").write_text(json.dumps({"qk": [1]}))
    with pytest.raises(ValueError, match="lacks ops"):
        sl_map.load_sl_map_json(str(tmp_path / "short.json"))


def _tiny(depth=3):
    return vit.vit_l14(seed=0, dim=64, depth=depth, heads=2, hidden=128, img=28)


def test_patch_model_with_sl_map_installs_per_block():
    scl.set_noise_model(True)
    try:
        m = _tiny(3)
        smap = {"qk": [128, 0, [256, 128]], "av": [0, 0, 128], "proj": [0, 192, 0],
                "mlp_fc1": [[256, 128], 0, 0], "mlp_fc2": [0, 0, 0]}
        stats = sl_map.patch_model_with_sl_map(m, 8, smap)
        assert stats == {"attn": 2, "qkv_proj": 1, "out_proj": 1, "mlp_fc1": 1}
        b = m.backbone.blocks
        assert isinstance(b[1].attn.qkv, scl.SCLinear) and isinstance(b[0].attn.qkv, nn.Linear)
        assert isinstance(b[0].mlp.fc1, scl.SCLinear) and isinstance(b[0].mlp.fc2, nn.Linear)
        assert b[1].attn.qkv.mp_cfg.stoc_len_levels == [192]
        with torch.no_grad():
            y = m(torch.randn(2, 3, 28, 28))
        assert y.shape == (2, 1000) and torch.isfinite(y).all()
        with pytest.raises(ValueError, match="entries for 3 blocks"):
            sl_map.patch_model_with_sl_map(_tiny(3), 8, {"qk": [128]})
    finally:
        scl.set_noise_model(False)


def test_ridge_fitter_matches_the_normal_equations():
    torch.manual_seed(0)
    X = torch.randn(300, 12)
    W, b = torch.randn(12, 5), torch.randn(5)
    R = X @ W + b + 0.01 * torch.randn(300, 5)
    f = qwt.RidgeFitter(X, ridge=1e-2)
    W2, b2 = f.fit(R)
    Xa = torch.cat([X, torch.ones(300, 1)], 1).double()
    reg = torch.diag(torch.tensor([1e-2] * 12 + [0.0], dtype=torch.float64))
    sol = torch.linalg.solve(Xa.T @ Xa + reg, Xa.T @ R.double())
    torch.testing.assert_close(W2, sol[:-1].float(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(b2, sol[-1].float(), rtol=1e-5, atol=1e-6)
    assert f.residual_norm_sq(R) == pytest.approx(float(((R.double() - Xa @ sol) ** 2).sum()))
    # the same smoke bound the reference's MP-search test uses
    assert 0.1 * (0.01 ** 2) * 300 * 5 < f.residual_norm_sq(R) < 3.0 * (0.01 ** 2) * 300 * 5


def test_admit_pair_gate():
    W = torch.randn(8, 8)
    ok, cos, Wm, bm = qwt.admit_pair(W, torch.ones(8), W + 0.01 * torch.randn(8, 8),
                                     3 * torch.ones(8))
    assert ok and cos > 0.99
    torch.testing.assert_close(bm, 2 * torch.ones(8))
    ok, cos, _, _ = qwt.admit_pair(W, torch.zeros(8), -W, torch.zeros(8))
    assert not ok and cos == pytest.approx(-1.0)
    ok, _, _, _ = qwt.admit_pair(W, torch.zeros(8), W, torch.zeros(8), eps=1e9)
    assert not ok


def test_compensation_block_and_factories(tmp_path):
    torch.manual_seed(1)
    inner = nn.Linear(16, 16)
    W, b = torch.randn(16, 16) * 0.1, torch.randn(16)
    lin = qwt.make_fp_factory(scale=0.5, polarity=-1)(W, b)
    torch.testing.assert_close(lin.weight, W.t() * -0.5)
    torch.testing.assert_close(lin.bias, -b)
    cb = qwt.CompensationBlock(inner, qwt.make_fp_factory()(W, b))
    x = torch.randn(4, 16)
    torch.testing.assert_close(cb(x), inner(x) + x @ W + b)
    cb.enabled = False
    torch.testing.assert_close(cb(x), inner(x))
    assert isinstance(qwt.make_sc_comp_factory(8)(W, b), scl.SCLinear)
    from scmp_vit_b200.head_aligned_comp import HeadAlignedSCLinear
    assert isinstance(qwt.make_head_aligned_comp_factory(8, n_heads=4)(W, b), HeadAlignedSCLinear)


def test_comp_state_save_load_install(tmp_path):
    m = _tiny(3)
    Ws = {1: torch.randn(64, 64) * 0.01, 2: torch.randn(64, 64) * 0.01}
    state = {i: {"W": W, "b": torch.randn(64), "enabled": i == 1, "cos_ab": 0.8}
             for i, W in Ws.items()}
    p = tmp_path / "comp.pt"
    qwt.save_comp_state(str(p), state, ridge=1e-4, tau=0.5)
    rec = qwt.load_comp_state(str(p))
    assert rec["meta"] == {"ridge": 1e-4, "tau": 0.5}
    x = torch.randn(2, 3, 28, 28)
    with torch.no_grad():
        ref = m(x)
    wrapped = qwt.install_compensation(m, rec, qwt.make_fp_factory())
    assert wrapped == [1]
    blocks = m.backbone.blocks
    assert isinstance(blocks[1], qwt.CompensationBlock) and blocks[1].block is not None
    assert not isinstance(blocks[2], qwt.CompensationBlock)
    with torch.no_grad():
        blocks[1].comp.weight.zero_()
        blocks[1].comp.bias.zero_()
        torch.testing.assert_close(m(x), ref)  # zero correction = the plain model
    torch.save({"format": "other"}, tmp_path / "x.pt")
    with pytest.raises(ValueError, match="not a"):
        qwt.load_comp_state(str(tmp_path / "x.pt"))


# the reference tree: SCMP_REFERENCE_DIR, else an install under baseline/_ref
REF = Path(os.environ.get("SCMP_REFERENCE_DIR",
                          Path(__file__).resolve().parents[1] / "baseline" / "_ref"))


@pytest.mark.skipif(not (REF / "sc_integration" / "mp_search.py").exists(),
                    reason="reference tree not available")
def test_reference_mp_search_imports_and_agrees():
    """The reference's MP-search module imports RidgeFitter through the shim,
    and its entry helpers agree with this package's."""
    from scmp_vit_b200 import shim
    saved = dict(sys.modules)
    sys.path.insert(0, str(REF))
    shim.install()
    try:
        ms = importlib.import_module("sc_integration.mp_search")
        assert ms.RidgeFitter is qwt.RidgeFitter
        for e in (128, [256, 128, 128, 64], [0, 192]):
            assert ms.entry_levels_fractions(e) == sl_map.entry_levels_fractions(e)
            assert ms.entry_avg_sl(e) == sl_map.entry_avg_sl(e)
        assert ms.make_entry(64, 3) == sl_map.make_entry(64, 3)
    finally:
        shim.uninstall()
        for name in list(sys.modules):
            if name not in saved and name.startswith("sc_integration"):
                sys.modules.pop(name, None)
        sys.path.remove(str(REF))
