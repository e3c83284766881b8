"""The reference's own Python modules import and route to this engine (CPU).

Runs only where the reference tree is available (SCMP_REFERENCE_DIR); it
checks the drop-in at the ``scmp_kernels`` import boundary: the reference's
unmodified ``sc_integration`` and ``cls/sc_attention_patch.py`` import, build
their modules, patch a DINOv2-style model, and send SC matmuls to
``scmp_vit_b200.sc.sc_matmul`` (which refuses CPU tensors: no CPU path).
"""
import importlib
import os
import sys
from pathlib import Path

import pytest
import torch
import torch.nn as nn

# the reference tree: SCMP_REFERENCE_DIR, else an install under baseline/_ref
REF = Path(os.environ.get("SCMP_REFERENCE_DIR",
                          Path(__file__).resolve().parents[1] / "baseline" / "_ref"))
pytestmark = pytest.mark.skipif(not (REF / "sc_integration" / "sc_linear.py").exists(),
                                reason="reference tree not available")


@pytest.fixture()
def ref_modules():
    from scmp_vit_b200 import shim
    saved = dict(sys.modules)
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(REF / "cls"))
    shim.install()
    try:
        yield
    finally:
        shim.uninstall()
        for name in list(sys.modules):
            if name not in saved and (name.startswith("sc_integration") or
                                      name.startswith("sc_attention_patch")):
                sys.modules.pop(name, None)
        sys.path.remove(str(REF))
        sys.path.remove(str(REF / "cls"))


def test_reference_sc_linear_imports_and_routes_to_engine(ref_modules):
    scl = importlib.import_module("sc_integration.sc_linear")
    assert scl.__file__.startswith(str(REF))
    from scmp_vit_b200.sc import sc_matmul
    assert scl.sc_matmul is sc_matmul
    lin = nn.Linear(16, 8)
    m = scl.SCLinear(lin, sc_prec=7)
    with pytest.raises(RuntimeError, match="no CPU path"):
        m(torch.randn(3, 16))
    cfg = scl._get_config(16, 7)
    assert cfg["dims"] == 16 and cfg["sc_prec"] == 7 and (16, 7) in scl._CFG_CACHE


def test_reference_mp_linear_range_dispatch(ref_modules):
    mpl = importlib.import_module("sc_integration.mp_linear")
    w = torch.randn(64, 16)
    entries = mpl.build_range_dispatch(w, mpl.RangeMPConfig([256, 128], base_threshold=0.5),
                                       group_size=16)
    assert sum(e.weight.shape[0] for e in entries) == 64
    a = mpl.classify_input_rows(torch.randn(40, 16), mpl.MPConfig([256, 128], [0.25, 0.75]))
    assert {k: v.numel() for k, v in a.level_row_indices.items()} == {256: 10, 128: 30}


def test_reference_cls_patch_model(ref_modules):
    patch = importlib.import_module("sc_attention_patch")
    from scmp_vit_b200 import vit
    model = vit.vit_l14(seed=0, dim=64, depth=2, heads=2, hidden=128, img=28)
    stats = patch.patch_model(model, sc_prec=7, sc_qk=True, sc_av=True, sc_qkv_proj=True,
                              sc_out_proj=True, sc_mlp=True)
    assert stats == {"attn": 2, "mlp_fc1": 2, "mlp_fc2": 2, "qkv_proj": 2, "out_proj": 2}
    with pytest.raises(RuntimeError, match="no CPU path"):
        with torch.no_grad():
            model(torch.randn(1, 3, 28, 28))
