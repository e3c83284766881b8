"""sl_map-driven patching and QwT compensation on the engine (B200).

A map of single-level entries runs the mixed-precision code path with one
level; it must give exactly the model output of uniform SC patching at the
same stream length.  A compensated block must equal block(x) + comp(x)
with the comp running as a head-aligned SC matmul.
"""
import random

import pytest
import torch

from scmp_vit_b200 import _lib, qwt, sl_map, vit

pytestmark = pytest.mark.gpu


def _model(dev, depth=2):
    return vit.vit_l14(seed=0, dim=128, depth=depth, heads=2, hidden=256, img=56).to(
        dev, torch.bfloat16)


def test_single_level_sl_map_equals_uniform_patching(cuda_device):
    dev = cuda_device
    x = torch.randn(3, 3, 56, 56, generator=torch.Generator().manual_seed(0)).to(
        dev, torch.bfloat16)
    random.seed(0)
    a = _model(dev)
    vit.patch_vit(a, 7, ("qk", "av", "proj"))
    random.seed(0)
    b = _model(dev)
    stats = sl_map.patch_model_with_sl_map(
        b, 7, {"qk": [128, 128], "av": [128, 128], "proj": [128, 128],
               "mlp_fc1": [0, 0], "mlp_fc2": [0, 0]})
    assert stats == {"attn": 2, "qkv_proj": 2, "out_proj": 2}
    with torch.no_grad():
        ya, yb = a(x), b(x)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    torch.testing.assert_close(yb, ya, rtol=0, atol=0)


def test_mixed_sl_map_runs_with_mlp(cuda_device):
    dev = cuda_device
    m = _model(dev)
    sl_map.patch_model_with_sl_map(
        m, 8, {"qk": [[256, 128], 128], "av": [128, [256, 128, 128, 64]],
               "proj": [[256, 192, 128], 0], "mlp_fc1": [0, [256, 128]], "mlp_fc2": [192, 0]})
    with torch.no_grad():
        y = m(torch.randn(2, 3, 56, 56, device=dev, dtype=torch.bfloat16))
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    assert y.shape == (2, 1000) and torch.isfinite(y.float()).all()


def test_head_aligned_compensation_block(cuda_device, tmp_path):
    dev = cuda_device
    m = _model(dev)
    vit.patch_vit(m, 8, ("qk", "av", "proj"))
    g = torch.Generator().manual_seed(3)
    state = {1: {"W": torch.randn(128, 128, generator=g) * 0.01,
                 "b": torch.randn(128, generator=g) * 0.1, "enabled": True}}
    qwt.save_comp_state(str(tmp_path / "c.pt"), state)
    rec = qwt.load_comp_state(str(tmp_path / "c.pt"))
    random.seed(1)
    done = qwt.install_compensation(m, rec, qwt.make_head_aligned_comp_factory(8, n_heads=2))
    assert done == [1]
    cb = m.backbone.blocks[1]
    x = torch.randn(2, 65, 128, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        y = cb(x)
        ref = cb.block(x) + cb.comp(x).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    torch.testing.assert_close(y, ref, rtol=0, atol=0)
