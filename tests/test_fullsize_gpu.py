"""Parity at the sizes the benchmark workloads run.

* Config 2, the attention core at [64, 16, 257, 64], L = 128: Q@K^T per head
  and Attn@V per row (softmax probabilities unipolar) over all 1024 slices in
  one launch each; slices are independent (per-slice or per-row scales), so
  a seeded sample of slices is recomputed by the oracle from the exact
  operands the engine read.
* One full-width ViT-L/14 block (d = 1024, 16 heads, MLP 4096, 257 tokens) of
  configs 3, 4 and 5, patched as the benchmark patches them: every SC matmul
  the block issues is recorded with its operands and recomputed by the oracle
  (the block composed from oracle calls, on the engine's own inputs).
* The det linears of ``det/experiments/_p8_breakdown.py:70-76`` (M = 6400,
  D = 1408 -> 6144 and 6144 -> 1408, chunk_d 64 and unchunked, p = 6 / 8):
  full launches, with a sample of rows recomputed by the oracle.

Rescaled outputs within the north star's 1e-5 relative (equal bits in
practice); popcount accumulators, where read, bit for bit.
"""
import random
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sc_oracle
from scmp_vit_b200 import _lib
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200 import sc_matmul

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from dropin_cases import oracle_sc_matmul  # noqa: E402

RTOL = 1e-5


def _close(got, want, what):
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=1e-30, err_msg=what)


# --------------------------------------------------------------- config 2

def test_attention_core_config2_full_size(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(64, 16, 257, 64, generator=g).to(dev) for _ in range(3))
    random.seed(0)
    cfg_qk = ch.make_sobol_simple_config(64, 64, 7)
    cfg_av = ch.make_sobol_simple_config(257, 257, 7)
    BH = 64 * 16
    qf, kf = q.reshape(BH, 257, 64), k.reshape(BH, 257, 64)
    acc = torch.empty(BH * 257 * 257, dtype=torch.int32, device=dev)
    s = sc_matmul(qf, kf, granularity="per_head", sc_prec=7, config=cfg_qk, stoc_len=128,
                  acc_out=acc)
    p = (s * 64 ** -0.5).softmax(dim=-1)
    vt = v.reshape(BH, 257, 64).transpose(1, 2).contiguous()
    o = sc_matmul(p, vt, granularity="per_row", mode="unipolar", sc_prec=7, config=cfg_av,
                  stoc_len=128)
    torch.cuda.synchronize()
    assert _lib.engine_status() == 0
    acc = acc.view(BH, 257, 257)
    for sl in np.random.default_rng(0).choice(BH, 12, replace=False).tolist():
        a_ref, y_ref = sc_oracle.sc_matmul_ref(qf[sl].cpu().numpy(), kf[sl].cpu().numpy(),
                                               granularity="per_head", sc_prec=7,
                                               pool=cfg_qk["table"], stoc_len=128)
        np.testing.assert_array_equal(acc[sl].cpu().numpy(), a_ref[0], err_msg=f"QK slice {sl}")
        _close(s[sl].cpu().numpy(), y_ref[0], f"QK slice {sl}")
        _, o_ref = sc_oracle.sc_matmul_ref(p[sl].cpu().numpy(), vt[sl].cpu().numpy(),
                                           mode="unipolar", sc_prec=7, pool=cfg_av["table"],
                                           stoc_len=128)
        _close(o[sl].cpu().numpy(), o_ref[0], f"AV slice {sl}")


# ------------------------------------------------------ full-width blocks

class Recorder:
    """Every engine call of a forward, with copies of its operands and of
    ``out`` before and after (calls may write only some rows of ``out``)."""

    def __init__(self, real):
        self.real = real
        self.calls = []

    def __call__(self, a, b, **kw):
        from scmp_vit_b200.sc import PackedWeight
        out = kw.get("out")
        before = None if out is None else out.detach().clone()
        y = self.real(a, b, **kw)
        src = b.source if isinstance(b, PackedWeight) else b
        kw_c = {k: (v.detach().clone() if torch.is_tensor(v) else v) for k, v in kw.items()
                if k not in ("out", "engine")}
        self.calls.append((a.detach().clone(), src.detach().clone(), kw_c, before,
                           (out if out is not None else y).detach().clone()))
        return y


def _record_block(monkeypatch, cfg_id):
    import bench
    from scmp_vit_b200 import attention
    from scmp_vit_b200 import sc as sc_mod
    from scmp_vit_b200 import sc_linear
    rec = Recorder(sc_mod.sc_matmul)
    for mod in (attention, sc_linear, sc_mod):
        monkeypatch.setattr(mod, "sc_matmul", rec)
    # record the probabilities as the Attn@V operand: the unfused softmax
    # (the fused one gives the same bits: tests/test_softmax_quant_gpu.py)
    monkeypatch.setattr(attention, "FUSED_SOFTMAX", False)
    # one full-width block, patched as the benchmark patches its 24 (config 5:
    # the LFSR-16 pool of block 0 and the head-aligned compensation on it)
    model = bench.build_model(cfg_id, torch.device("cuda", 0), torch.float32, depth=1,
                              comp_blocks=[0])
    x = torch.randn(1, 257, 1024, generator=torch.Generator().manual_seed(cfg_id)).cuda()
    with torch.no_grad():
        model.backbone.blocks[0](x)
    torch.cuda.synchronize()
    assert _lib.engine_status() == 0
    return rec.calls


def _check_calls(calls, label):
    assert calls, f"{label}: no SC calls recorded"
    for i, (a, b, kw, before, after) in enumerate(calls):
        kw = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in kw.items()}
        out = None if before is None else before.cpu()
        y = oracle_sc_matmul(a.cpu(), b.cpu(), out=out, **kw)
        _close(after.cpu().numpy().reshape(-1), y.numpy().reshape(-1),
               f"{label} call {i} ({tuple(a.shape)} x {tuple(b.shape)})")


@pytest.mark.parametrize("cfg_id,min_calls", [(3, 4), (4, 8), (5, 5)])
def test_full_width_block_matches_oracle_composition(cuda_device, monkeypatch, cfg_id, min_calls):
    calls = _record_block(monkeypatch, cfg_id)
    assert len(calls) >= min_calls
    _check_calls(calls, f"config {cfg_id} block")


# --------------------------------------------------------------- det shapes

@pytest.mark.parametrize("D,N", [(1408, 6144), (6144, 1408)])
@pytest.mark.parametrize("p,chunk", [(8, 64), (8, 0), (6, 64)])
def test_det_linear_shapes(cuda_device, D, N, p, chunk):
    dev = cuda_device
    M = 6400
    g = torch.Generator().manual_seed(D + N + p + chunk)
    a = torch.randn(M, D, generator=g) * 0.5
    b = torch.randn(N, D, generator=g) * 0.05
    random.seed(p)
    cfg = ch.make_sobol_simple_config(chunk or D, chunk or D, p)
    y = sc_matmul(a.to(dev), b.to(dev), sc_prec=p, config=cfg, chunk_d=chunk)
    torch.cuda.synchronize()
    assert _lib.engine_status() == 0
    rows = np.sort(np.random.default_rng(p).choice(M, 24, replace=False))
    if chunk:
        _, y_ref = sc_oracle.sc_matmul_segments_ref(a[rows].numpy(), b.numpy(), chunk, sc_prec=p,
                                                    pool=cfg["table"])
    else:
        _, y_ref = sc_oracle.sc_matmul_ref(a[rows].numpy(), b.numpy(), sc_prec=p,
                                           pool=cfg["table"])
    _close(y[torch.from_numpy(rows).to(dev)].cpu().numpy(), y_ref[0], f"rows of {M}x{D}->{N}")
