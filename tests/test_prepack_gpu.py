"""Prepacked weights (scmp_prepack_b / sc.prepack_b) on the engine (B200).

A prepacked b must give exactly what the weight itself gives: the same
popcount sums and the same outputs, on the CTA-pair kernels that load the
packed bytes with TMA (int8 bytes, or e2m1 nibbles for p = 7 / 8; including
b tiles past the last weight row), on the
single-CTA and CUDA-core paths that read the packed codes, and through
SCLinear's cache (rebuilt when the weight changes in place).
"""
import random

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import sc_oracle
from scmp_vit_b200 import _lib
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200 import sc_linear as scl
from scmp_vit_b200.sc import prepack_b, sc_matmul

pytestmark = pytest.mark.gpu


def _same(dev, a, w, p, L=None, mode="bipolar", granularity="per_row", bias=None):
    random.seed(p + a.shape[0])
    K = a.shape[-1]
    cfg = ch.make_sobol_simple_config(K, K, p)
    M, N = a.shape[-2], w.shape[0]
    BH = a.shape[0] if a.dim() == 3 else 1
    acc1 = torch.empty(BH * M * N, dtype=torch.int32, device=dev)
    acc2 = torch.empty_like(acc1)
    kw = dict(granularity=granularity, mode=mode, sc_prec=p, config=cfg, stoc_len=L, bias=bias)
    y1 = sc_matmul(a, w, acc_out=acc1, **kw)
    pk = prepack_b(w, granularity=granularity, mode=mode, sc_prec=p, config=cfg)
    y2 = sc_matmul(a, pk, acc_out=acc2, **kw)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    assert torch.equal(acc1, acc2)
    assert torch.equal(y1, y2)
    return cfg, acc2, y2


@pytest.mark.parametrize("M,N,K,p,L", [
    (600, 384, 256, 7, None),    # CTA pairs + TMA b, odd CTA of the last pair part-filled
    (513, 300, 64, 7, None),     # b tile past the last row (zero-filled box) + 1-row strip
    (1024, 256, 40, 8, None),    # Lp = 256, K padded to 40
    (700, 260, 72, 6, None),     # Lp = 64
    (600, 384, 256, 7, 64),      # shorter stream: Lp 64 != 2^p, codes path
    (200, 384, 128, 7, None),    # one a tile: single-CTA kernel on the packed codes
    # e2m1 packed bytes (p = 7 / 8, N > 128) by TMA at the tile widths the
    # pair kernel picks: 208 b rows (104-row boxes), 240 (120-row boxes)
    (600, 1024, 64, 7, None),
    (520, 3072, 32, 7, None),
    (700, 520, 48, 8, 256),
    (600, 1024, 64, 8, 192),     # TMA b, three of the four MMA steps per stage
])
def test_prepacked_equals_weight(cuda_device, M, N, K, p, L):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(cuda_device)
    w = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device)
    _same(cuda_device, a, w, p, L)


def test_prepacked_matches_oracle_and_bias(cuda_device):
    g = torch.Generator().manual_seed(9)
    a = torch.randn(520, 96, generator=g)
    w = torch.randn(300, 96, generator=g) * 0.05
    bias = torch.randn(300, generator=g)
    cfg, acc, y = _same(cuda_device, a.to(cuda_device), w.to(cuda_device), 7,
                        bias=bias.to(cuda_device))
    acc_ref, y_ref = sc_oracle.sc_matmul_ref(a.numpy(), w.numpy(), granularity="per_row",
                                             mode="bipolar", sc_prec=7, pool=cfg["table"],
                                             stoc_len=128, bias=bias.numpy())
    np.testing.assert_array_equal(acc.view(1, 520, 300).cpu().numpy(), acc_ref)
    np.testing.assert_allclose(y.view(1, 520, 300).cpu().numpy(), y_ref, rtol=1e-5, atol=1e-30)


def test_prepacked_unipolar_bf16_and_batched_a(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(4)
    a = torch.rand(2, 400, 128, generator=g).to(dev, torch.bfloat16)
    w = torch.randn(320, 128, generator=g).to(dev, torch.bfloat16)
    _same(dev, a, w, 7, mode="unipolar")
    _same(dev, a, w, 7, granularity="per_tensor")


def test_sclinear_cache_follows_the_weight(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(5)
    lin = nn.Linear(256, 384).to(dev)
    x = torch.randn(600, 256, generator=g).to(dev)
    random.seed(0)
    m = scl.SCLinear(lin, 7)
    try:
        scl.set_weight_prepack(False)
        y_plain = m(x)
        scl.set_weight_prepack(True)
        y_packed = m(x)
        assert m._packed is not None
        torch.testing.assert_close(y_packed, y_plain, rtol=0, atol=0)
        with torch.no_grad():
            lin.weight.mul_(-0.5)  # in place: bumps the version counter
        y2 = m(x)
        scl.set_weight_prepack(False)
        torch.testing.assert_close(y2, m(x), rtol=0, atol=0)
    finally:
        scl.set_weight_prepack(None)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0


@pytest.mark.parametrize("M,N,K,kseg,p,L", [
    (600, 1024, 1024, 64, 8, None),   # the head-aligned compensation shape
    (300, 250, 256, 32, 7, None),     # ragged b tile, Lp = 128
    (257, 176, 512, 64, 8, 160),      # L < 2^p: b generated from the packed codes
])
def test_segmented_prepack_matches_weight_and_oracle(cuda_device, M, N, K, kseg, p, L):
    """A weight packed for segmented calls (per-segment quantisation, pool rows
    per index inside the segment) gives the weight's own results bit for bit,
    and the oracle's segment sums."""
    dev = cuda_device
    g = torch.Generator().manual_seed(M + N)
    a = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.02
    bias = torch.randn(N, generator=g)
    cfg = ch.make_lfsr_config(kseg, kseg, p, seed=N)
    kw = dict(sc_prec=p, config=cfg, stoc_len=L, k_segment=kseg, bias=bias.to(dev))
    y1 = sc_matmul(a.to(dev), w.to(dev), **kw)
    pk = prepack_b(w.to(dev), sc_prec=p, config=cfg, k_segment=kseg)
    y2 = sc_matmul(a.to(dev), pk, **kw)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    assert torch.equal(y1, y2)
    _, y_ref = sc_oracle.sc_matmul_segments_ref(a.numpy(), w.numpy(), kseg, sc_prec=p,
                                                pool=cfg["table"], stoc_len=L, bias=bias.numpy())
    np.testing.assert_allclose(y2.cpu().numpy(), y_ref[0], rtol=1e-5, atol=1e-30)
    with pytest.raises(ValueError, match="k_segment"):
        sc_matmul(a.to(dev), pk, sc_prec=p, config=cfg, stoc_len=L)


def test_head_aligned_keeps_its_packed_weight(cuda_device):
    """With prepacking forced on, HeadAlignedSCLinear packs its weight once per
    weight version; results equal the generated path bit for bit."""
    from scmp_vit_b200.head_aligned_comp import HeadAlignedSCLinear
    dev = cuda_device
    lin = nn.Linear(256, 96).to(dev)
    cfg = ch.make_lfsr_config(64, 64, 8, seed=3)
    m = HeadAlignedSCLinear(lin, 8, n_heads=4, cfg_override=cfg)
    x = torch.randn(700, 256, generator=torch.Generator().manual_seed(2)).to(dev)
    y0 = m(x)  # default: b generated in the kernel
    assert getattr(m, "_packed", None) is None
    scl.set_weight_prepack(True)
    try:
        y1 = m(x)
        assert m._packed is not None and m._packed.k_segment == 64
        packed = m._packed
        y2 = m(x)
        assert m._packed is packed  # cached
        with torch.no_grad():
            lin.weight.mul_(0.5)  # in place: the cache notices the new version
        y3 = m(x)
        assert m._packed is not packed
    finally:
        scl.set_weight_prepack(None)
    y4 = m(x)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1) and torch.equal(y1, y2) and torch.equal(y3, y4)


def test_mixed_precision_linears_use_packed_weights(cuda_device):
    """Mixed-precision linears run one call per precision class; each loads
    the weight prepacked for its precision (SCLinear with an MP config, and
    the benchmark's seeded-random MP linear), bit-identical to generating b."""
    from scmp_vit_b200.mp import MPConfig, SeededRandomMPConfig
    from scmp_vit_b200.vit import _RowMPLinear
    dev = cuda_device
    g = torch.Generator().manual_seed(11)
    lin = nn.Linear(256, 300).to(dev)
    x = torch.randn(2, 257, 256, generator=g).to(dev)
    scl._CFG_CACHE.clear()
    random.seed(4)
    m = scl.SCLinear(lin, 8, mp_cfg=MPConfig([128, 192, 256]), operator="mlp_fc1")
    r = _RowMPLinear(lin, SeededRandomMPConfig([128, 192, 256], None, seed=0), 5, scl._get_config)
    ys = []
    for prepack in (None, False):
        scl.set_weight_prepack(prepack)
        try:
            r.calls = 0
            ys.append((m(x), r(x)))
        finally:
            scl.set_weight_prepack(None)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    assert len(m._packed_levels._cache) == 2 and len(r.packed._cache) == 2  # p = 7 and 8
    assert torch.equal(ys[0][0], ys[1][0]) and torch.equal(ys[0][1], ys[1][1])
