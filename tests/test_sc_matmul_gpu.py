"""GPU parity of ``sc_matmul`` against the CPU oracle.

Popcount accumulators must match bit for bit; rescaled outputs within 1e-5
relative (the engine reproduces the oracle's fp32 sequence, so they are in
practice identical).
"""
import random

import numpy as np
import pytest
import torch

from oracle import sc_oracle
from scmp_vit_b200 import _lib
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200 import sc_matmul
from scmp_vit_b200._lib import EngineError

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _cfg(kind, D, p, seed=0):
    random.seed(seed)
    if kind == "sobol":
        return ch.make_sobol_simple_config(D, D, p)
    if kind == "anti":
        return ch.make_sobol_antithetic_config(D, D, p)
    if kind == "alt":
        return ch.make_sobol_altseed_config(D, D, p, [1, 3, 5, 11, 17, 33, 65, 129][:p])
    return ch.make_lfsr_config(D, D, p, seed=seed)


def _run(dev, a, b, cfg, *, engine="auto", pool_dims=None, **kw):
    BH = a.shape[0] if a.dim() == 3 else 1
    M, N = a.shape[-2], b.shape[-2]
    acc = torch.empty(BH * M * N, dtype=torch.int32, device=dev)
    bias = kw.pop("bias", None)
    y = sc_matmul(a.to(dev), b.to(dev), config=cfg, acc_out=acc, engine=engine,
                  bias=None if bias is None else bias.to(dev), **kw)
    torch.cuda.synchronize()
    acc_ref, y_ref = sc_oracle.sc_matmul_ref(
        a.numpy(), b.numpy(), granularity=kw.get("granularity", "per_row"),
        mode=kw.get("mode", "bipolar"), sc_prec=kw["sc_prec"], pool=cfg["table"],
        pool_dims=pool_dims, group_a=kw.get("group_a", 1), group_b=kw.get("group_b", 1),
        stoc_len=kw.get("stoc_len"), bias=None if bias is None else bias.numpy())
    acc_g = acc.view(BH, M, N).cpu().numpy()
    y_g = y.reshape(BH, M, N).cpu().numpy()
    np.testing.assert_array_equal(acc_g, acc_ref)
    np.testing.assert_allclose(y_g, y_ref, rtol=RTOL, atol=1e-30)
    return acc_g, y_g


CASES = [
    # (M, N, K, p, L, mode)
    (1, 1, 1, 7, 128, "bipolar"),
    (31, 33, 17, 7, 128, "bipolar"),
    (64, 64, 64, 7, 128, "bipolar"),
    (65, 130, 100, 8, 256, "bipolar"),
    (40, 70, 96, 8, 192, "bipolar"),
    (33, 31, 50, 6, 64, "bipolar"),
    (17, 9, 40, 5, 20, "bipolar"),
    (29, 45, 64, 2, 3, "bipolar"),
    (37, 41, 72, 6, 64, "unipolar"),
    (20, 66, 33, 8, 256, "unipolar"),
    (20, 66, 33, 1, 2, "unipolar"),
]


@pytest.mark.parametrize("engine", ["popc", "auto"])
@pytest.mark.parametrize("M,N,K,p,L,mode", CASES)
def test_per_row_parity(cuda_device, M, N, K, p, L, mode, engine):
    g = torch.Generator().manual_seed(M * 1000 + N)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    _run(cuda_device, a, b, _cfg("sobol", K, p), sc_prec=p, stoc_len=L, mode=mode, engine=engine)


@pytest.mark.parametrize("kind", ["anti", "alt", "lfsr"])
def test_pool_variants(cuda_device, kind):
    g = torch.Generator().manual_seed(7)
    a = torch.randn(48, 80, generator=g)
    b = torch.randn(56, 80, generator=g)
    _run(cuda_device, a, b, _cfg(kind, 80, 8, seed=5), sc_prec=8, stoc_len=256)


@pytest.mark.parametrize("gran", ["per_head", "per_tensor", "per_row"])
def test_batched_granularity(cuda_device, gran):
    g = torch.Generator().manual_seed(11)
    a = torch.randn(5, 33, 64, generator=g)
    b = torch.randn(5, 37, 64, generator=g)
    a[2] *= 10.0  # a loud slice must not rescale the others under per_head
    _run(cuda_device, a, b, _cfg("sobol", 64, 7), sc_prec=7, stoc_len=128, granularity=gran)


def test_groups_and_shared_b(cuda_device):
    g = torch.Generator().manual_seed(3)
    a = torch.randn(3, 50, 48, generator=g)
    b = torch.randn(45, 48, generator=g)
    _run(cuda_device, a, b, _cfg("sobol", 48, 8), sc_prec=8, stoc_len=256, group_a=4, group_b=7)


def test_chunk_d_is_chunk_sum(cuda_device):
    """chunk_d=64 over K=192: three 64-wide chunks, each quantised per row and
    rescaled on its own with the (64, p) pool, summed in chunk order."""
    dev = cuda_device
    g = torch.Generator().manual_seed(4)
    a = torch.randn(40, 192, generator=g)
    b = torch.randn(30, 192, generator=g)
    cfg = _cfg("sobol", 64, 7)
    acc = torch.empty(40 * 30, dtype=torch.int32, device=dev)
    y = sc_matmul(a.to(dev), b.to(dev), sc_prec=7, config=cfg, chunk_d=64, acc_out=acc)
    torch.cuda.synchronize()
    acc_ref, y_ref = sc_oracle.sc_matmul_segments_ref(a.numpy(), b.numpy(), 64, sc_prec=7,
                                                      pool=cfg["table"])
    np.testing.assert_array_equal(acc.view(40, 30).cpu().numpy(), acc_ref[0])
    np.testing.assert_allclose(y.cpu().numpy(), y_ref[0], rtol=RTOL, atol=1e-30)


def test_bias_fused(cuda_device):
    g = torch.Generator().manual_seed(5)
    a = torch.randn(70, 64, generator=g)
    b = torch.randn(90, 64, generator=g)
    bias = torch.randn(90, generator=g)
    _run(cuda_device, a, b, _cfg("sobol", 64, 7), sc_prec=7, stoc_len=128, bias=bias)


def test_row_stream_lengths(cuda_device):
    """Per-row L at one sc_prec (256/192/128 share p=8), pruned rows (0) and
    rows left to another call (-1)."""
    dev = cuda_device
    g = torch.Generator().manual_seed(6)
    M, N, K = 90, 40, 64
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g)
    bias = torch.randn(N, generator=g)
    cfg = _cfg("sobol", K, 8)
    levels = np.array([256, 192, 129, 0, -1])
    rowL = levels[np.random.default_rng(0).integers(0, len(levels), M)].astype(np.int32)
    out = torch.full((M, N), 7.0, device=dev)
    acc = torch.empty(M * N, dtype=torch.int32, device=dev)
    sc_matmul(a.to(dev), b.to(dev), sc_prec=8, config=cfg, bias=bias.to(dev),
              row_stoc_len=torch.from_numpy(rowL), out=out, acc_out=acc)
    torch.cuda.synchronize()
    acc_ref, y_ref = sc_oracle.sc_matmul_ref(a.numpy(), b.numpy(), sc_prec=8, pool=cfg["table"],
                                             bias=bias.numpy(), L_row=np.maximum(rowL, 0))
    y = out.cpu().numpy()
    keep = rowL >= 0
    np.testing.assert_array_equal(acc.view(M, N).cpu().numpy()[keep], acc_ref[0][keep])
    np.testing.assert_allclose(y[keep], y_ref[0][keep], rtol=RTOL, atol=1e-30)
    assert np.all(y[~keep] == 7.0)
    # Bucket restatement of the reference loop gives the same rows.
    acc_b, y_b = sc_oracle.sc_matmul_rows_ref(a.numpy(), b.numpy(), np.maximum(rowL, 0),
                                              {8: cfg["table"]}, bias=bias.numpy())
    np.testing.assert_array_equal(acc_b[keep], acc_ref[0][keep])


def test_slice_stream_lengths(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(8)
    a = torch.randn(4, 20, 64, generator=g)
    b = torch.randn(4, 24, 64, generator=g)
    cfg = _cfg("sobol", 64, 8)
    sl = torch.tensor([256, 128, 200, 0], dtype=torch.int32)
    acc = torch.empty(4 * 20 * 24, dtype=torch.int32, device=dev)
    y = sc_matmul(a.to(dev), b.to(dev), granularity="per_head", sc_prec=8, config=cfg,
                  slice_stoc_len=sl, acc_out=acc)
    torch.cuda.synchronize()
    acc = acc.view(4, 20, 24).cpu().numpy()
    for s, L in enumerate(sl.tolist()):
        if L == 0:
            assert np.all(acc[s] == 0) and np.all(y[s].cpu().numpy() == 0)
            continue
        acc_ref, y_ref = sc_oracle.sc_matmul_ref(a[s].numpy(), b[s].numpy(), granularity="per_head",
                                                 sc_prec=8, pool=cfg["table"], stoc_len=L)
        np.testing.assert_array_equal(acc[s], acc_ref[0])
        np.testing.assert_allclose(y[s].cpu().numpy(), y_ref[0], rtol=RTOL, atol=1e-30)


@pytest.mark.parametrize("M,N,K", [(257, 16, 96), (16, 300, 96), (3, 257, 96),
                                   (5, 40, 600)])  # K > 512: one warp per output
def test_thin_windows_on_cuda_cores(cuda_device, M, N, K):
    g = torch.Generator().manual_seed(M + N)
    a = torch.randn(2, M, K, generator=g)
    b = torch.randn(2, N, K, generator=g)
    _run(cuda_device, a, b, _cfg("sobol", K, 7), sc_prec=7, stoc_len=128, engine="popc")


def test_qkv_shape_full_size(cuda_device):
    """The qkv projection of one ViT-L/14 image: [257,1024] @ [3072,1024]^T
    at L=128 (per-tensor max-abs scaling, bipolar), checked in full."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(257, 1024, generator=g)
    b = torch.nn.init.trunc_normal_(torch.empty(3072, 1024), std=0.02, generator=g)
    _run(cuda_device, a, b, _cfg("sobol", 1024, 7), sc_prec=7, stoc_len=128,
         granularity="per_tensor")


def test_cpu_tensors_raise():
    with pytest.raises(RuntimeError, match="no CPU path"):
        sc_matmul(torch.randn(3, 4), torch.randn(5, 4), sc_prec=7,
                  config=_cfg("sobol", 4, 7))


def test_bad_stoc_len_raises(cuda_device):
    a = torch.randn(3, 4, device=cuda_device)
    with pytest.raises(EngineError, match="stoc_len"):
        sc_matmul(a, a, sc_prec=7, config=_cfg("sobol", 4, 7), stoc_len=129)


@pytest.mark.parametrize("shape_a,shape_b", [
    ((0, 16), (5, 16)),          # no a rows
    ((7, 16), (0, 16)),          # no b rows
    ((0, 9, 16), (0, 4, 16)),    # no slices
    ((3, 0, 16), (4, 16)),       # batched, no rows per slice
])
def test_empty_operands_give_empty_outputs(cuda_device, shape_a, shape_b):
    """Empty inputs (as the reference's torch code produces for an empty
    batch) return correctly shaped empty outputs without a launch error."""
    a = torch.randn(*shape_a, device=cuda_device)
    b = torch.randn(*shape_b, device=cuda_device)
    y = sc_matmul(a, b, sc_prec=7, config=_cfg("sobol", 16, 7))
    torch.cuda.synchronize()
    assert y.shape == (*shape_a[:-1], shape_b[-2])
    assert y.numel() == 0
    assert _lib.engine_status(reset=True) == 0
