"""Parity of the tcgen05 (tensor-core) engine against the oracle.

Same contract as the CUDA-core engine: popcount accumulators bit-exact,
rescaled outputs within 1e-5 relative.  Shapes cover full tiles, ragged
tails taken by the CUDA-core strips (257 rows / columns), padded tails,
every padded stream length (Lp = 32, 64, 128, 256), early termination,
unipolar, per-row stream lengths and the error word staying clear.
"""
import random

import numpy as np
import pytest
import torch

from oracle import sc_oracle
from scmp_vit_b200 import _lib
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200 import sc_matmul

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def _check(dev, a, b, p, L, *, mode="bipolar", granularity="per_row", bias=None, rowL=None):
    random.seed(p * 1000 + L)
    K = a.shape[-1]
    cfg = ch.make_sobol_simple_config(K, K, p)
    BH = a.shape[0] if a.dim() == 3 else 1
    M, N = a.shape[-2], b.shape[-2]
    acc = torch.empty(BH * M * N, dtype=torch.int32, device=dev)
    kw = {}
    if rowL is not None:
        kw["row_stoc_len"] = torch.from_numpy(rowL)
    y = sc_matmul(a.to(dev), b.to(dev), granularity=granularity, mode=mode, sc_prec=p,
                  config=cfg, stoc_len=L, acc_out=acc, engine="tcgen05",
                  bias=None if bias is None else bias.to(dev), **kw)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    acc_ref, y_ref = sc_oracle.sc_matmul_ref(
        a.numpy(), b.numpy(), granularity=granularity, mode=mode, sc_prec=p, pool=cfg["table"],
        stoc_len=L, bias=None if bias is None else bias.numpy(), L_row=rowL)
    np.testing.assert_array_equal(acc.view(BH, M, N).cpu().numpy(), acc_ref)
    np.testing.assert_allclose(y.reshape(BH, M, N).cpu().numpy(), y_ref, rtol=RTOL, atol=1e-30)


def test_tc_single_tile(cuda_device):
    g = torch.Generator().manual_seed(0)
    _check(cuda_device, torch.randn(256, 64, generator=g), torch.randn(256, 64, generator=g), 7, 128)


@pytest.mark.parametrize("M,N,K,p,L", [
    (512, 256, 96, 7, 128),     # two row tiles
    (256, 512, 40, 8, 256),     # p=8 bipolar (shifted pool compare), 2 k-blocks per d
    (256, 256, 50, 8, 192),     # early termination, Lp = 256
    (256, 256, 33, 6, 64),      # Lp = 64: two dims per k-block
    (256, 256, 65, 5, 32),      # Lp = 32: four dims per k-block, ragged last k-block
    (257, 257, 64, 7, 128),     # 257th row/column through the CUDA-core strips
    (300, 64, 257, 7, 128),     # padded row tail, BN = 64
    (256, 100, 80, 7, 100),     # BN = 128 with padded columns, L not a power of two
    # row producers (K % 8 == 0) at every padded length and tile width
    (256, 256, 64, 6, 64),      # Lp = 64, BN = 256: a chunks of index 2j + half
    (256, 128, 48, 6, 50),      # Lp = 64, BN = 128, L not a power of two
    (300, 64, 72, 6, 64),       # Lp = 64, BN = 64, padded row tail
    (256, 64, 64, 8, 256),      # Lp = 256, BN = 64
    (512, 128, 40, 8, 200),     # Lp = 256, BN = 128, early termination
    (256, 256, 8, 7, 128),      # one macro step (8 reduction indices)
    # CTA pairs (N > 128): the odd CTA's a rows / b rows partly or wholly past the end
    (300, 300, 64, 7, 128),
    (4096, 2560, 16, 7, 128),   # 80 pair tiles: clusters loop over several tiles
    (280, 264, 64, 7, 128),     # 24-row tail in a padded tile, 8-column tail on the CUDA cores
    (256, 128, 257, 7, 128),    # K = 257: codes padded to 264 for the row producers
])
def test_tc_shapes(cuda_device, M, N, K, p, L):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    _check(cuda_device, a, b, p, L)


def test_tc_batched_per_head(cuda_device):
    g = torch.Generator().manual_seed(1)
    a = torch.randn(3, 257, 64, generator=g)
    b = torch.randn(3, 257, 64, generator=g)
    _check(cuda_device, a, b, 7, 128, granularity="per_head")


def test_tc_unipolar_bias(cuda_device):
    g = torch.Generator().manual_seed(2)
    a = torch.rand(256, 70, generator=g)
    b = torch.randn(128, 70, generator=g)
    _check(cuda_device, a, b, 7, 128, mode="unipolar", bias=torch.randn(128, generator=g))


def test_tc_unipolar_rows(cuda_device):
    """Unipolar through the row producers (K % 8 == 0): zero points and row sums."""
    g = torch.Generator().manual_seed(4)
    a = torch.rand(256, 72, generator=g)
    b = torch.randn(192, 72, generator=g)
    _check(cuda_device, a, b, 7, 128, mode="unipolar", bias=torch.randn(192, generator=g))


def test_tc_sparse_windows_attn_v(cuda_device):
    """Attn@V-shaped: peaked softmax rows give mostly short enable windows, so
    the narrow-tile producers skip whole all-zero chunks; counts stay exact."""
    g = torch.Generator().manual_seed(6)
    a = torch.softmax(torch.randn(300, 264, generator=g) * 3.0, dim=-1)
    b = torch.randn(64, 264, generator=g)
    _check(cuda_device, a, b, 7, 128)


def test_tc_row_stream_lengths(cuda_device):
    g = torch.Generator().manual_seed(3)
    a = torch.randn(256, 64, generator=g)
    b = torch.randn(256, 64, generator=g)
    rowL = np.random.default_rng(0).choice([256, 192, 130, 0], size=256).astype(np.int32)
    _check(cuda_device, a, b, 8, 256, rowL=rowL)


def test_tc_qkv_image(cuda_device):
    """qkv_proj of one ViT-L/14 image on the tensor-core engine (with the
    257th-row strip), per-tensor scaling, L=128."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(257, 1024, generator=g)
    b = torch.nn.init.trunc_normal_(torch.empty(3072, 1024), std=0.02, generator=g)
    _check(cuda_device, a, b, 7, 128, granularity="per_tensor")


@pytest.mark.parametrize("M,N,K,kseg,p,L,mode", [
    (256, 128, 256, 64, 8, 256, "bipolar"),    # head-aligned: 4 heads of 64, L=256
    (300, 200, 128, 32, 7, 128, "bipolar"),    # row tail 44 (padded tile), BN=128 + column tail
    (256, 64, 192, 64, 7, 100, "unipolar"),    # BN=64, L not a power of two
])
def test_tc_segments(cuda_device, M, N, K, kseg, p, L, mode):
    """Segmented K on the tensor cores: per-segment quantisation and rescale,
    fp32 segment sums in order (head-aligned compensation, chunk-D sum)."""
    dev = cuda_device
    g = torch.Generator().manual_seed(M + K + kseg)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    if mode == "unipolar":
        a = a.abs()
    bias = torch.randn(N, generator=g)
    random.seed(9)
    cfg = ch.make_sobol_simple_config(kseg, kseg, p)
    y = sc_matmul(a.to(dev), b.to(dev), mode=mode, sc_prec=p, config=cfg, stoc_len=L,
                  k_segment=kseg, bias=bias.to(dev), engine="tcgen05")
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    _, y_ref = sc_oracle.sc_matmul_segments_ref(a.numpy(), b.numpy(), kseg, mode=mode, sc_prec=p,
                                                pool=cfg["table"], stoc_len=L, bias=bias.numpy())
    np.testing.assert_allclose(y.cpu().numpy(), y_ref[0], rtol=RTOL, atol=1e-30)
