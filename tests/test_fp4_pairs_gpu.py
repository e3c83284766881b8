"""Parity of the e2m1 CTA-pair kernel (tcgen05.mma kind::mxf4 with unit block
scales) against the oracle.

The engine routes every row-producer problem with one K segment at Lp = 128
or 256 there: 512-row tiles with two accumulators when a has more than 256
rows and b more than 128, else 256-row tiles with one accumulator of up to
256 columns (Q@Kᵀ and Attn@V per head).  Counts must be bit-exact (the fp32
accumulators hold integers below 2^24) and the rescaled outputs within 1e-5
relative, exactly as on the int8 path.  Shapes cover every tile width the
column heuristic picks (128 .. 240 b rows per tile), ragged a and b tails,
early termination, Lp = 256 with the shifted p = 8 compare, per-row stream
lengths, unipolar codes, batched slices, bias and bf16 output.
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


def _run(dev, a, b, p, L, *, mode="bipolar", granularity="per_row", bias=None, rowL=None,
         out_dtype=None):
    random.seed(p * 977 + L)
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
                  bias=None if bias is None else bias.to(dev), out_dtype=out_dtype, **kw)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    acc_ref, y_ref = sc_oracle.sc_matmul_ref(
        a.numpy(), b.numpy(), granularity=granularity, mode=mode, sc_prec=p, pool=cfg["table"],
        stoc_len=L, bias=None if bias is None else bias.numpy(), L_row=rowL)
    np.testing.assert_array_equal(acc.view(BH, M, N).cpu().numpy(), acc_ref)
    return y.reshape(BH, M, N).float().cpu().numpy(), y_ref


@pytest.mark.parametrize("M,N,K,p,L", [
    (512, 256, 64, 7, 128),     # one pair tile, 240-wide: the last 16 b rows in a second tile
    (300, 300, 64, 7, 128),     # 160-wide tiles, odd CTA's a rows mostly past the end
    (1024, 1024, 32, 7, 128),   # 208-wide tiles, last one partly past N
    (600, 3072, 16, 7, 128),    # 240-wide tiles (13 per row of tiles)
    (520, 400, 40, 7, 100),     # early termination inside Lp = 128, ragged everything
    (512, 272, 24, 8, 256),     # Lp = 256 (p = 8: shifted compare), 2 positions per half-row
    (768, 384, 40, 8, 200),     # Lp = 256 with early termination
    (513, 257, 72, 7, 128),     # 257th a row and b column on the CUDA-core strips
    (4096, 2560, 16, 7, 128),   # many tiles per cluster
    (600, 640, 257, 7, 128),    # K = 257: codes padded to 264
    # one stream length below 2^p at Lp = 256: the MMAs stop at the last
    # 64-position step a window can reach (3 of 4 at L = 192 and 160, 3 at
    # 129 -> windows up to 128 positions need only 2)
    (512, 272, 24, 8, 192),     # two accumulators
    (300, 300, 32, 8, 129),
    (256, 1000, 64, 8, 160),    # one accumulator
    (257, 64, 257, 8, 192),     # narrow tiles (Attn@V shape)
])
def test_fp4_pair_shapes(cuda_device, M, N, K, p, L):
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    y, y_ref = _run(cuda_device, a, b, p, L)
    np.testing.assert_allclose(y[0], y_ref[0], rtol=RTOL, atol=1e-30)


def test_fp4_pair_row_stream_lengths(cuda_device):
    """Per-row stream lengths (the MP split): windows k = |c| L_m >> p."""
    g = torch.Generator().manual_seed(11)
    M, N, K, p = 640, 320, 48, 7
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.1
    rowL = np.random.default_rng(3).choice(np.array([16, 64, 100, 128], np.int32), size=M)
    y, y_ref = _run(cuda_device, a, b, p, 128, rowL=rowL)
    np.testing.assert_allclose(y[0], y_ref[0], rtol=RTOL, atol=1e-30)


def test_fp4_pair_unipolar(cuda_device):
    g = torch.Generator().manual_seed(12)
    a = torch.rand(600, 40, generator=g)
    b = torch.rand(288, 40, generator=g)
    y, y_ref = _run(cuda_device, a, b, 7, 128, mode="unipolar")
    np.testing.assert_allclose(y[0], y_ref[0], rtol=RTOL, atol=1e-30)


def test_fp4_pair_sign_patterns(cuda_device):
    """Rows and columns whose codes are all negative, all positive or zero:
    every nibble value (0x0, 0x2, 0xA) in both operands."""
    g = torch.Generator().manual_seed(13)
    M, N, K = 520, 300, 32
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    a[:64] = -a[:64].abs()
    a[64:128] = a[64:128].abs()
    a[128:140] = 0.0
    b[:40] = -b[:40].abs()
    b[40:80] = 0.0
    y, y_ref = _run(cuda_device, a, b, 7, 128)
    np.testing.assert_allclose(y[0], y_ref[0], rtol=RTOL, atol=1e-30)


def test_fp4_pair_batched_bias_bf16(cuda_device):
    """Batched slices with a shared b (a weight), bias and bf16 output: the
    bf16 result is the fp32 result rounded to nearest even."""
    g = torch.Generator().manual_seed(14)
    a = torch.randn(3, 300, 64, generator=g)
    b = torch.randn(400, 64, generator=g) * 0.05
    bias = torch.randn(400, generator=g)
    y, y_ref = _run(cuda_device, a, b, 7, 128, bias=bias, out_dtype=torch.bfloat16)
    ref_bf16 = torch.from_numpy(y_ref.astype(np.float32)).to(torch.bfloat16).float().numpy()
    np.testing.assert_allclose(y, ref_bf16, rtol=1e-2, atol=1e-2)
    y32, y_ref32 = _run(cuda_device, a, b, 7, 128, bias=bias)
    np.testing.assert_allclose(y32, y_ref32, rtol=RTOL, atol=1e-30)


def test_fp4_pair_batched_per_slice_b(cuda_device):
    """Batched a and b (batch_b = batch), as Q @ K^T per head at M > 256."""
    g = torch.Generator().manual_seed(15)
    a = torch.randn(2, 520, 64, generator=g)
    b = torch.randn(2, 300, 64, generator=g)
    y, y_ref = _run(cuda_device, a, b, 7, 128, granularity="per_head")
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-30)


@pytest.mark.parametrize("M,N,K,p,L", [
    (256, 256, 64, 7, 128),     # Q@Kᵀ-shaped tile: one accumulator, 256 columns
    (200, 64, 264, 7, 128),     # Attn@V-shaped: 64 columns, odd CTA's a rows partly past the end
    (100, 16, 40, 7, 128),      # a rows only in the even CTA, the narrowest MMA (N = 16)
    (256, 100, 72, 8, 256),     # Lp = 256, 112 columns
    (240, 600, 48, 7, 96),      # 3 column tiles of up to 256, early termination
    (1024, 64, 32, 7, 128),     # narrow b with many a tiles
    (257, 200, 64, 7, 128),     # 257th a row on the CUDA-core strip
])
def test_fp4_one_accumulator_shapes(cuda_device, M, N, K, p, L):
    g = torch.Generator().manual_seed(M * 5 + N * 11 + K)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    y, y_ref = _run(cuda_device, a, b, p, L)
    np.testing.assert_allclose(y[0], y_ref[0], rtol=RTOL, atol=1e-30)


def test_fp4_one_accumulator_attention(cuda_device):
    """Q@Kᵀ per head (per_head scales, batched b) and Attn@V per row on
    peaked softmax rows, 257 tokens: one-accumulator tiles plus the strips."""
    g = torch.Generator().manual_seed(21)
    q = torch.randn(3, 257, 64, generator=g)
    k = torch.randn(3, 257, 64, generator=g)
    y, y_ref = _run(cuda_device, q, k, 7, 128, granularity="per_head")
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-30)
    attn = torch.softmax(torch.randn(3, 257, 257, generator=g) * 3.0, dim=-1)
    vt = torch.randn(3, 64, 257, generator=g)
    y, y_ref = _run(cuda_device, attn, vt, 7, 128)
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-30)


def test_fp4_one_accumulator_row_lengths_unipolar(cuda_device):
    g = torch.Generator().manual_seed(22)
    a = torch.randn(240, 48, generator=g)
    b = torch.randn(96, 48, generator=g) * 0.1
    rowL = np.random.default_rng(5).choice(np.array([0, 32, 77, 128], np.int32), size=240)
    y, y_ref = _run(cuda_device, a, b, 7, 128, rowL=rowL)
    np.testing.assert_allclose(y[0], y_ref[0], rtol=RTOL, atol=1e-30)
    a = torch.rand(250, 40, generator=g)
    b = torch.rand(120, 40, generator=g)
    y, y_ref = _run(cuda_device, a, b, 7, 128, mode="unipolar")
    np.testing.assert_allclose(y[0], y_ref[0], rtol=RTOL, atol=1e-30)


@pytest.mark.parametrize("temp", [0.01, 1.0, 30.0])
def test_fp4_narrow_window_chunk_shortcuts(cuda_device, temp):
    """Attn@V on flat (temp 0.01: every window near full length), mixed and
    peaked (temp 30: almost every window empty) softmax rows: the narrow
    kernel stores whole 32-position chunks without arithmetic when they lie
    inside or past every window of a warp's rows; counts stay exact."""
    g = torch.Generator().manual_seed(int(temp * 100) + 7)
    attn = torch.softmax(torch.randn(2, 257, 257, generator=g) * temp, dim=-1)
    vt = torch.randn(2, 64, 257, generator=g)
    y, y_ref = _run(cuda_device, attn, vt, 7, 128)
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-30)
    y, y_ref = _run(cuda_device, attn, vt, 8, 256)
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-30)


# ------------------------------------------------------------- K segments
# Segmented K (head-aligned compensation, chunk-D sums) runs on one-accumulator
# pair tiles (<= 240 columns, fp32 running sums in tensor memory next to the
# accumulator): each segment quantised and rescaled on its own, the fp32
# segment results summed in segment order, then the bias.

@pytest.mark.parametrize("M,N,K,kseg,p,L", [
    (600, 1024, 1024, 64, 8, 256),   # the compensation shape: 16 heads of 64, 5 tiles of 208
    (1000, 300, 512, 64, 8, 192),    # early termination, ragged a rows and b columns
    (513, 250, 256, 32, 7, 128),     # Lp = 128, 8 segments, one-row a tail
    (257, 1040, 128, 64, 8, 256),    # two segments, wide b
    (128, 40, 192, 16, 8, 256),      # narrow b, 12 segments of 16
])
def test_segments_on_pairs(cuda_device, M, N, K, kseg, p, L):
    dev = cuda_device
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    bias = torch.randn(N, generator=g)
    random.seed(kseg + p)
    cfg = ch.make_lfsr_config(kseg, kseg, p, seed=M)
    y = sc_matmul(a.to(dev), b.to(dev), sc_prec=p, config=cfg, stoc_len=L, k_segment=kseg,
                  bias=bias.to(dev), engine="tcgen05")
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    _, y_ref = sc_oracle.sc_matmul_segments_ref(a.numpy(), b.numpy(), kseg, sc_prec=p,
                                                pool=cfg["table"], stoc_len=L, bias=bias.numpy())
    np.testing.assert_allclose(y.cpu().numpy(), y_ref[0], rtol=RTOL, atol=1e-30)


def test_segments_on_pairs_per_row_lengths_and_batches(cuda_device):
    """Per-row stream lengths (0 = pruned row, bias only) across segments, and
    batched slices with their own b."""
    dev = cuda_device
    g = torch.Generator().manual_seed(77)
    BH, M, N, K, kseg = 3, 300, 176, 256, 64
    a = torch.randn(BH, M, K, generator=g)
    b = torch.randn(BH, N, K, generator=g) * 0.05
    rowL = np.random.default_rng(1).choice([0, 160, 256], BH * M).astype(np.int32)
    random.seed(3)
    cfg = ch.make_sobol_simple_config(kseg, kseg, 8)
    y = sc_matmul(a.to(dev), b.to(dev), sc_prec=8, config=cfg, k_segment=kseg,
                  row_stoc_len=torch.from_numpy(rowL), engine="tcgen05")
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    Lc = np.where(rowL > 0, rowL, 1).astype(np.int32)
    _, y_ref = sc_oracle.sc_matmul_segments_ref(a.numpy(), b.numpy(), kseg, sc_prec=8,
                                                pool=cfg["table"], L_row=Lc)
    y_ref = y_ref.reshape(BH * M, N)
    y_ref[rowL == 0] = 0.0
    np.testing.assert_allclose(y.cpu().numpy().reshape(BH * M, N), y_ref, rtol=RTOL, atol=1e-30)


# ----------------------------------------------------------------- K splits
# Problems whose output tiles would leave most SM pairs idle (one image's
# linear) split K across pairs: each split writes exact int32 partial counts
# and a reduce kernel rescales their sum, so results are those of one pass.

@pytest.mark.parametrize("prepacked", [False, True])
def test_k_splits_match_oracle_with_row_lengths(cuda_device, prepacked):
    from scmp_vit_b200.sc import prepack_b
    dev = cuda_device
    g = torch.Generator().manual_seed(5)
    M, N, K, p = 250, 1024, 768, 8
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    bias = torch.randn(N, generator=g)
    rowL = np.random.default_rng(2).choice([-1, 0, 64, 200, 256], M).astype(np.int32)
    random.seed(7)
    cfg = ch.make_sobol_simple_config(K, K, p)
    bd = b.to(dev)
    bb = prepack_b(bd, sc_prec=p, config=cfg) if prepacked else bd
    out = torch.full((M, N), 7.0, device=dev)
    acc = torch.full((M * N,), -9, dtype=torch.int32, device=dev)
    l0 = _lib.kernel_launches()
    sc_matmul(a.to(dev), bb, sc_prec=p, config=cfg, bias=bias.to(dev), out=out, acc_out=acc,
              row_stoc_len=torch.from_numpy(rowL), engine="tcgen05")
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    Lc = np.where(rowL > 0, rowL, 1).astype(np.int32)
    acc_ref, y_ref = sc_oracle.sc_matmul_ref(a.numpy(), b.numpy(), sc_prec=p, pool=cfg["table"],
                                             bias=bias.numpy(), L_row=Lc)
    y = out.cpu().numpy()
    accg = acc.view(M, N).cpu().numpy()
    keep, pruned = rowL > 0, rowL == 0
    np.testing.assert_array_equal(accg[keep], acc_ref[0][keep])
    np.testing.assert_allclose(y[keep], y_ref[0][keep], rtol=RTOL, atol=1e-30)
    np.testing.assert_array_equal(accg[pruned], 0)
    np.testing.assert_array_equal(y[pruned], np.broadcast_to(bias.numpy(), y[pruned].shape))
    np.testing.assert_array_equal(y[rowL < 0], 7.0)  # rows of another call: untouched
    np.testing.assert_array_equal(accg[rowL < 0], -9)
    assert _lib.kernel_launches() - l0 >= 3  # quantise, tiles, reduce (at least)


def test_k_splits_bf16_output(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(6)
    a = torch.randn(257, 1024, generator=g)
    b = torch.randn(3072, 1024, generator=g) * 0.02
    random.seed(1)
    cfg = ch.make_sobol_simple_config(1024, 1024, 7)
    y32 = sc_matmul(a.to(dev), b.to(dev), granularity="per_tensor", sc_prec=7, config=cfg,
                    stoc_len=128)
    y16 = sc_matmul(a.to(dev), b.to(dev), granularity="per_tensor", sc_prec=7, config=cfg,
                    stoc_len=128, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    assert torch.equal(y16, y32.to(torch.bfloat16))

