"""bf16 operands and bf16 output through the C ABI (io_flags).

A bf16 operand is widened to fp32 exactly, so the engine quantises the same
values as for an fp32 copy; a bf16 output is the fp32 result (bias
included) rounded to nearest even.  Both engines must therefore give
bit-identical counts and exactly ``y_fp32.to(torch.bfloat16)``.
"""
import random

import pytest
import torch

from scmp_vit_b200 import _lib
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200 import sc_matmul

pytestmark = pytest.mark.gpu


def _pair(dev, a, b, *, engine, out_bf16=True, **kw):
    BH = a.shape[0] if a.dim() == 3 else 1
    M, N = a.shape[-2], b.shape[-2]
    acc32 = torch.empty(BH * M * N, dtype=torch.int32, device=dev)
    acc16 = torch.empty_like(acc32)
    y32 = sc_matmul(a.float(), b.float(), acc_out=acc32, engine=engine, **kw)
    y16 = sc_matmul(a, b, acc_out=acc16, engine=engine,
                    out_dtype=torch.bfloat16 if out_bf16 else None, **kw)
    torch.cuda.synchronize()
    assert _lib.engine_status(reset=True) == 0
    assert torch.equal(acc16, acc32)
    return y32, y16


@pytest.mark.parametrize("engine", ["auto", "popc"])
def test_linear_bf16_in_out_with_bias(cuda_device, engine):
    dev = cuda_device
    g = torch.Generator().manual_seed(0)
    a = torch.randn(300, 512, generator=g).to(dev, torch.bfloat16)
    b = (torch.randn(700, 512, generator=g) * 0.02).to(dev, torch.bfloat16)
    bias = torch.randn(700, generator=g).to(dev)
    random.seed(1)
    cfg = ch.make_sobol_simple_config(512, 512, 7)
    y32, y16 = _pair(dev, a, b, engine=engine, sc_prec=7, config=cfg, stoc_len=128, bias=bias)
    assert y16.dtype == torch.bfloat16
    assert torch.equal(y16, y32.to(torch.bfloat16))


def test_qk_per_head_and_av_per_row_bf16(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(1)
    q = torch.randn(3, 257, 64, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(3, 257, 64, generator=g).to(dev, torch.bfloat16)
    random.seed(2)
    cq = ch.make_sobol_simple_config(64, 64, 7)
    y32, y16 = _pair(dev, q, k, engine="auto", granularity="per_head", sc_prec=7, config=cq)
    assert torch.equal(y16, y32.to(torch.bfloat16))
    attn = torch.softmax(y16.float(), -1).to(torch.bfloat16)
    vt = torch.randn(3, 64, 257, generator=g).to(dev, torch.bfloat16)
    cv = ch.make_sobol_simple_config(257, 257, 7)
    y32, y16 = _pair(dev, attn, vt, engine="auto", sc_prec=7, config=cv)
    assert torch.equal(y16, y32.to(torch.bfloat16))


def test_mixed_operands_fp32_out_and_segments(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(2)
    a = torch.randn(256, 256, generator=g).to(dev, torch.bfloat16)
    b = (torch.randn(128, 256, generator=g) * 0.05).to(dev)  # fp32 b, bf16 a
    random.seed(3)
    cfg = ch.make_sobol_simple_config(64, 64, 8)
    y32, y = _pair(dev, a, b, engine="auto", out_bf16=False, sc_prec=8, config=cfg,
                   stoc_len=256, k_segment=64)
    assert y.dtype == torch.float32
    assert torch.equal(y, y32)
