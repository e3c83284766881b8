"""The fused softmax + Attn@V a-operand quantisation (scmp_softmax_quantize)
against the unfused steps: torch.softmax's bits, and Attn@V results equal to
quantising torch's probabilities."""
import random

import pytest
import torch

from scmp_vit_b200 import attention
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200.sc import QuantizedRows, sc_matmul, softmax_quantize

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K", [33, 64, 100, 256, 257, 288, 289, 513, 1000])
def test_probabilities_match_torch_softmax(cuda_device, K):
    g = torch.Generator().manual_seed(K)
    rows = 700
    x = (torch.randn(rows, K, generator=g) * torch.rand(rows, 1, generator=g) * 40).to(cuda_device)
    x[0] = 0.0                       # a flat row
    x[1, 5] = 1e4                    # one dominant element
    scale = 64 ** -0.5
    qa = softmax_quantize(x, scale, mode="bipolar", sc_prec=8, keep_probs=True)
    ref = (x * scale).softmax(dim=-1)
    torch.cuda.synchronize()
    assert torch.equal(qa.probs, ref)


@pytest.mark.parametrize("mode,p", [("bipolar", 8), ("bipolar", 7), ("unipolar", 7)])
def test_quantised_a_matches_probabilities(cuda_device, mode, p):
    dev = cuda_device
    g = torch.Generator().manual_seed(p)
    BH, N, D = 3, 257, 64
    scores = (torch.randn(BH, N, N, generator=g) * 6).to(dev)
    vt = torch.randn(BH, D, N, generator=g).to(dev)
    random.seed(p)
    cfg = ch.make_sobol_simple_config(N, N, p)
    scale = D ** -0.5
    probs = (scores * scale).softmax(dim=-1)
    kw = dict(granularity="per_row", mode=mode, sc_prec=p, config=cfg)
    acc_ref = torch.empty(BH * N * D, dtype=torch.int32, device=dev)
    acc = torch.empty_like(acc_ref)
    y_ref = sc_matmul(probs, vt, acc_out=acc_ref, **kw)
    qa = softmax_quantize(scores, scale, mode=mode, sc_prec=p)
    assert isinstance(qa, QuantizedRows) and qa.shape == (BH, N, N)
    y = sc_matmul(qa, vt, acc_out=acc, **kw)
    torch.cuda.synchronize()
    assert torch.equal(acc, acc_ref)
    assert torch.equal(y, y_ref)
    with pytest.raises(ValueError, match="quantised a"):
        sc_matmul(qa, vt, granularity="per_row", mode=mode, sc_prec=p, config=cfg, group_a=2)


def test_attention_forward_fused_equals_unfused(cuda_device):
    """The patched attention forward gives the same bits with the fused
    softmax as with torch.softmax followed by Attn@V."""
    from scmp_vit_b200 import vit
    dev = cuda_device
    torch.manual_seed(0)
    m = vit.vit_l14(seed=0, dim=128, depth=2, heads=2, hidden=256, img=56).to(dev)
    vit.patch_vit(m, 8, ("qk", "av", "proj"))
    x = torch.randn(3, 3, 56, 56, generator=torch.Generator().manual_seed(1)).to(dev)
    try:
        attention.set_fused_softmax(False)
        with torch.no_grad():
            y0 = m(x)
        attention.set_fused_softmax(True)
        with torch.no_grad():
            y1 = m(x)
    finally:
        attention.set_fused_softmax(True)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
