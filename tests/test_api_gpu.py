"""GPU parity of the reference-facing layers (SCLinear, mixed precision,
HeadAlignedSCLinear, chunk-D, batched attention) against the oracle."""
import random

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import sc_oracle
from scmp_vit_b200 import attention, sc_linear
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200.head_aligned_comp import HeadAlignedSCLinear
from scmp_vit_b200.mp import MPConfig
from scmp_vit_b200.sc_linear import SCLinear

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def _linear(i, o, seed):
    g = torch.Generator().manual_seed(seed)
    lin = nn.Linear(i, o)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(o, i, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(o, generator=g) * 0.1)
    return lin


def test_sclinear_uniform(cuda_device):
    lin = _linear(96, 80, 0)
    random.seed(0)
    cfg = ch.make_sobol_simple_config(96, 96, 7)
    m = SCLinear(lin, 7, cfg_override=cfg).to(cuda_device)
    x = torch.randn(3, 11, 96, generator=torch.Generator().manual_seed(1))
    y = m(x.to(cuda_device)).cpu().numpy().reshape(33, 80)
    _, y_ref = sc_oracle.sc_matmul_ref(x.reshape(33, 96).numpy(), lin.weight.detach().cpu().numpy(),
                                       sc_prec=7, pool=cfg["table"],
                                       bias=lin.bias.detach().cpu().numpy())
    np.testing.assert_allclose(y, y_ref[0], rtol=RTOL, atol=1e-30)


def test_sclinear_fixed_mp_matches_bucket_loop(cuda_device):
    """Grouped launches give the same rows as the reference's per-level loop."""
    sc_linear._CFG_CACHE.clear()
    lin = _linear(64, 48, 2)
    mp = MPConfig([256, 192, 128], [0.3, 0.3, 0.4])
    m = SCLinear(lin, 8, mp_cfg=mp).to(cuda_device)
    x = torch.randn(70, 64, generator=torch.Generator().manual_seed(3))
    y = m(x.to(cuda_device)).cpu().numpy()
    from scmp_vit_b200.mp_linear import classify_input_rows
    row_L = classify_input_rows(x, mp).row_levels.numpy()
    assert sorted(set(row_L.tolist())) == [128, 192, 256]
    pools = {p: sc_linear._get_config(64, p)["table"] for p in (7, 8)}
    _, y_ref = sc_oracle.sc_matmul_rows_ref(x.numpy(), lin.weight.detach().cpu().numpy(), row_L,
                                            pools, bias=lin.bias.detach().cpu().numpy())
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-30)


def test_head_aligned_is_ordered_segment_sum(cuda_device):
    lin = _linear(128, 72, 4)
    random.seed(5)
    cfg = ch.make_sobol_simple_config(16, 16, 8)
    m = HeadAlignedSCLinear(lin, 8, n_heads=8, cfg_override=cfg).to(cuda_device)
    x = torch.randn(2, 21, 128, generator=torch.Generator().manual_seed(6))
    y = m(x.to(cuda_device)).cpu().numpy().reshape(42, 72)
    _, y_ref = sc_oracle.sc_matmul_segments_ref(x.reshape(42, 128).numpy(),
                                                lin.weight.detach().cpu().numpy(), 16, sc_prec=8,
                                                pool=cfg["table"], bias=lin.bias.detach().cpu().numpy())
    np.testing.assert_allclose(y, y_ref[0], rtol=RTOL, atol=1e-30)


def test_chunk_d_path(cuda_device):
    sc_linear._CFG_CACHE.clear()
    lin = _linear(200, 40, 7)  # 200 = 3 chunks of 64 + a zero-padded 8
    m = SCLinear(lin, 7, chunk_d=64).to(cuda_device)
    x = torch.randn(30, 200, generator=torch.Generator().manual_seed(8))
    y = m(x.to(cuda_device)).cpu().numpy()
    xp = np.pad(x.numpy(), ((0, 0), (0, 56)))
    wp = np.pad(lin.weight.detach().cpu().numpy(), ((0, 0), (0, 56)))
    _, y_ref = sc_oracle.sc_matmul_segments_ref(xp, wp, 64, sc_prec=7,
                                                pool=sc_linear._get_config(64, 7)["table"],
                                                bias=lin.bias.detach().cpu().numpy())
    np.testing.assert_allclose(y, y_ref[0], rtol=RTOL, atol=1e-30)


def test_attention_qk_av_batched(cuda_device):
    sc_linear._CFG_CACHE.clear()
    g = torch.Generator().manual_seed(9)
    B, H, N, D = 2, 3, 19, 64
    q, k, v = (torch.randn(B, H, N, D, generator=g) for _ in range(3))
    qk = attention.sc_qk(q.to(cuda_device), k.to(cuda_device), 7).cpu().numpy()
    _, qk_ref = sc_oracle.sc_matmul_ref(q.reshape(B * H, N, D).numpy(),
                                        k.reshape(B * H, N, D).numpy(), granularity="per_head",
                                        sc_prec=7, pool=sc_linear._get_config(D, 7)["table"])
    np.testing.assert_allclose(qk.reshape(B * H, N, N), qk_ref, rtol=RTOL, atol=1e-30)
    attn = torch.softmax(torch.from_numpy(qk_ref).reshape(B, H, N, N) * D ** -0.5, dim=-1)
    for mode in ("bipolar", "unipolar"):
        av = attention.sc_av(attn.to(cuda_device), v.to(cuda_device), 7, mode=mode).cpu().numpy()
        _, av_ref = sc_oracle.sc_matmul_ref(attn.reshape(B * H, N, N).numpy(),
                                            v.transpose(-1, -2).reshape(B * H, D, N).numpy(),
                                            mode=mode, sc_prec=7,
                                            pool=sc_linear._get_config(N, 7)["table"])
        np.testing.assert_allclose(av.reshape(B * H, N, D), av_ref, rtol=RTOL, atol=1e-30)


def test_attention_mp_per_head_and_per_row(cuda_device):
    sc_linear._CFG_CACHE.clear()
    g = torch.Generator().manual_seed(10)
    B, H, N, D = 2, 4, 17, 64
    q, k, v = (torch.randn(B, H, N, D, generator=g) for _ in range(3))
    mp = MPConfig([128, 256], [0.5, 0.5])
    qk = attention.sc_qk(q.to(cuda_device), k.to(cuda_device), 8, mp_cfg=mp).cpu().numpy()
    head_L = mp_head = q.abs().amax(dim=(0, 2, 3))
    order = torch.argsort(mp_head, descending=True, stable=True)
    head_L = torch.empty(H, dtype=torch.int64)
    head_L[order[:2]] = 256
    head_L[order[2:]] = 128
    for b in range(B):
        for h in range(H):
            L = int(head_L[h])
            p = 7 if L == 128 else 8
            _, ref = sc_oracle.sc_matmul_ref(q[b, h].numpy(), k[b, h].numpy(),
                                             granularity="per_head", sc_prec=p, stoc_len=L,
                                             pool=sc_linear._get_config(D, p)["table"])
            np.testing.assert_allclose(qk[b, h], ref[0], rtol=RTOL, atol=1e-30)
    attn = torch.softmax(torch.randn(B, H, N, N, generator=g), dim=-1)
    av = attention.sc_av(attn.to(cuda_device), v.to(cuda_device), 8, mp_cfg=mp).cpu().numpy()
    score = attention.av_row_score(attn.reshape(B * H, N, N))
    from scmp_vit_b200.mp import quantile_levels_batched
    row_L = quantile_levels_batched(score, [128, 256], [0.5, 0.5]).numpy()
    pools = {p: sc_linear._get_config(N, p)["table"] for p in (7, 8)}
    for i in range(B * H):
        _, ref = sc_oracle.sc_matmul_rows_ref(attn.reshape(B * H, N, N)[i].numpy(),
                                              v.transpose(-1, -2).reshape(B * H, D, N)[i].numpy(),
                                              row_L[i], pools)
        np.testing.assert_allclose(av.reshape(B * H, N, D)[i], ref, rtol=RTOL, atol=1e-30)


def test_vit_forward_small(cuda_device):
    """A small patched ViT runs end to end on the engine and stays close to FP."""
    from scmp_vit_b200 import vit
    torch.manual_seed(0)
    fp = vit.vit_l14(seed=0, dim=128, depth=2, heads=2, hidden=256, img=56).to(cuda_device)
    sc = vit.vit_l14(seed=0, dim=128, depth=2, heads=2, hidden=256, img=56).to(cuda_device)
    vit.patch_vit(sc, 8, ("qk", "av", "proj"), comp_blocks=[1])
    x = torch.randn(4, 3, 56, 56, device=cuda_device)
    with torch.no_grad():
        y_fp, y_sc = fp(x), sc(x)
    assert torch.isfinite(y_sc).all()
    rel = (y_sc - y_fp).norm() / y_fp.norm()
    assert rel < 0.2, float(rel)


@pytest.mark.parametrize("rows,d_in,d_out", [(514, 1024, 4096), (514, 4096, 1024), (77, 96, 40)])
def test_fp_mlp_linear_matches_f_linear(cuda_device, rows, d_in, d_out):
    """The ViT's FP MLP linears (matmul, then the bias added in place) give
    F.linear's bits on CUDA fp32 (the ViT-L/14 fc1 / fc2 shapes and a ragged
    one); bf16 inputs keep F.linear itself."""
    from scmp_vit_b200 import vit
    torch.backends.cuda.matmul.allow_tf32 = False
    lin = _linear(d_in, d_out, rows).to(cuda_device)
    x = torch.randn(2, rows // 2, d_in, generator=torch.Generator().manual_seed(d_in)).to(cuda_device)
    with torch.no_grad():
        assert torch.equal(vit._fp_linear(lin, x), nn.functional.linear(x, lin.weight, lin.bias))
        lb = lin.to(torch.bfloat16)
        xb = x.to(torch.bfloat16)
        assert torch.equal(vit._fp_linear(lb, xb), nn.functional.linear(xb, lb.weight, lb.bias))
