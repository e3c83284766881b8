"""The fused fp32 block glue (scmp_bias_gelu, scmp_scale_residual) against
the torch ops it replaces: identical bits."""
import pytest
import torch
import torch.nn.functional as F

from scmp_vit_b200 import vit

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols", [(514, 4096), (77, 96), (5, 7)])
def test_bias_gelu_matches_torch(cuda_device, rows, cols):
    g = torch.Generator().manual_seed(cols)
    t = (torch.randn(rows, cols, generator=g) * torch.rand(rows, 1, generator=g) * 12)
    t[0, :3] = torch.tensor([0.0, -1e-30, 30.0])
    t = t.to(cuda_device)
    b = torch.randn(cols, generator=g).to(cuda_device)
    ref = F.gelu(t + b)
    got = vit.bias_gelu_(t.clone(), b)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


@pytest.mark.parametrize("with_bias,with_extra", [(False, False), (True, False), (True, True)])
@pytest.mark.parametrize("rows,cols", [(514, 1024), (33, 10)])
def test_scale_residual_matches_torch(cuda_device, rows, cols, with_bias, with_extra):
    g = torch.Generator().manual_seed(rows + cols)
    x, y, e = (torch.randn(rows, cols, generator=g).to(cuda_device) for _ in range(3))
    gamma = (torch.rand(cols, generator=g) * 2).to(cuda_device)
    bias = torch.randn(cols, generator=g).to(cuda_device) if with_bias else None
    yb = y + bias if with_bias else y
    ref = x + yb * gamma
    if with_extra:
        ref = ref + e
    got = vit.scale_residual(x, y, gamma, bias=bias, extra=e if with_extra else None)
    yc = y.clone()
    inplace = vit.scale_residual(x, yc, gamma, bias=bias, extra=e if with_extra else None, out=yc)
    torch.cuda.synchronize()
    assert torch.equal(got, ref) and torch.equal(inplace, ref)


def test_block_forward_fused_glue_equals_unfused(cuda_device):
    """A small patched ViT (head-aligned compensation on one block) gives the
    same logits with the fused block glue as with the separate torch ops."""
    dev = cuda_device
    m = vit.vit_l14(seed=0, dim=128, depth=2, heads=2, hidden=256, img=56).to(dev)
    with torch.no_grad():
        for blk in m.backbone.blocks:  # non-trivial layer scales
            blk.ls1.gamma.uniform_(0.5, 1.5)
            blk.ls2.gamma.uniform_(0.5, 1.5)
    vit.patch_vit(m, 8, ("qk", "av", "proj"), comp_blocks=[1])
    x = torch.randn(3, 3, 56, 56, generator=torch.Generator().manual_seed(4)).to(dev)
    try:
        vit.set_fused_glue(False)
        with torch.no_grad():
            y0 = m(x)
        vit.set_fused_glue(True)
        with torch.no_grad():
            y1 = m(x)
    finally:
        vit.set_fused_glue(True)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
