"""scmp_split_qkv: the fused qkv projection output split into the attention
SC operands (q, k [B, H, N, D], v^T [B, H, D, N]) in one engine pass.

The GPU tests compare it element for element with torch's
reshape / unbind / transpose (pure copies, so bit equality), for bf16 and
fp32, 16-byte and odd row lengths; the CPU test checks that bad arguments are
rejected before any device work.
"""
import ctypes

import pytest
import torch

from scmp_vit_b200 import _lib
from scmp_vit_b200.attention import split_qkv

EINVAL, EUNSUPPORTED = -1, -4  # enum scmp_status


def test_split_qkv_rejects_bad_arguments():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    assert lib.scmp_split_qkv(nul, 1, 1, 1, 8, 3, nul, nul, nul, nul) == EINVAL
    assert "elem_bytes" in _lib.last_error()
    assert lib.scmp_split_qkv(nul, 1, 1, 1, 512, 2, nul, nul, nul, nul) == EUNSUPPORTED
    assert lib.scmp_split_qkv(nul, 1, 4, 2, 8, 2, nul, nul, nul, nul) == EINVAL
    assert lib.scmp_split_qkv(nul, 0, 4, 2, 8, 2, nul, nul, nul, nul) == _lib.SCMP_OK


@pytest.mark.gpu
@pytest.mark.parametrize("B,N,H,D,dtype", [
    (2, 257, 16, 64, torch.bfloat16),   # ViT-L/14 attention, 16-byte rows
    (3, 257, 4, 64, torch.float32),
    (2, 33, 3, 36, torch.bfloat16),     # 72-byte rows: element-by-element path
    (1, 70, 5, 20, torch.float32),      # 80-byte rows, ragged token tiles
    (1, 130, 2, 256, torch.float32),    # the widest head: 66 KB transpose tile
])
def test_split_qkv_matches_torch(cuda_device, B, N, H, D, dtype):
    g = torch.Generator().manual_seed(B * 100 + N + H + D)
    qkv = torch.randn(B, N, 3 * H * D, generator=g).to(dtype).to(cuda_device)
    q, k, v = split_qkv(qkv, H)
    torch.cuda.synchronize()
    rq, rk, rv = torch.unbind(qkv.reshape(B, N, 3, H, D), 2)
    rq, rk, rv = rq.transpose(1, 2), rk.transpose(1, 2), rv.transpose(1, 2)
    assert q.is_contiguous() and k.is_contiguous()
    assert v.transpose(-1, -2).is_contiguous()  # v^T is the stored layout
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)
