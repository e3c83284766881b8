"""scmp_sc_matmul_noalloc against scmp_sc_matmul, through the C ABI.

The no-alloc entry point serves callers that cannot allocate device memory
per call (a plain C / FFI host without a caching allocator, or a runtime
that owns the whole memory budget): it runs the same SC matmul with scratch
from a fixed array inside the library.  This file is named to be collected
last, so a stop-at-first-failure run has already run every other test.
"""
import ctypes
import random

import numpy as np
import pytest
import torch

from scmp_vit_b200 import _lib
from scmp_vit_b200 import config_helpers as ch
from scmp_vit_b200.sc import device_pool

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _args(a, b, pool, out, acc, *, p, L, dims, bias=None, engine="auto"):
    BH, M, K = a.shape
    N = b.shape[-2]
    x = _lib.MatmulArgs()
    x.abi_version = _lib.ABI_VERSION
    x.engine = _lib.ENGINE[engine]
    x.a, x.b = a.data_ptr(), b.data_ptr()
    x.batch, x.batch_b, x.M, x.N, x.K = BH, 1 if b.dim() == 2 else b.shape[0], M, N, K
    x.granularity = _lib.GRANULARITY["per_row"]
    x.mode = _lib.MODE["bipolar"]
    x.sc_prec, x.stoc_len = p, L
    x.group_a = x.group_b = 1
    x.pool, x.pool_dims = pool.data_ptr(), dims
    x.bias = None if bias is None else bias.data_ptr()
    x.out, x.acc_out = out.data_ptr(), acc.data_ptr()
    return x


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


# A sequence on the one shared array: a large tensor-core problem first, then
# smaller ones with other K paddings, stream lengths and engine routes, so each
# later call runs over bytes an earlier, different call left behind.
SEQUENCE = [
    # (BH, M, N, K, p, L, engine)
    (1, 700, 300, 200, 8, 256, "auto"),    # e2m1 CTA pairs, two accumulators
    (2, 65, 70, 90, 7, 128, "popc"),       # CUDA cores, codes padded 90 -> 96
    (2, 65, 70, 96, 7, 128, "auto"),       # tensor cores plus the one-row strips
    (1, 300, 64, 128, 7, 100, "auto"),     # e2m1 narrow tile, L < 2^p
    (2, 65, 70, 96, 7, 128, "auto"),       # the third call again
]


def test_noalloc_matches_workspace_entry_point_over_a_sequence(cuda_device):
    dev = cuda_device
    lib = _lib.load()
    g = torch.Generator().manual_seed(0)
    for call, (BH, M, N, K, p, L, engine) in enumerate(SEQUENCE):
        random.seed(call)
        cfg = ch.make_sobol_simple_config(K, K, p)
        pool = device_pool(cfg, dev)
        a = torch.randn(BH, M, K, generator=g).to(dev)
        b = (torch.randn(N, K, generator=g) * 0.05).to(dev)
        bias = torch.randn(N, generator=g).to(dev)
        out_ref = torch.empty(BH, M, N, device=dev)
        acc_ref = torch.empty(BH, M, N, dtype=torch.int32, device=dev)
        ref = _args(a, b, pool, out_ref, acc_ref, p=p, L=L, dims=K, bias=bias, engine=engine)
        need = lib.scmp_sc_matmul_workspace_size(ctypes.byref(ref))
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES
        # the workspace entry point on a workspace full of 0xFF bytes (NaN floats)
        ws = torch.full((need,), 0xFF, dtype=torch.uint8, device=dev)
        ref.workspace, ref.workspace_bytes = ws.data_ptr(), need
        _lib.check(lib.scmp_sc_matmul(ctypes.byref(ref), _stream(dev)))

        out = torch.full((BH, M, N), float("nan"), device=dev)
        acc = torch.full((BH, M, N), -7, dtype=torch.int32, device=dev)
        na = _args(a, b, pool, out, acc, p=p, L=L, dims=K, bias=bias, engine=engine)
        _lib.check(lib.scmp_sc_matmul_noalloc(ctypes.byref(na), _stream(dev)))
        torch.cuda.synchronize(dev)
        assert _lib.engine_status() == 0
        np.testing.assert_array_equal(acc.cpu().numpy(), acc_ref.cpu().numpy(),
                                      err_msg=f"call {call}")
        np.testing.assert_allclose(out.cpu().numpy(), out_ref.cpu().numpy(), rtol=RTOL,
                                   atol=1e-30, err_msg=f"call {call}")


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    x = _lib.MatmulArgs()
    x.abi_version = _lib.ABI_VERSION
    x.batch, x.batch_b, x.M, x.N, x.K = 1, 1, 8192, 8192, 1024
    x.sc_prec, x.stoc_len, x.group_a, x.group_b, x.pool_dims = 7, 128, 1, 1, 1024
    x.a = x.b = x.pool = x.out = 16  # never dereferenced: rejected before any launch
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(x)) > _lib.NOALLOC_SCRATCH_BYTES
    rc = lib.scmp_sc_matmul_noalloc(ctypes.byref(x), None)
    assert rc == -3
    assert "SCMP_NOALLOC_SCRATCH_BYTES" in _lib.last_error()
