"""The give-up path of the engine's bounded device waits, and the e2m1 MMA-rate
probe.

Every mbarrier wait of the tensor-core engine spins for at most a limit, then
marks its CTA aborted; the CTA waits for the tensor-core work it already
issued, frees its tensor memory and returns, and the launch raises bit 0 of
the engine error word.  Here the wait is made to run out on purpose: the
producers of the e2m1 kernels are held on a device flag that nothing sets,
with a short (20 ms) limit.  The test checks that the launch returns, the
error word says so, and that the very next normal call on the same context
is bit-exact against the oracle.
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

DEFAULT_LIMIT_NS = 2_000_000_000


@pytest.mark.parametrize("M,N", [(600, 300), (300, 64)])  # e2m1 CTA pairs / narrow tiles
def test_bounded_wait_gives_up_and_the_engine_recovers(cuda_device, M, N):
    dev = cuda_device
    K, p = 128, 7
    random.seed(0)
    cfg = ch.make_sobol_simple_config(K, K, p)
    g = torch.Generator().manual_seed(M + N)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    ad, bd = a.to(dev), b.to(dev)
    _lib.engine_status(reset=True)
    out = torch.full((M, N), float("nan"), device=dev)
    _lib.set_wait_limit(20_000_000)
    _lib.hold_producers(True)
    try:
        sc_matmul(ad, bd, sc_prec=p, config=cfg, stoc_len=128, engine="tcgen05", out=out)
        torch.cuda.synchronize(dev)
        status = _lib.engine_status(reset=True)
    finally:
        _lib.hold_producers(False)
        _lib.set_wait_limit(DEFAULT_LIMIT_NS)
    assert status & 1, "the held launch should report that its waits gave up"
    assert _lib.engine_status() == 0

    # the same context runs the next call normally, bit-exact
    acc = torch.empty(M * N, dtype=torch.int32, device=dev)
    y = sc_matmul(ad, bd, sc_prec=p, config=cfg, stoc_len=128, engine="tcgen05", acc_out=acc)
    torch.cuda.synchronize(dev)
    assert _lib.engine_status() == 0
    acc_ref, y_ref = sc_oracle.sc_matmul_ref(a.numpy(), b.numpy(), sc_prec=p, pool=cfg["table"],
                                             stoc_len=128)
    np.testing.assert_array_equal(acc.view(M, N).cpu().numpy(), acc_ref[0])
    np.testing.assert_allclose(y.cpu().numpy(), y_ref[0], rtol=1e-5, atol=1e-30)


def test_wait_limit_rejects_zero(cuda_device):
    with pytest.raises(_lib.EngineError, match="positive"):
        _lib.set_wait_limit(0)


@pytest.mark.parametrize("kind,n", [(3, 256), (4, 64)])
def test_mxf4_mma_rate_probe(cuda_device, kind, n):
    """The measured e2m1 MMA rate (MACs/s = SC bit-products/s) lies between
    1e14 and 16384 MAC/clk/SM x 148 SMs x 2.1 GHz (above any B200 clock)."""
    rate = _lib.probe_int_peak(kind)
    assert 1e14 < rate < 16384 * 148 * 2.1e9
    assert _lib.engine_status() == 0
