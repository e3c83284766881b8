"""Closed-form Gaussian stand-in for SC matmuls (the reference's
``sc_integration/noise_matmul.py`` switch, kept so ``set_noise_model(True)``
still routes around the engine for fast sensitivity sweeps).

It is not an engine and makes no bit-level claim.  Restated from the
reference's docstring (``noise_matmul.py:12-34``): operands are re-quantised
to the SC grid of ``p = ceil(log2 L)``; the output is the exact product of
the quantised operands plus Gaussian noise whose variance is the Bernoulli
variance divided by ``L^2`` (Sobol scaling) times an empirical correction
(``noise_matmul.py:64-72``: 0.15 with local scales, 0.60 with a global one):

    bipolar:  Var = (D - a^2 @ (b^2)^T) / L^2     a, b normalised to [-1, 1]
    unipolar: Var = (a @ b^T - a^2 @ (b^2)^T) / L^2   a, b normalised to [0, 1]
"""
from __future__ import annotations

import math
from typing import Optional

import torch

NOISE_LOCAL_CORRECTION: float = 0.15
NOISE_GLOBAL_CORRECTION: float = 0.60


def set_noise_corrections(local: float, global_: float) -> None:
    global NOISE_LOCAL_CORRECTION, NOISE_GLOBAL_CORRECTION
    NOISE_LOCAL_CORRECTION = float(local)
    NOISE_GLOBAL_CORRECTION = float(global_)


def _grid(x: torch.Tensor, qmax: int) -> torch.Tensor:
    return torch.round(x * qmax) / qmax


@torch.no_grad()
def _noisy_matmul_core(a: torch.Tensor, b: torch.Tensor, L: int, mode: str = "bipolar",
                       per_row_scale: bool = False) -> torch.Tensor:
    """``a @ b^T`` (..., M, N) in fp32 plus calibrated SC noise."""
    if mode not in ("bipolar", "unipolar"):
        raise ValueError(f"unknown SC mode: {mode}")
    a = a.float()
    b = b.float()
    if L is None or L <= 0:
        return (a @ b.transpose(-2, -1)) * 0.0
    p = max(1, int(math.ceil(math.log2(L))))
    local = per_row_scale or a.dim() > 2
    corr = NOISE_LOCAL_CORRECTION if local else NOISE_GLOBAL_CORRECTION
    dims = (-1,) if per_row_scale else (-2, -1)
    if mode == "bipolar":
        sa = a.abs().amax(dim=dims, keepdim=True).clamp(min=1e-12)
        sb = b.abs().amax(dim=dims, keepdim=True).clamp(min=1e-12)
        qmax = max(1, 2 ** (p - 1) - 1)
        an, bn = _grid(a / sa, qmax), _grid(b / sb, qmax)
        exact = an @ bn.transpose(-2, -1)
        var = (a.shape[-1] - (an * an) @ (bn * bn).transpose(-2, -1)).clamp(min=0)
    else:
        lo_a, lo_b = a.amin(dim=dims, keepdim=True), b.amin(dim=dims, keepdim=True)
        sa = (a.amax(dim=dims, keepdim=True) - lo_a).clamp(min=1e-12)
        sb = (b.amax(dim=dims, keepdim=True) - lo_b).clamp(min=1e-12)
        qmax = 2 ** p - 1
        an, bn = _grid((a - lo_a) / sa, qmax), _grid((b - lo_b) / sb, qmax)
        exact = an @ bn.transpose(-2, -1)
        var = (exact - (an * an) @ (bn * bn).transpose(-2, -1)).clamp(min=0)
    noisy = exact + torch.randn_like(exact) * torch.sqrt(var * corr) / float(L)
    scale = sa * sb.transpose(-2, -1)
    if mode == "bipolar":
        return noisy * scale
    # undo the offsets: (an*sa + lo_a) . (bn*sb + lo_b)
    D = a.shape[-1]
    out = noisy * scale
    out = out + lo_a * (bn * sb).sum(-1, keepdim=True).transpose(-2, -1)
    out = out + (an * sa).sum(-1, keepdim=True) * lo_b.transpose(-2, -1)
    return out + D * lo_a * lo_b.transpose(-2, -1)


def _resolve_L(stoc_len: Optional[int], sc_prec: int) -> int:
    if stoc_len is not None and stoc_len > 0:
        return int(stoc_len)
    return int(2 ** int(sc_prec))


@torch.no_grad()
def noisy_sc_matmul_grouped(a, b, group_a: int = 1, group_b: int = 1, mode: str = "unipolar",
                            sc_prec: int = 8, config: Optional[dict] = None,
                            stoc_len: Optional[int] = None) -> torch.Tensor:
    return _noisy_matmul_core(a, b, L=_resolve_L(stoc_len, sc_prec), mode=mode,
                              per_row_scale=(group_a == 1 and group_b == 1))


@torch.no_grad()
def noisy_sc_matmul(a, b, max_fp_a=0.0, min_fp_a=0.0, max_fp_b=None, min_fp_b=None,
                    mode: str = "bipolar", sc_prec: int = 8, config: Optional[dict] = None,
                    stoc_len: Optional[int] = None) -> torch.Tensor:
    return _noisy_matmul_core(a, b, L=_resolve_L(stoc_len, sc_prec), mode=mode)
