"""QwT-style block compensation at inference: ``out = block_sc(x) + comp(x)``.

Per transformer block ``i`` a ridge fit of the SC->FP residual gives an
affine correction ``comp(x) = x @ W_i + b_i`` (``docs/SC_COMP_ALGORITHM.md``
§1); a block is admitted when the fits on two calibration batches agree in
direction (cosine > tau, and both norms > eps), and the installed correction
is their average (§2). At inference the correction runs through the SC
engine too, normally as a ``HeadAlignedSCLinear`` (§3).

This module holds the inference side:

* ``CompensationBlock`` — the wrapper, with the wrapped block at ``.block``
  (the reference's ``qwt_sc.compensation.CompensationBlock`` shape, used by
  ``det/experiments/qwt_debug.py:97-115``);
* the (W, b) -> layer factories of ``det/experiments/qwt_det_compensate.py:
  54-101`` (FP ``nn.Linear``, ``SCLinear``, ``HeadAlignedSCLinear``; W is
  ``(D_in, D_out)``, the layer weight is ``W^T * scale * polarity``);
* ``RidgeFitter`` — the closed-form ridge solve with the bias column
  unregularised, which the reference's MP search imports from
  ``scmp_kernels.mp`` (``sc_integration/mp_search.py:49,728``);
* ``admit_pair`` — the cross-seed gate and average;
* ``save_comp_state`` / ``load_comp_state`` / ``install_compensation`` — an
  on-disk record of the admitted (W̄, b̄) per block. The reference keeps its
  fits inside the QwT-SC submodule, which is not vendored, so the file
  format here is this package's own (a ``torch.save`` dict, versioned).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn

from .head_aligned_comp import HeadAlignedSCLinear
from .sc_linear import SCLinear

COMP_FORMAT = "scmp_vit_b200.qwt_comp/1"


class CompensationBlock(nn.Module):
    """``block(x, ...) + comp(x)`` (the correction cast to the block's dtype);
    ``enabled=False`` passes the block through unchanged."""

    def __init__(self, block: nn.Module, comp: nn.Module, enabled: bool = True):
        super().__init__()
        self.block = block
        self.comp = comp
        self.enabled = bool(enabled)

    def forward(self, x, *args, **kwargs):
        y = self.block(x, *args, **kwargs)
        if not self.enabled:
            return y
        return y + self.comp(x).to(y.dtype)


def _linear_from(W: torch.Tensor, b: torch.Tensor, scale: float, polarity: int) -> nn.Linear:
    d_in, d_out = W.shape
    layer = nn.Linear(d_in, d_out, bias=True)
    with torch.no_grad():
        layer.weight.copy_(W.t().contiguous() * (scale * polarity))
        layer.bias.copy_(b * polarity if polarity == -1 else b)
    return layer.to(W.device)


def make_fp_factory(scale: float = 1.0, polarity: int = 1) -> Callable:
    """(W, b) -> FP ``nn.Linear`` (debug / baseline: an FP multiplier)."""
    return lambda W, b: _linear_from(W, b, scale, polarity)


def make_sc_comp_factory(sc_prec: int, mode: str = "bipolar", scale: float = 1.0,
                         polarity: int = 1) -> Callable:
    """(W, b) -> ``SCLinear`` over the whole ``D_in`` (pool ``(D_in, p)``)."""
    return lambda W, b: SCLinear(_linear_from(W, b, scale, polarity), sc_prec, mode=mode)


def make_head_aligned_comp_factory(sc_prec: int, mode: str = "bipolar", n_heads: int = 16,
                                   scale: float = 1.0, polarity: int = 1) -> Callable:
    """(W, b) -> ``HeadAlignedSCLinear``: the comp matmul as ``n_heads``
    segments of ``D_in / n_heads`` sharing the ``(D_in / n_heads, p)`` pool
    that the block's per-head Q@K^T already uses; one launch on this engine."""
    return lambda W, b: HeadAlignedSCLinear(_linear_from(W, b, scale, polarity), sc_prec,
                                            mode=mode, n_heads=n_heads)


class RidgeFitter:
    """Closed-form ridge regression of targets R on ``[X | 1]`` with the
    slope regularised and the bias not:
    ``[W; b] = (X_aug^T X_aug + ridge * diag(I, 0))^-1 X_aug^T R``.
    The Gram matrix is factorised once (Cholesky) and reused per target."""

    def __init__(self, X: torch.Tensor, ridge: float = 1e-4):
        X = X.reshape(-1, X.shape[-1]).to(torch.float64)
        self.n, self.d = X.shape
        self.X_aug = torch.cat([X, torch.ones(self.n, 1, dtype=X.dtype, device=X.device)], 1)
        G = self.X_aug.T @ self.X_aug
        reg = torch.full((self.d + 1,), float(ridge), dtype=X.dtype, device=X.device)
        reg[-1] = 0.0
        G = G + torch.diag(reg)
        self.L = torch.linalg.cholesky(G)

    def fit(self, R: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(W [D, D_out], b [D_out]) in fp32 for targets R [N, D_out]."""
        R = R.reshape(self.n, -1).to(torch.float64)
        sol = torch.cholesky_solve(self.X_aug.T @ R, self.L)
        return sol[:-1].to(torch.float32), sol[-1].to(torch.float32)

    def residual_norm_sq(self, R: torch.Tensor) -> float:
        """||R - [X | 1] [W; b]||^2 after the fit."""
        R = R.reshape(self.n, -1).to(torch.float64)
        sol = torch.cholesky_solve(self.X_aug.T @ R, self.L)
        return float(((R - self.X_aug @ sol) ** 2).sum())


def admit_pair(W_a: torch.Tensor, b_a: torch.Tensor, W_b: torch.Tensor, b_b: torch.Tensor,
               tau: float = 0.5, eps: float = 0.0) -> tuple[bool, float, torch.Tensor, torch.Tensor]:
    """Cross-seed gate: admitted iff cos(W_a, W_b) > tau and both norms > eps;
    returns (admitted, cos, (W_a + W_b) / 2, (b_a + b_b) / 2)."""
    wa, wb = W_a.flatten().double(), W_b.flatten().double()
    na, nb = float(wa.norm()), float(wb.norm())
    cos = float(wa @ wb) / (na * nb) if na > 0 and nb > 0 else 0.0
    ok = cos > tau and min(na, nb) > eps
    return ok, cos, (W_a + W_b) / 2, (b_a + b_b) / 2


def save_comp_state(path: str, blocks: dict, **meta) -> None:
    """``blocks``: {block index: {"W": [D_in, D_out], "b": [D_out],
    "enabled": bool, optional "cos_ab": float}}."""
    rec = {"format": COMP_FORMAT, "meta": meta, "blocks": {}}
    for i, e in blocks.items():
        rec["blocks"][int(i)] = {"W": e["W"].detach().float().cpu(),
                                 "b": e["b"].detach().float().cpu(),
                                 "enabled": bool(e.get("enabled", True)),
                                 "cos_ab": float(e.get("cos_ab", float("nan")))}
    torch.save(rec, path)


def load_comp_state(path: str) -> dict:
    rec = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(rec, dict) or rec.get("format") != COMP_FORMAT:
        raise ValueError(f"{path}: not a {COMP_FORMAT} file")
    for i, e in rec["blocks"].items():
        W, b = e["W"], e["b"]
        if W.dim() != 2 or b.shape != (W.shape[1],):
            raise ValueError(f"{path}: block {i} has W {tuple(W.shape)} and b {tuple(b.shape)}")
    return rec


def _block_list(model: nn.Module) -> nn.ModuleList:
    if hasattr(model, "backbone") and hasattr(model.backbone, "blocks"):
        return model.backbone.blocks
    if hasattr(model, "blocks"):
        return model.blocks
    raise RuntimeError("cannot find transformer blocks (model.backbone.blocks or model.blocks)")


def install_compensation(model: nn.Module, state: dict, factory: Callable,
                         device: Optional[torch.device] = None) -> list[int]:
    """Wrap every admitted block of ``model`` in a ``CompensationBlock`` whose
    comp is ``factory(W̄, b̄)``; returns the wrapped block indices."""
    blocks = _block_list(model)
    dev = device if device is not None else next(model.parameters()).device
    done = []
    for i, e in sorted(state["blocks"].items()):
        if not e["enabled"]:
            continue
        if i >= len(blocks):
            raise ValueError(f"comp state has block {i}, model has {len(blocks)}")
        blk = blocks[i]
        inner = blk.block if isinstance(blk, CompensationBlock) else blk
        blocks[i] = CompensationBlock(inner, factory(e["W"].to(dev), e["b"].to(dev)))
        done.append(i)
    return done
