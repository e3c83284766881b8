"""HeadAlignedSCLinear -- the compensation linear split per attention head
(mirror of the reference's ``sc_integration/head_aligned_comp.py``).

``D_in`` is split into ``n_heads`` chunks of ``D_head``; chunk ``h`` is an SC
matmul ``x[:, h] @ W[:, h]^T`` that draws on the ``(D_head, sc_prec)`` pool
(the pool the block's per-head Q@K^T uses), the fp32 partials are summed in
head order, then the bias is added (``head_aligned_comp.py:94-144``).

The reference runs the heads as ``n_heads`` Triton launches on ``n_heads``
CUDA streams.  Here all heads are one engine launch: ``k_segment = D_head``
makes each head a segment with its own per-row quantisation and rescale,
and the segment results are summed in head order inside the kernel, which
is the same fp32 sequence as the reference's ``y = y + partials[h]`` loop.
"""
from __future__ import annotations

import torch
import torch.nn as nn


class HeadAlignedSCLinear(nn.Module):
    def __init__(self, linear: nn.Linear, sc_prec: int, mode: str = "bipolar",
                 n_heads: int = 16, cfg_override: dict | None = None, use_streams: bool = True):
        super().__init__()
        D_in = linear.weight.shape[1]
        D_out = linear.weight.shape[0]
        if D_in % n_heads:
            raise AssertionError(f"D_in={D_in} must be divisible by n_heads={n_heads}")
        self.weight = linear.weight
        self.bias = linear.bias
        self.sc_prec = sc_prec
        self.mode = mode
        self.n_heads = n_heads
        self.D_head = D_in // n_heads
        self.in_features = D_in
        self.out_features = D_out
        self.cfg_override = cfg_override
        self.use_streams = use_streams  # kept for API fidelity; one launch covers every head

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .sc_linear import USE_NOISE_MODEL, _get_config, _sc_linear
        from .sc import sc_matmul

        orig_shape = x.shape
        D_in = orig_shape[-1]
        D_out = self.weight.shape[0]
        if USE_NOISE_MODEL:
            x2 = x.reshape(-1, D_in).float()
            y = torch.zeros(x2.shape[0], D_out, device=x.device, dtype=torch.float32)
            for h in range(self.n_heads):
                sl = slice(h * self.D_head, (h + 1) * self.D_head)
                y = y + _sc_linear(x2[:, sl].contiguous(), self.weight[:, sl].contiguous(), None,
                                   self.sc_prec, mode=self.mode, cfg_override=self.cfg_override)
            if self.bias is not None:
                y = y + self.bias.float()
            return y.to(x.dtype).reshape(*orig_shape[:-1], D_out)
        cfg = self.cfg_override if self.cfg_override is not None else _get_config(
            self.D_head, self.sc_prec)
        x2 = x.reshape(-1, D_in)
        if x2.dtype not in (torch.float32, torch.bfloat16):
            x2 = x2.float()
        b = self._packed_weight(cfg) if self._prepack_applies() else self.weight
        y = sc_matmul(x2, b, granularity="per_row", mode=self.mode, sc_prec=self.sc_prec,
                      config=cfg, k_segment=self.D_head, bias=self.bias)
        return y.to(x.dtype).reshape(*orig_shape[:-1], D_out)

    def _prepack_applies(self) -> bool:
        """Whether the weight is packed once for segmented calls (its operand
        bytes then reach the e2m1 pair tiles by TMA instead of being generated
        in every call; bit-identical either way).  Only when forced with
        ``sc_linear.set_weight_prepack(True)``: on B200 the one-accumulator
        segmented tiles ran slower with TMA-fed b (the compensation at 512
        images: 30.5 vs 26.1 ms), their L2 reads of the packed bytes being
        twice those of the two-accumulator linears per multiply-add."""
        from . import sc_linear
        if sc_linear._PREPACK is not True or not self.weight.is_cuda:
            return False
        if self.sc_prec not in (7, 8) or (self.mode == "unipolar" and self.sc_prec == 8):
            return False
        return self.D_head % 8 == 0 and self.D_head < self.in_features

    def _packed_weight(self, cfg: dict):
        """The weight's segmented prepacked operand (cached; rebuilt when the
        weight's storage, version counter or the SC settings change)."""
        from .sc import prepack_b
        w = self.weight
        key = (w.data_ptr(), w._version, w.dtype, str(w.device), self.sc_prec, self.mode,
               cfg["uid"])
        if key != getattr(self, "_packed_key", None):
            self._packed = None  # free the old buffer before building the new one
            self._packed = prepack_b(w.detach(), granularity="per_row", mode=self.mode,
                                     sc_prec=self.sc_prec, config=cfg, k_segment=self.D_head)
            self._packed_key = key
        return self._packed
