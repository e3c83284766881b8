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
        x2 = x.reshape(-1, D_in).float()
        if USE_NOISE_MODEL:
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
        y = sc_matmul(x2, self.weight.float(), granularity="per_row", mode=self.mode,
                      sc_prec=self.sc_prec, config=cfg, k_segment=self.D_head,
                      bias=self.bias)
        return y.to(x.dtype).reshape(*orig_shape[:-1], D_out)
