"""Mixed-precision helpers for SC linears (mirror of the reference's
``sc_integration/mp_linear.py``).

* fixed / adaptive MP classify *input rows* by per-row abs-max
  (``mp_linear.py:122-147``);
* range MP classifies *output row groups* of the weight by (max - min) and
  bakes ``DispatchEntry`` buckets once (``mp_linear.py:81-119``);
* combined, a (row, output-group) pair uses ``min(row_sl, group_sl)``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch

from .mp import (  # noqa: F401  (re-exported, as the reference does)
    AdaptiveMPConfig,
    FreeBoundaryMPConfig,
    MPConfig,
    RangeMPConfig,
    RowAssignment,
    adaptive_classify_rows,
    classify_groups_by_range,
    classify_rows_by_metric,
    get_current_block_idx,
    set_current_block_idx,
)

__all__ = [
    "MPConfig", "RangeMPConfig", "AdaptiveMPConfig", "FreeBoundaryMPConfig", "DispatchEntry",
    "build_range_dispatch", "classify_input_rows", "classify_input_rows_adaptive",
    "sc_prec_for_stoc_len", "set_current_block_idx", "get_current_block_idx",
]


def sc_prec_for_stoc_len(stoc_len: int) -> int:
    """Smallest ``sc_prec`` with ``2**sc_prec >= stoc_len`` (reference
    ``mp_linear.py:65-69``)."""
    if stoc_len <= 1:
        return 1
    return int(math.ceil(math.log2(stoc_len)))


@dataclass
class DispatchEntry:
    """One (stoc_len, weight-slice, output-indices) bucket."""
    stoc_len: int
    sc_prec: int
    weight: torch.Tensor       # (n_out_in_bucket, D_in), contiguous
    out_indices: torch.Tensor  # LongTensor of output rows in the full weight


def build_range_dispatch(weight: torch.Tensor, cfg: RangeMPConfig,
                         operator: Optional[str] = None, group_size: int = 0
                         ) -> List[DispatchEntry]:
    """Split the weight's output rows into contiguous groups, classify each
    by range, and merge groups that share a level into one entry."""
    out_features = weight.shape[0]
    g = group_size if 0 < group_size < out_features else out_features
    num_groups = out_features // g
    group_sls = classify_groups_by_range(weight, group_size=g, config=cfg, operator=operator)
    if len(group_sls) != num_groups:
        raise AssertionError(f"classify_groups_by_range returned {len(group_sls)} levels for "
                             f"{num_groups} groups")
    by_level: dict[int, list[int]] = {}
    for gi, sl in enumerate(group_sls):
        by_level.setdefault(int(sl), []).extend(range(gi * g, (gi + 1) * g))
    entries = []
    for sl, rows in by_level.items():
        idx = torch.as_tensor(rows, dtype=torch.long, device=weight.device)
        entries.append(DispatchEntry(stoc_len=int(sl), sc_prec=sc_prec_for_stoc_len(int(sl)),
                                     weight=weight.index_select(0, idx).contiguous(),
                                     out_indices=idx))
    return entries


def classify_input_rows(x_flat: torch.Tensor, cfg: MPConfig) -> RowAssignment:
    """Bucket activation rows by abs-max into MP levels."""
    metric = x_flat.float().abs().amax(dim=-1)
    return classify_rows_by_metric(metric, cfg.stoc_len_levels, cfg.level_fractions)


def classify_input_rows_adaptive(x_flat: torch.Tensor, cfg: AdaptiveMPConfig, timestep: int,
                                 total_timesteps: int, operator: Optional[str] = None
                                 ) -> RowAssignment:
    """Timestep-aware per-row classification (same abs-max metric)."""
    metric = x_flat.float().abs().amax(dim=-1)
    return adaptive_classify_rows(metric, timestep, total_timesteps, cfg, operator=operator)
