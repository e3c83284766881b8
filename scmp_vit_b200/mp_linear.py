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
    """Static per-output-row stream lengths of a weight (range MP).

    The output rows form contiguous groups of ``group_size`` (the whole weight
    when 0 or too large); ``classify_groups_by_range`` gives each group a level
    from its value range.  Every output row inherits its group's level in one
    ``repeat_interleave``, and one entry per distinct level (in order of first
    appearance) holds that level's rows and their weight slice, so a forward
    runs one bucket per level instead of one per group.  Rows past the last
    whole group belong to no entry, as in the reference
    (``sc_integration/mp_linear.py:81-119``)."""
    n_out = weight.shape[0]
    size = group_size if 0 < group_size < n_out else n_out
    n_groups = n_out // size
    levels = torch.as_tensor([int(v) for v in classify_groups_by_range(
        weight, group_size=size, config=cfg, operator=operator)], dtype=torch.long)
    if levels.numel() != n_groups:
        raise AssertionError(f"classify_groups_by_range returned {levels.numel()} levels for "
                             f"{n_groups} groups")
    row_level = levels.repeat_interleave(size).to(weight.device)  # level of row r < n_groups*size
    entries: List[DispatchEntry] = []
    for level in dict.fromkeys(levels.tolist()):
        rows = torch.nonzero(row_level == level).flatten()
        entries.append(DispatchEntry(stoc_len=level, sc_prec=sc_prec_for_stoc_len(level),
                                     weight=weight.index_select(0, rows).contiguous(),
                                     out_indices=rows))
    return entries


def _row_absmax(x_flat: torch.Tensor) -> torch.Tensor:
    """The input-row MP metric: the largest magnitude of each row (fp32)."""
    return torch.linalg.vector_norm(x_flat.float(), ord=float("inf"), dim=-1)


def classify_input_rows(x_flat: torch.Tensor, cfg: MPConfig) -> RowAssignment:
    """Fixed-quantile MP levels of activation rows, ranked by ``_row_absmax``
    (reference ``sc_integration/mp_linear.py:122-127``)."""
    return classify_rows_by_metric(_row_absmax(x_flat), cfg.stoc_len_levels,
                                   cfg.level_fractions)


def classify_input_rows_adaptive(x_flat: torch.Tensor, cfg: AdaptiveMPConfig, timestep: int,
                                 total_timesteps: int, operator: Optional[str] = None
                                 ) -> RowAssignment:
    """Timestep-aware MP levels of activation rows, same metric
    (reference ``sc_integration/mp_linear.py:130-147``)."""
    return adaptive_classify_rows(_row_absmax(x_flat), timestep, total_timesteps, cfg,
                                  operator=operator)
