"""Mixed-precision (MP) stream-length maps -- the ``scmp_kernels.mp`` surface.

The reference imports these names from its un-vendored kernel package
(``sc_integration/mp_linear.py:37-48``, ``sc_integration/mp_config.py:7-17``,
``cls/sc_attention_patch.py:29-34``, ``det/sc_patch/sc_matmul.py:38-41``).
Their behaviour is fixed here by the reference's own smoke tests and
docstrings:

* fixed MP is a sort-based quantile split, higher metric -> longer stream,
  exact up to count rounding (``experiments/custom_fractions_smoke.py:1-7``,
  ``sc_integration/mp_linear.py:5-9``);
* free-boundary MP splits the min-max normalised metric at per-(op, block)
  boundaries, default equal spacing, a flat metric going wholly to the top
  level (``experiments/test_free_boundary_classifier.py:24-70``);
* adaptive MP is timestep-aware, ``theta = alpha * t / max(T-1, 1) + beta``
  (``sc_integration/mp_linear.py:130-147``), or a quantile split when
  ``target_fractions`` is given (``experiments/custom_fractions_smoke.py``).

Every classifier also returns the per-row level as a device tensor
(``RowAssignment.row_levels``) so the engine can run all levels in one
launch without host synchronisation; ``level_row_indices`` is materialised
only when a caller asks for it.
"""
from __future__ import annotations

import math
import threading
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

__all__ = [
    "MPConfig", "AdaptiveMPConfig", "RangeMPConfig", "FreeBoundaryMPConfig", "RowAssignment",
    "classify_rows_by_metric", "adaptive_classify_rows", "classify_groups_by_range",
    "set_current_block_idx", "get_current_block_idx", "AutoMPBudgetLogger",
    "MPDistributionLogger", "MetricProfiler", "quantile_levels_batched", "SeededRandomMPConfig",
    "quantile_counts",
]

_BLOCK = threading.local()


def set_current_block_idx(idx: int) -> None:
    _BLOCK.idx = int(idx)


def get_current_block_idx() -> int:
    return getattr(_BLOCK, "idx", 0)


# ------------------------------------------------------------------ configs

@dataclass
class MPConfig:
    """Fixed-quantile per-row MP: ``level_fractions[i]`` of the rows (highest
    metric first) get the i-th longest stream.  ``None`` = equal split."""
    stoc_len_levels: List[int]
    level_fractions: Optional[List[float]] = None

    def __post_init__(self):
        self.stoc_len_levels = [int(v) for v in self.stoc_len_levels]
        if not self.stoc_len_levels:
            raise ValueError("stoc_len_levels must be non-empty")
        if self.level_fractions is not None:
            self.level_fractions = [float(f) for f in self.level_fractions]
            if len(self.level_fractions) != len(self.stoc_len_levels):
                raise ValueError("level_fractions must match stoc_len_levels")
            if any(f < 0 for f in self.level_fractions):
                raise ValueError("level_fractions must be non-negative")


@dataclass
class AdaptiveMPConfig:
    """Timestep-aware per-row MP (see module docstring)."""
    stoc_len_levels: List[int]
    alpha: float = 0.3
    beta: float = 0.05
    enable_pruning: bool = False
    target_fractions: Optional[List[float]] = None
    operator_params: Dict[str, tuple] = field(default_factory=dict)

    def __post_init__(self):
        self.stoc_len_levels = [int(v) for v in self.stoc_len_levels]
        if self.target_fractions is not None:
            self.target_fractions = [float(f) for f in self.target_fractions]
            if len(self.target_fractions) != len(self.stoc_len_levels):
                raise ValueError("target_fractions must match stoc_len_levels")

    def params_for(self, operator: Optional[str]) -> tuple:
        if operator is not None and operator in self.operator_params:
            a, b = self.operator_params[operator]
            return float(a), float(b)
        return float(self.alpha), float(self.beta)


@dataclass
class RangeMPConfig:
    """Static per-weight-row-group MP from the group's (max - min) range.
    A group whose normalised range is >= ``base_threshold / 2**i`` (first i
    that matches) gets the i-th longest level; the rest get the shortest."""
    stoc_len_levels: List[int]
    base_threshold: float = 0.3
    operator_thresholds: Dict[str, float] = field(default_factory=dict)

    def __post_init__(self):
        self.stoc_len_levels = [int(v) for v in self.stoc_len_levels]

    def threshold_for(self, operator: Optional[str]) -> float:
        if operator is not None and operator in self.operator_thresholds:
            return float(self.operator_thresholds[operator])
        return float(self.base_threshold)


class FreeBoundaryMPConfig:
    """Per-(operator, block) boundaries on the normalised metric; unset pairs
    use equal spacing ``(n-1-i)/n``."""

    def __init__(self, stoc_len_levels: Sequence[int]):
        self.stoc_len_levels = [int(v) for v in stoc_len_levels]
        self._bounds: Dict[tuple, torch.Tensor] = {}

    def default_boundaries(self) -> torch.Tensor:
        n = len(self.stoc_len_levels)
        return torch.tensor([(n - 1 - i) / n for i in range(n - 1)], dtype=torch.float32)

    def set_boundaries(self, operator: str, block_idx: int, boundaries) -> None:
        b = torch.as_tensor(boundaries, dtype=torch.float32).flatten().cpu()
        if b.numel() != len(self.stoc_len_levels) - 1:
            raise ValueError(f"need {len(self.stoc_len_levels) - 1} boundaries")
        self._bounds[(operator, int(block_idx))] = b

    def get_boundaries(self, operator: Optional[str], block_idx: int) -> torch.Tensor:
        return self._bounds.get((operator, int(block_idx)), self.default_boundaries())


# --------------------------------------------------------------- assignment

class RowAssignment:
    """Result of a classifier: ``row_levels[r]`` is the stream length of row
    ``r`` (device tensor); ``level_row_indices`` maps every level to the
    ascending LongTensor of its rows (built lazily, needs a host sync)."""

    def __init__(self, row_levels: torch.Tensor, levels: Sequence[int],
                 host_counts: Optional[Dict[int, int]] = None):
        self.row_levels = row_levels
        self.levels = [int(v) for v in levels]
        # rows per level when the split fixes them without looking at the
        # data (quantile splits); None when only the device knows
        self.host_counts = host_counts
        self._idx: Optional[Dict[int, torch.Tensor]] = None

    @property
    def level_row_indices(self) -> Dict[int, torch.Tensor]:
        if self._idx is None:
            self._idx = {sl: torch.nonzero(self.row_levels == sl, as_tuple=False).squeeze(-1)
                         for sl in self.levels}
        return self._idx

    def counts(self) -> Dict[int, int]:
        return {sl: int(idx.numel()) for sl, idx in self.level_row_indices.items()}


def _sorted_levels(levels, fracs):
    pairs = sorted(zip(levels, fracs), key=lambda p: -p[0])
    return [p[0] for p in pairs], [p[1] for p in pairs]


def _quantile_split(metric: torch.Tensor, levels, fractions) -> RowAssignment:
    metric = metric.detach().float().flatten()
    n = metric.numel()
    if fractions is None:
        fractions = [1.0 / len(levels)] * len(levels)
    total = float(sum(fractions)) or 1.0
    lv, fr = _sorted_levels(list(levels), [f / total for f in fractions])
    counts = [int(round(f * n)) for f in fr[:-1]]
    used = 0
    for i, c in enumerate(counts):
        counts[i] = max(0, min(c, n - used))
        used += counts[i]
    counts.append(n - used)
    order = torch.sort(metric, descending=True, stable=True).indices
    row_levels = torch.empty(n, dtype=torch.int32, device=metric.device)
    start = 0
    host = {}
    for L, c in zip(lv, counts):
        if c:
            row_levels[order[start:start + c]] = L
        host[L] = host.get(L, 0) + c
        start += c
    return RowAssignment(row_levels, lv, host_counts=host)


def _normalise(metric: torch.Tensor) -> torch.Tensor:
    m = metric.detach().float().flatten()
    lo, hi = m.min(), m.max()
    rng = hi - lo
    return torch.where(rng > 0, (m - lo) / torch.where(rng > 0, rng, torch.ones_like(rng)),
                       torch.ones_like(m))


def _boundary_split(metric: torch.Tensor, levels, boundaries: torch.Tensor) -> RowAssignment:
    lv = sorted(levels, reverse=True)
    mn = _normalise(metric)
    b = boundaries.to(device=mn.device, dtype=torch.float32)
    # level index = number of boundaries the row falls below (first match wins)
    idx = (mn[:, None] < b[None, :]).sum(dim=1)
    lut = torch.tensor(lv, dtype=torch.int32, device=mn.device)
    return RowAssignment(lut[idx.clamp(max=len(lv) - 1)], lv)


def classify_rows_by_metric(metric: torch.Tensor, stoc_len_levels, level_fractions=None
                            ) -> RowAssignment:
    """Fixed-quantile split (higher metric -> longer stream)."""
    return _quantile_split(metric, stoc_len_levels, level_fractions)


def quantile_counts(n: int, levels, fractions=None) -> Dict[int, int]:
    """Rows per level of a quantile split of ``n`` rows (host-side)."""
    if fractions is None:
        fractions = [1.0 / len(levels)] * len(levels)
    total = float(sum(fractions)) or 1.0
    lv, fr = _sorted_levels(list(levels), [f / total for f in fractions])
    counts = [int(round(f * n)) for f in fr[:-1]]
    used = 0
    for i, c in enumerate(counts):
        counts[i] = max(0, min(c, n - used))
        used += counts[i]
    counts.append(n - used)
    out: Dict[int, int] = {}
    for L, c in zip(lv, counts):
        out[L] = out.get(L, 0) + c
    return out


def quantile_levels_batched(metric: torch.Tensor, levels, fractions=None) -> torch.Tensor:
    """Row-wise ``classify_rows_by_metric`` over the last dim of ``metric``
    ``[S, N]`` (one independent split per slice, e.g. per (batch, head));
    returns int32 levels ``[S, N]`` without host synchronisation."""
    S, n = metric.shape
    if fractions is None:
        fractions = [1.0 / len(levels)] * len(levels)
    total = float(sum(fractions)) or 1.0
    lv, fr = _sorted_levels(list(levels), [f / total for f in fractions])
    counts = [int(round(f * n)) for f in fr[:-1]]
    used = 0
    for i, c in enumerate(counts):
        counts[i] = max(0, min(c, n - used))
        used += counts[i]
    counts.append(n - used)
    by_rank = torch.empty(n, dtype=torch.int32, device=metric.device)
    start = 0
    for L, c in zip(lv, counts):
        by_rank[start:start + c] = L
        start += c
    order = torch.sort(metric.float(), dim=-1, descending=True, stable=True).indices
    out = torch.empty(S, n, dtype=torch.int32, device=metric.device)
    out.scatter_(1, order, by_rank.unsqueeze(0).expand(S, n).contiguous())
    return out


@dataclass
class SeededRandomMPConfig:
    """Per-row levels drawn at random with fixed fractions (a seeded random
    permutation per call site); an assignment that does not look at the
    data, for throughput studies of mixed stream lengths."""
    stoc_len_levels: List[int]
    level_fractions: Optional[List[float]] = None
    seed: int = 0

    def assign(self, n_rows: int, device, salt: int = 0) -> torch.Tensor:
        g = torch.Generator(device="cpu").manual_seed((int(self.seed) << 20) ^ int(salt))
        metric = torch.rand(n_rows, generator=g).to(device)
        return _quantile_split(metric, self.stoc_len_levels, self.level_fractions).row_levels


def adaptive_classify_rows(metric: torch.Tensor, timestep: int, total_timesteps: int, config,
                           operator: Optional[str] = None) -> RowAssignment:
    """Free-boundary or timestep-aware adaptive split (see module docstring)."""
    if isinstance(config, FreeBoundaryMPConfig):
        bounds = config.get_boundaries(operator, get_current_block_idx())
        return _boundary_split(metric, config.stoc_len_levels, bounds)
    if not isinstance(config, AdaptiveMPConfig):
        raise TypeError(f"unsupported adaptive config {type(config).__name__}")
    if config.target_fractions is not None:
        return _quantile_split(metric, config.stoc_len_levels, config.target_fractions)
    alpha, beta = config.params_for(operator)
    progress = float(timestep) / max(int(total_timesteps) - 1, 1)
    theta = min(max(alpha * progress + beta, 0.0), 1.0)
    n = len(config.stoc_len_levels)
    bounds = torch.tensor([theta + (1.0 - theta) * (n - 1 - i) / n for i in range(n - 1)],
                          dtype=torch.float32)
    return _boundary_split(metric, config.stoc_len_levels, bounds)


def classify_groups_by_range(weight: torch.Tensor, group_size: int, config: RangeMPConfig,
                             operator: Optional[str] = None) -> List[int]:
    """Stream length per contiguous group of ``group_size`` weight rows."""
    W = weight.detach().float()
    out_features = W.shape[0]
    g = int(group_size) if 0 < int(group_size) <= out_features else out_features
    ng = out_features // g
    Wg = W[: ng * g].reshape(ng, g * W.shape[1])
    rng = (Wg.max(dim=1).values - Wg.min(dim=1).values).cpu()
    top = float(rng.max()) if ng else 0.0
    norm = rng / top if top > 0 else torch.ones_like(rng)
    lv = sorted(config.stoc_len_levels, reverse=True)
    thr = config.threshold_for(operator)
    out = []
    for v in norm.tolist():
        level = lv[-1]
        for i, L in enumerate(lv[:-1]):
            if v >= thr / (2 ** i):
                level = L
                break
        out.append(int(level))
    return out


# ------------------------------------------------------------------ loggers

class AutoMPBudgetLogger:
    """Accumulates (baseline, actual) SC bit-op budgets per (block, op)
    (reference ``sc_integration/sc_linear.py:237-251``)."""
    _lock = threading.Lock()
    _data: Dict[tuple, List[float]] = defaultdict(lambda: [0.0, 0.0, 0])
    enabled = True

    @classmethod
    def record(cls, block_idx, operator, compute_baseline, compute_actual) -> None:
        if not cls.enabled:
            return
        # Tensors stay on their device (no host sync); summary() reads them.
        with cls._lock:
            rec = cls._data[(int(block_idx), str(operator))]
            rec[0] = rec[0] + compute_baseline
            rec[1] = rec[1] + compute_actual
            rec[2] += 1

    @classmethod
    def summary(cls) -> Dict[tuple, dict]:
        with cls._lock:
            out = {}
            for k, v in cls._data.items():
                base, act = float(v[0]), float(v[1])
                out[k] = {"baseline": base, "actual": act, "calls": v[2],
                          "ratio": (act / base) if base else math.nan}
            return out

    @classmethod
    def reset(cls) -> None:
        with cls._lock:
            cls._data.clear()


class MPDistributionLogger:
    """Per (timestep, block, op) level histograms."""
    enabled = False
    _data: Dict[tuple, Dict[int, int]] = defaultdict(lambda: defaultdict(int))
    _compute: Dict[tuple, List[float]] = defaultdict(lambda: [0.0, 0.0])

    @classmethod
    def log(cls, timestep, block_idx, operator, assignment: RowAssignment, n_rows) -> None:
        if not cls.enabled:
            return
        h = cls._data[(timestep, block_idx, operator)]
        for sl, c in assignment.counts().items():
            h[sl] += c

    @classmethod
    def log_compute(cls, timestep, block_idx, operator, baseline, actual) -> None:
        if not cls.enabled:
            return
        rec = cls._compute[(timestep, block_idx, operator)]
        rec[0] += float(baseline)
        rec[1] += float(actual)

    @classmethod
    def reset(cls) -> None:
        cls._data.clear()
        cls._compute.clear()


class MetricProfiler:
    """Keeps per (timestep, block, op) metric summaries (min/mean/max)."""
    enabled = False
    _data: Dict[tuple, List[tuple]] = defaultdict(list)

    @classmethod
    def record(cls, metric: torch.Tensor, timestep, block_idx, operator) -> None:
        if not cls.enabled:
            return
        m = metric.detach().float()
        cls._data[(timestep, block_idx, operator)].append(
            (float(m.min()), float(m.mean()), float(m.max())))

    @classmethod
    def reset(cls) -> None:
        cls._data.clear()


def __getattr__(name):
    # ``from scmp_kernels.mp import RidgeFitter`` (sc_integration/mp_search.py:49):
    # the ridge solve lives with the QwT compensation code
    if name == "RidgeFitter":
        from .qwt import RidgeFitter
        return RidgeFitter
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
