"""SCLinear and helpers (mirror of the reference's ``sc_integration/sc_linear.py``).

Same public surface (``sc_linear.py:7-16``): ``SCLinear``, ``set_noise_model``,
``USE_NOISE_MODEL``, ``set_vit_timestep`` / ``get_vit_timestep``,
``_sc_linear``, ``_sc_linear_mp``, ``_mm_one_bucket``, ``_get_config``,
``_CFG_CACHE``.  What changes is the execution of mixed precision: the
reference launches one kernel per distinct stream length, with
``unique().tolist()`` / ``nonzero`` host syncs in between
(``sc_linear.py:253-284``).  Here a classifier returns the per-row level as
a device tensor and every level that shares a precision runs in one grouped
launch (``row_stoc_len``); levels at another precision (e.g. L=128 at p=7
next to L=256 at p=8) take one more launch.  Each row's result is the same
as the reference's per-bucket call, because per-row quantisation makes rows
independent.
"""
from __future__ import annotations

from typing import Callable, Iterable, Optional

import torch
import torch.nn as nn

from . import noise_matmul
from .config_helpers import make_sobol_simple_config
from .mp import AutoMPBudgetLogger
from .mp_linear import (
    AdaptiveMPConfig,
    DispatchEntry,
    MPConfig,
    RangeMPConfig,
    build_range_dispatch,
    classify_input_rows,
    classify_input_rows_adaptive,
    get_current_block_idx,
    sc_prec_for_stoc_len,
)
from .sc import sc_matmul

__all__ = ["SCLinear", "set_noise_model", "set_vit_timestep", "get_vit_timestep",
           "_sc_linear", "_sc_linear_mp", "_mm_one_bucket", "_get_config", "_CFG_CACHE",
           "sc_linear_rows", "PackedWeights"]

# Read at call time through the module (``sc_linear.USE_NOISE_MODEL``).
USE_NOISE_MODEL = False


def set_noise_model(enabled: bool):
    global USE_NOISE_MODEL
    USE_NOISE_MODEL = bool(enabled)


_VIT_TIMESTEP: int = 0
_VIT_TOTAL_TIMESTEPS: int = 1


def set_vit_timestep(t: int, total: int | None = None):
    """External (t, T) for adaptive MP in callers without a diffusion step."""
    global _VIT_TIMESTEP, _VIT_TOTAL_TIMESTEPS
    _VIT_TIMESTEP = int(t)
    if total is not None:
        _VIT_TOTAL_TIMESTEPS = max(int(total), 1)


def get_vit_timestep() -> tuple[int, int]:
    return _VIT_TIMESTEP, _VIT_TOTAL_TIMESTEPS


_CFG_CACHE: dict = {}


def _get_config(D, sc_prec):
    """``(D, sc_prec)`` pool, created on first use (creation order matters:
    the scramble shifts come from Python's ``random``)."""
    key = (D, sc_prec)
    if key not in _CFG_CACHE:
        _CFG_CACHE[key] = make_sobol_simple_config(D, D, sc_prec)
    return _CFG_CACHE[key]


def _sc_linear(x: torch.Tensor, weight: torch.Tensor, bias, sc_prec: int,
               mode: str = "bipolar", cfg_override: dict = None,
               stoc_len: int | None = None, chunk_d: int = 0, packed=None):
    """``y = x @ weight^T + bias`` via SC; per-row scales for x and weight
    rows.  Bias is added in the engine's epilogue (same fp32 add)."""
    orig_shape = x.shape
    D_in = orig_shape[-1]
    # bf16 operands go to the engine as they are (widening is exact) and the
    # engine writes bf16: fp32 result + fp32 bias, rounded to nearest even --
    # the values of the fp32 path followed by .to(bfloat16)
    bf16 = x.dtype == torch.bfloat16 and not USE_NOISE_MODEL
    x2 = x.reshape(-1, D_in) if bf16 else x.reshape(-1, D_in).float()
    w = weight if bf16 and weight.dtype == torch.bfloat16 else weight.float()
    odt = torch.bfloat16 if bf16 else None
    if USE_NOISE_MODEL:
        y = noise_matmul.noisy_sc_matmul_grouped(x2, w, group_a=1, group_b=1, mode=mode,
                                                 sc_prec=sc_prec, stoc_len=stoc_len)
        if bias is not None:
            y = y + bias.float()
    elif chunk_d > 0 and mode == "bipolar" and D_in > chunk_d and cfg_override is None:
        y = sc_matmul(x2, w, granularity="per_row", mode=mode, sc_prec=sc_prec,
                      config=_get_config(chunk_d, sc_prec), group_a=1, group_b=1,
                      chunk_d=chunk_d, stoc_len=stoc_len, bias=bias, out_dtype=odt)
    else:
        cfg = cfg_override if cfg_override is not None else _get_config(D_in, sc_prec)
        y = sc_matmul(x2, packed if packed is not None else w, granularity="per_row", group_a=1,
                      group_b=1, mode=mode, sc_prec=sc_prec, config=cfg, stoc_len=stoc_len,
                      bias=bias, out_dtype=odt)
    return y.to(x.dtype).reshape(*orig_shape[:-1], w.shape[0])


def _mm_one_bucket(x_sub: torch.Tensor, w_sub: torch.Tensor, stoc_len: int, sc_prec: int,
                   mode: str, chunk_d: int = 0) -> torch.Tensor:
    """One SC matmul at a chosen ``stoc_len`` (noise surrogate when enabled)."""
    if USE_NOISE_MODEL:
        return noise_matmul.noisy_sc_matmul_grouped(x_sub, w_sub, group_a=1, group_b=1,
                                                    mode=mode, sc_prec=sc_prec,
                                                    stoc_len=stoc_len)
    D_in = x_sub.shape[-1]
    if chunk_d > 0 and mode == "bipolar" and D_in > chunk_d:
        return sc_matmul(x_sub, w_sub, granularity="per_row", mode=mode, sc_prec=sc_prec,
                         config=_get_config(chunk_d, sc_prec), group_a=1, group_b=1,
                         chunk_d=chunk_d, stoc_len=stoc_len)
    return sc_matmul(x_sub, w_sub, granularity="per_row", group_a=1, group_b=1, mode=mode,
                     sc_prec=sc_prec, config=_get_config(D_in, sc_prec), stoc_len=stoc_len)


def sc_linear_rows(x2: torch.Tensor, w: torch.Tensor, row_L: torch.Tensor,
                   levels: Iterable[int], mode: str, *, bias: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None, chunk_d: int = 0,
                   cfg_for: Optional[Callable[[int, int], dict]] = None,
                   host_counts: Optional[dict] = None,
                   packed_for: Optional[Callable[[int, dict], object]] = None) -> torch.Tensor:
    """Per-row stream lengths in grouped launches: one engine call per
    distinct precision among ``levels`` (the host-known set of values that
    ``row_L`` may hold; 0 = pruned row -> bias only).

    With ``host_counts`` (rows per level, known without a device sync for
    quantile splits) the rows are sorted by level once and every call runs
    on its own contiguous rows only, one call per level; otherwise every call spans all rows and
    skips the others (``row_stoc_len = -1``).  ``packed_for(p, config)``, if
    given, returns the weight prepacked for precision ``p`` (or None): the
    per-row calls then load its operand bytes instead of generating them."""
    M, K = x2.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=x2.device)
    cfg_for = cfg_for or _get_config
    by_prec: dict[int, list[int]] = {}
    for L in sorted({int(v) for v in levels if int(v) > 0}):
        by_prec.setdefault(sc_prec_for_stoc_len(L), []).append(L)
    if not by_prec:
        out.zero_()
        if bias is not None:
            out += bias.float()
        return out
    row_L = row_L.to(torch.int32)
    use_chunk = chunk_d > 0 and mode == "bipolar" and K > chunk_d
    if host_counts is not None and len(by_prec) > 1:
        # rows ordered by level: pruned first, then each precision's levels
        order = torch.sort(row_L, stable=True).indices
        xs = x2.index_select(0, order)
        ys = torch.empty(M, N, dtype=torch.float32, device=x2.device)
        start = sum(c for L, c in host_counts.items() if int(L) <= 0)
        if start:
            ys[:start] = 0.0 if bias is None else bias.float()
        for p, Lset in by_prec.items():
            if sum(host_counts.get(L, 0) for L in Lset) == 0:
                continue
            cfg = cfg_for(chunk_d if use_chunk else K, p)
            b = _packed_or(w, packed_for, p, cfg, use_chunk)
            # one call per level: with a single stream length the engine runs
            # only the stream positions a window can reach (L = 192 at p = 8:
            # three quarters of each 256-position stage)
            for L in Lset:
                n_rows = host_counts.get(L, 0)
                if n_rows == 0:
                    continue
                sc_matmul(xs[start:start + n_rows], b, granularity="per_row", mode=mode,
                          sc_prec=p, config=cfg, chunk_d=chunk_d if use_chunk else 0, bias=bias,
                          stoc_len=L, out=ys[start:start + n_rows])
                start += n_rows
        out.index_copy_(0, order, ys)
        return out
    first = True
    for p, Ls in by_prec.items():
        mask = torch.zeros_like(row_L, dtype=torch.bool)
        for L in Ls:
            mask |= row_L == L
        if first:
            mask |= row_L <= 0  # the first launch writes the pruned rows
        sel = torch.where(mask, row_L.clamp(min=0), torch.full_like(row_L, -1))
        cfg = cfg_for(chunk_d if use_chunk else K, p)
        sc_matmul(x2, _packed_or(w, packed_for, p, cfg, use_chunk), granularity="per_row",
                  mode=mode, sc_prec=p, config=cfg, chunk_d=chunk_d if use_chunk else 0,
                  bias=bias, row_stoc_len=sel, out=out)
        first = False
    return out


def _packed_or(w, packed_for, p: int, cfg: dict, chunked: bool):
    """The prepacked weight for precision ``p`` if one applies, else ``w``."""
    if packed_for is None or chunked:
        return w
    pk = packed_for(p, cfg)
    return w if pk is None else pk


class PackedWeights:
    """A weight's prepacked SC operands, one per (precision, pool), rebuilt
    when the weight's storage or version counter changes (mixed-precision
    linears run one call per precision class, each of which can load packed
    bytes instead of generating them)."""

    def __init__(self, weight: torch.Tensor, mode: str):
        self.weight = weight
        self.mode = mode
        self._cache: dict = {}
        self._key = None

    def __call__(self, p: int, cfg: dict):
        if not _prepack_applies(self.weight, p, self.mode, None, 0):
            return None
        from .sc import prepack_b
        w = self.weight
        key = (w.data_ptr(), w._version, w.dtype, str(w.device))
        if key != self._key:
            self._cache.clear()
            self._key = key
        ck = (p, cfg["uid"])
        if ck not in self._cache:
            self._cache[ck] = prepack_b(w.detach(), granularity="per_row", mode=self.mode,
                                        sc_prec=p, config=cfg, group_b=1)
        return self._cache[ck]


def _record_budget(operator, row_L: torch.Tensor, M: int, D_out: int, max_sl: int):
    if operator is None or not AutoMPBudgetLogger.enabled:
        return
    actual = row_L.clamp(min=0).to(torch.float64).sum() * D_out
    AutoMPBudgetLogger.record(get_current_block_idx(), operator, M * D_out * max_sl, actual)


def _sc_linear_mp(x: torch.Tensor, weight: torch.Tensor, bias, sc_prec: int, mode: str,
                  range_entries: list[DispatchEntry] | None = None,
                  mp_cfg: MPConfig | None = None,
                  adaptive_mp_cfg: AdaptiveMPConfig | None = None,
                  operator: str | None = None, chunk_d: int = 0,
                  packed_for=None) -> torch.Tensor:
    """MP-aware SC linear (reference ``sc_linear.py:183-288``): per-row levels
    from fixed or adaptive MP (adaptive wins), per-output-group levels from
    range MP, ``min(row_sl, group_sl)`` when combined."""
    orig_shape = x.shape
    D_in = orig_shape[-1]
    x_flat = x.reshape(-1, D_in).float()
    w = weight.float()
    M, D_out = x_flat.shape[0], w.shape[0]
    if range_entries is None and mp_cfg is None and adaptive_mp_cfg is None:
        y = _mm_one_bucket(x_flat, w, 2 ** sc_prec, sc_prec, mode, chunk_d=chunk_d)
        if bias is not None:
            y = y + bias.float()
        return y.to(x.dtype).reshape(*orig_shape[:-1], D_out)

    if adaptive_mp_cfg is not None:
        t, T = get_vit_timestep()
        assign = classify_input_rows_adaptive(x_flat, adaptive_mp_cfg, t, T, operator=operator)
        levels = list(adaptive_mp_cfg.stoc_len_levels)
    elif mp_cfg is not None:
        assign = classify_input_rows(x_flat, mp_cfg)
        levels = list(mp_cfg.stoc_len_levels)
    else:
        assign = None
        levels = [2 ** sc_prec]
    row_L = (assign.row_levels if assign is not None
             else torch.full((M,), 2 ** sc_prec, dtype=torch.int32, device=x.device))
    if range_entries is None and assign is not None:
        _record_budget(operator, row_L, M, D_out, max(levels))

    if USE_NOISE_MODEL:
        result = torch.zeros(M, D_out, dtype=torch.float32, device=x.device)
        entries = range_entries or [DispatchEntry(2 ** 30, sc_prec, w,
                                                  torch.arange(D_out, device=x.device))]
        for e in entries:
            eff = torch.clamp(row_L, max=e.stoc_len)
            for sl in torch.unique(eff).tolist():
                if sl <= 0:
                    continue
                rows = torch.nonzero(eff == sl).squeeze(-1)
                sub = _mm_one_bucket(x_flat.index_select(0, rows), e.weight.float(), int(sl),
                                     sc_prec_for_stoc_len(int(sl)), mode, chunk_d=chunk_d)
                result[rows.unsqueeze(1), e.out_indices.unsqueeze(0)] = sub
        if bias is not None:
            result = result + bias.float()
        return result.to(x.dtype).reshape(*orig_shape[:-1], D_out)

    if range_entries is None:
        result = sc_linear_rows(x_flat, w, row_L, levels, mode, bias=bias, chunk_d=chunk_d,
                                host_counts=None if assign is None else assign.host_counts,
                                packed_for=packed_for)
    else:
        result = torch.empty(M, D_out, dtype=torch.float32, device=x.device)
        for e in range_entries:
            if e.stoc_len <= 0:
                result[:, e.out_indices] = 0.0 if bias is None else bias.float()[e.out_indices]
                continue
            eff = torch.clamp(row_L, max=e.stoc_len)
            eff_levels = {min(int(L), e.stoc_len) for L in levels}
            b_sub = None if bias is None else bias.float().index_select(0, e.out_indices)
            sub = sc_linear_rows(x_flat, e.weight.float(), eff, eff_levels, mode, bias=b_sub,
                                 chunk_d=chunk_d)
            result.index_copy_(1, e.out_indices, sub)
    return result.to(x.dtype).reshape(*orig_shape[:-1], D_out)


_PREPACK = None  # None: automatic (see set_weight_prepack)


def set_weight_prepack(enabled) -> None:
    """Whether ``SCLinear`` keeps its weight's SC operand bytes expanded once
    (``sc.prepack_b``) instead of regenerating them in every call.  Results
    are bit-identical either way; the cache is rebuilt when the weight
    changes.  ``None`` (the default) prepacks where it pays on B200: p = 7 or
    8 with more than 128 output features, whose packed bytes are e2m1 nibbles
    (``N * K * 2**p / 2`` bytes per layer) that the e2m1 CTA-pair kernel loads
    by TMA so that its producers generate only the activation windows
    (qkv_proj at 256 images: 11.7 -> 9.6 ms).  The int8 form (p = 5 / 6, or
    N <= 128) does not pay (the int8 kernel is bound by shared-memory traffic,
    which a TMA-fed b does not reduce), so automatic mode leaves it off;
    ``True`` / ``False`` force it on / off."""
    global _PREPACK
    _PREPACK = None if enabled is None else bool(enabled)


def _prepack_applies(weight: torch.Tensor, sc_prec: int, mode: str, stoc_len, chunk_d: int) -> bool:
    from . import sc as _sc
    if _PREPACK is False or USE_NOISE_MODEL or not weight.is_cuda or chunk_d != 0:
        return False
    if not (5 <= sc_prec <= 8) or (mode == "unipolar" and sc_prec == 8):
        return False
    if stoc_len not in (None, 1 << sc_prec) or _sc._DEFAULT_ENGINE == "popc":
        return False
    return _PREPACK is True or (sc_prec in (7, 8) and weight.shape[0] > 128)


class SCLinear(nn.Module):
    """Drop-in ``nn.Linear`` replacement running the matmul through SC
    (reference ``sc_linear.py:291-354``, same constructor)."""

    def __init__(self, linear: nn.Linear, sc_prec: int, mode: str = "bipolar",
                 cfg_override: dict = None, mp_cfg: MPConfig | None = None,
                 adaptive_mp_cfg: AdaptiveMPConfig | None = None,
                 range_mp_cfg: RangeMPConfig | None = None, range_mp_group_size: int = 0,
                 operator: str | None = None, stoc_len: int | None = None, chunk_d: int = 0):
        super().__init__()
        self.sc_prec = sc_prec
        self.stoc_len = stoc_len
        self.mode = mode
        self.weight = linear.weight
        self.bias = linear.bias
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.cfg_override = cfg_override
        self.mp_cfg = mp_cfg
        self.adaptive_mp_cfg = adaptive_mp_cfg
        self.operator = operator
        self.chunk_d = chunk_d
        if range_mp_cfg is not None:
            self.range_entries = build_range_dispatch(self.weight.detach(), range_mp_cfg,
                                                      operator=operator,
                                                      group_size=range_mp_group_size)
        else:
            self.range_entries = None
        self._packed = None
        self._packed_key = None

    def _packed_weight(self, D_in: int):
        """The weight's prepacked SC operand (cached; rebuilt when the weight's
        storage, version counter or the SC settings change)."""
        from .sc import prepack_b
        cfg = self.cfg_override if self.cfg_override is not None else _get_config(D_in, self.sc_prec)
        w = self.weight
        key = (w.data_ptr(), w._version, w.dtype, str(w.device), self.sc_prec, self.mode,
               cfg["uid"])
        if key != self._packed_key:
            self._packed = None  # free the old buffer before building the new one
            self._packed = prepack_b(w.detach(), granularity="per_row", mode=self.mode,
                                     sc_prec=self.sc_prec, config=cfg, group_b=1)
            self._packed_key = key
        return self._packed

    def forward(self, x):
        if self.range_entries is None and self.mp_cfg is None and self.adaptive_mp_cfg is None:
            packed = None
            if _prepack_applies(self.weight, self.sc_prec, self.mode, self.stoc_len,
                                self.chunk_d):
                packed = self._packed_weight(x.shape[-1])
            return _sc_linear(x, self.weight, self.bias, self.sc_prec, mode=self.mode,
                              cfg_override=self.cfg_override, stoc_len=self.stoc_len,
                              chunk_d=self.chunk_d, packed=packed)
        if getattr(self, "_packed_levels", None) is None:
            self._packed_levels = PackedWeights(self.weight, self.mode)
        return _sc_linear_mp(x, self.weight, self.bias, self.sc_prec, self.mode,
                             range_entries=self.range_entries, mp_cfg=self.mp_cfg,
                             adaptive_mp_cfg=self.adaptive_mp_cfg, operator=self.operator,
                             chunk_d=self.chunk_d, packed_for=self._packed_levels)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"sc_prec={self.sc_prec}, stoc_len={self.stoc_len}, mode={self.mode}")
