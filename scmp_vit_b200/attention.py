"""SC attention core: Q@K^T and Attn@V on the engine, batched over (batch, head).

Mirrors the reference's DINOv2 patch (``cls/sc_attention_patch.py:51-328``)
and EVA ``SCMatMul`` (``det/sc_patch/sc_matmul.py:67-195``) with the same
numerics per slice, but without their host loops:

* Q@K^T: one ``per_head`` launch over all B*H slices (one scale per slice).
  Per-head MP (``_classify_per_head``: metric ``|q|.amax((0,2,3))``) becomes
  a per-slice stream-length table, one launch per precision.
* Attn@V: one ``per_row`` launch over all B*H slices instead of the
  reference's B*H Python loop (``cls/sc_attention_patch.py:311-318``).
  Per-row MP (entropy / amax / ipr metric, ``:75-140``) is classified for
  every slice at once and becomes a per-row stream-length table.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn

from . import sc_linear as _scl
from .mp import (
    AdaptiveMPConfig,
    AutoMPBudgetLogger,
    MPConfig,
    adaptive_classify_rows,
    classify_rows_by_metric,
    get_current_block_idx,
    quantile_counts,
    quantile_levels_batched,
)
from .mp_linear import sc_prec_for_stoc_len
from .noise_matmul import _noisy_matmul_core
from .config_helpers import make_sobol_simple_config
from .sc import sc_matmul, softmax_quantize

CfgFor = Callable[[int, int], dict]

AV_METRIC_REVERSE = False
AV_METRIC_KIND = "entropy"  # "amax" | "entropy" | "ipr"


def set_av_metric_reverse(flag: bool):
    global AV_METRIC_REVERSE
    AV_METRIC_REVERSE = bool(flag)


def set_av_metric_kind(kind: str):
    global AV_METRIC_KIND
    if kind not in ("amax", "entropy", "ipr"):
        raise ValueError(f"unknown AV metric: {kind}")
    AV_METRIC_KIND = kind


def av_row_score(attn: torch.Tensor) -> torch.Tensor:
    """Per-row score over the last dim, higher = needs more precision
    (reference ``cls/sc_attention_patch.py:106-126``)."""
    if AV_METRIC_KIND == "amax":
        m = attn.amax(-1)
        return -m if AV_METRIC_REVERSE else m
    if AV_METRIC_KIND == "entropy":
        return -(attn * attn.clamp(min=1e-9).log()).sum(-1)
    return 1.0 / (attn.pow(2).sum(-1) + 1e-9)


def _levels_by_prec(levels):
    by_prec: dict[int, list[int]] = {}
    for L in sorted({int(v) for v in levels if int(v) > 0}):
        by_prec.setdefault(sc_prec_for_stoc_len(L), []).append(L)
    return by_prec


# det/sc_patch/sc_matmul.py keeps a pool cache of its own (``_CFG_CACHE`` at
# :43-53), apart from sc_linear's; SCMatMul draws its pools from this one.
_DET_CFG_CACHE: dict = {}


def _det_get_config(D: int, sc_prec: int) -> dict:
    """``(D, sc_prec)`` pool of the det ``SCMatMul``, created on first use."""
    key = (D, sc_prec)
    if key not in _DET_CFG_CACHE:
        _DET_CFG_CACHE[key] = make_sobol_simple_config(D, D, sc_prec)
    return _DET_CFG_CACHE[key]


def _create_pools_in_first_use_order(cfg_for: CfgFor, D: int, levels,
                                     order: Callable[[], list]) -> None:
    """Pools drawn from Python's ``random`` depend on the order in which they
    are first created.  The reference's bucket loops create a level's pool
    when they first reach that level (head order for per-head MP, the levels
    of each slice longest first for per-row MP), while the grouped launches
    here run the precisions shortest first.  So when a cache-backed factory
    lacks one of the pools, create them first in the reference's order
    (``order()`` lists the levels so; it may read device data, once per
    missing pool).  Other factories (e.g. LFSR pools seeded per block) do not
    depend on the order and are left alone."""
    cache = _scl._CFG_CACHE if cfg_for is _scl._get_config else (
        _DET_CFG_CACHE if cfg_for is _det_get_config else None)
    if cache is None:
        return
    if all((D, sc_prec_for_stoc_len(int(L))) in cache for L in levels if int(L) > 0):
        return
    for L in order():
        if int(L) > 0:
            cfg_for(D, sc_prec_for_stoc_len(int(L)))


def _levels_in_slice_order(row_L: torch.Tensor, levels) -> list:
    """Levels of ``row_L`` [S, N] in the order a loop over slices, each
    visiting its non-empty levels longest first, first reaches them."""
    desc = sorted({int(v) for v in levels}, reverse=True)
    lut = torch.tensor(desc, dtype=row_L.dtype, device=row_L.device)
    present = (row_L.unsqueeze(-1) == lut).any(dim=1).cpu().tolist()  # [S][levels]
    seen: list = []
    for row in present:
        for L, has in zip(desc, row):
            if has and L not in seen:
                seen.append(L)
    return seen


def _run_levels(a, b, table: torch.Tensor, levels, per: str, *, granularity: str, mode: str,
                D_pool: int, cfg_for: CfgFor, out: torch.Tensor) -> torch.Tensor:
    """One engine launch per precision among ``levels``; ``table`` holds the
    stream length per slice (``per='slice'``) or per row (``per='row'``)."""
    by_prec = _levels_by_prec(levels)
    if not by_prec:
        return out.zero_()
    first = True
    for p, Ls in by_prec.items():
        mask = torch.zeros_like(table, dtype=torch.bool)
        for L in Ls:
            mask |= table == L
        if first:
            mask |= table <= 0
        sel = torch.where(mask, table.clamp(min=0), torch.full_like(table, -1))
        kw = {"slice_stoc_len": sel} if per == "slice" else {"row_stoc_len": sel}
        sc_matmul(a, b, granularity=granularity, mode=mode, sc_prec=p,
                  config=cfg_for(D_pool, p), out=out, **kw)
        first = False
    return out


def _qk_slices_by_prec(qf, kf, head_L: torch.Tensor, B: int, levels, counts, *, D: int,
                       cfg_for: CfgFor, out: torch.Tensor) -> torch.Tensor:
    """Per-head levels with host-known counts: the slices of each precision
    class are gathered, run in one launch, and scattered back."""
    H = head_L.numel()
    order = torch.sort(head_L.to(torch.int32), stable=True).indices  # heads by level
    Ls = head_L.to(torch.int32).index_select(0, order)
    base = torch.arange(B, device=qf.device).unsqueeze(1) * H
    start = sum(c for L, c in counts.items() if int(L) <= 0)
    if start:
        idx = (base + order[:start].unsqueeze(0)).reshape(-1)
        out.index_fill_(0, idx, 0.0)
    for p, Lset in _levels_by_prec(levels).items():
        n = sum(counts.get(L, 0) for L in Lset)
        if n == 0:
            continue
        heads = order[start:start + n]
        idx = (base + heads.unsqueeze(0)).reshape(-1)            # slices b*H + h
        sl = Ls[start:start + n].unsqueeze(0).expand(B, n).reshape(-1)
        res = sc_matmul(qf.index_select(0, idx), kf.index_select(0, idx), granularity="per_head",
                        mode="bipolar", sc_prec=p, config=cfg_for(D, p), slice_stoc_len=sl)
        out.index_copy_(0, idx, res)
        start += n
    return out


def _av_rows_by_prec(a_flat, b_flat, row_L: torch.Tensor, levels, counts, *, mode: str,
                     D_pool: int, cfg_for: CfgFor, out: torch.Tensor) -> torch.Tensor:
    """Per-row levels inside every slice with the same host-known counts per
    slice: rows are sorted by level inside each slice, each precision class
    runs as one batched launch over its rows, results are scattered back."""
    S, M, K = a_flat.shape
    order = torch.sort(row_L, dim=1, stable=True).indices          # [S, M]
    Ls = torch.gather(row_L, 1, order)
    a_sorted = torch.gather(a_flat, 1, order.unsqueeze(-1).expand(S, M, K))
    N = b_flat.shape[1]
    out_sorted = torch.empty(S, M, N, dtype=torch.float32, device=a_flat.device)
    start = sum(c for L, c in counts.items() if int(L) <= 0)
    if start:
        out_sorted[:, :start] = 0.0
    for p, Lset in _levels_by_prec(levels).items():
        n = sum(counts.get(L, 0) for L in Lset)
        if n == 0:
            continue
        res = sc_matmul(a_sorted[:, start:start + n].contiguous(), b_flat, granularity="per_row",
                        mode=mode, sc_prec=p, config=cfg_for(D_pool, p),
                        row_stoc_len=Ls[:, start:start + n].reshape(-1))
        out_sorted[:, start:start + n] = res
        start += n
    out.scatter_(1, order.unsqueeze(-1).expand(S, M, N), out_sorted)
    return out


def sc_qk(q: torch.Tensor, k: torch.Tensor, sc_prec: int, *, mp_cfg=None,
          cfg_for: Optional[CfgFor] = None,
          out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """SC ``q @ k^T`` for q, k ``[B, H, N, D]`` -> ``[B, H, N, N]`` fp32, unscaled.

    ``out_dtype=torch.bfloat16`` lets the uniform path write the scores in
    bf16 directly (the fp32 result rounded to nearest even); bf16 q, k are
    read without an fp32 copy (widening is exact)."""
    cfg_for = cfg_for or _scl._get_config
    B, H, N, D = q.shape
    if mp_cfg is None:
        if _scl.USE_NOISE_MODEL:
            return _noisy_matmul_core(q.float(), k.float(), L=2 ** sc_prec, mode="bipolar")
        out = sc_matmul(q.reshape(B * H, N, D), k.reshape(B * H, N, D), granularity="per_head",
                        sc_prec=sc_prec, config=cfg_for(D, sc_prec), stoc_len=2 ** sc_prec,
                        out_dtype=out_dtype)
        return out.reshape(B, H, N, N)
    qf = q.float().reshape(B * H, N, D)
    kf = k.float().reshape(B * H, N, D)
    metric = q.float().abs().amax(dim=(0, 2, 3))  # per head
    if isinstance(mp_cfg, AdaptiveMPConfig):
        t, T = _scl.get_vit_timestep()
        head_L = adaptive_classify_rows(metric, t, T, mp_cfg, operator="qk").row_levels
    else:
        head_L = classify_rows_by_metric(metric, mp_cfg.stoc_len_levels,
                                         mp_cfg.level_fractions).row_levels
    if AutoMPBudgetLogger.enabled:
        maxL = max(int(v) for v in mp_cfg.stoc_len_levels)
        AutoMPBudgetLogger.record(get_current_block_idx(), "qk", B * H * N * N * maxL,
                                  head_L.clamp(min=0).to(torch.float64).sum() * B * N * N)
    if not _scl.USE_NOISE_MODEL:  # reference order: buckets by first head (:168-197)
        _create_pools_in_first_use_order(cfg_for, D, mp_cfg.stoc_len_levels,
                                         lambda: list(dict.fromkeys(head_L.tolist())))
    slice_L = head_L.to(torch.int32).repeat(B)  # slice b*H + h -> head h
    out = torch.empty(B * H, N, N, dtype=torch.float32, device=q.device)
    counts = None if isinstance(mp_cfg, AdaptiveMPConfig) and mp_cfg.target_fractions is None \
        else quantile_counts(H, mp_cfg.stoc_len_levels,
                             getattr(mp_cfg, "level_fractions", None)
                             if not isinstance(mp_cfg, AdaptiveMPConfig) else mp_cfg.target_fractions)
    if counts is not None and not _scl.USE_NOISE_MODEL and len(_levels_by_prec(mp_cfg.stoc_len_levels)) > 1:
        _qk_slices_by_prec(qf, kf, head_L, B, mp_cfg.stoc_len_levels, counts, D=D,
                           cfg_for=cfg_for, out=out)
        return out.reshape(B, H, N, N)
    if _scl.USE_NOISE_MODEL:
        for L in sorted({int(v) for v in mp_cfg.stoc_len_levels}):
            sel = slice_L == L
            if L > 0 and bool(sel.any()):
                out[sel] = _noisy_matmul_core(qf[sel], kf[sel], L=L, mode="bipolar")
            elif L <= 0:
                out[sel] = 0.0
        return out.reshape(B, H, N, N)
    _run_levels(qf, kf, slice_L, mp_cfg.stoc_len_levels, "slice", granularity="per_head",
                mode="bipolar", D_pool=D, cfg_for=cfg_for, out=out)
    return out.reshape(B, H, N, N)


def sc_av(attn: torch.Tensor, v: torch.Tensor, sc_prec: int, *, mode: str = "bipolar",
          mp_cfg=None, cfg_for: Optional[CfgFor] = None,
          out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """SC ``attn @ v`` for attn ``[B, H, N, N]``, v ``[B, H, N, D]`` ->
    ``[B, H, N, D]`` fp32; per-row scales for attn rows and v columns.
    ``out_dtype`` and bf16 inputs as in ``sc_qk`` (uniform path)."""
    cfg_for = cfg_for or _scl._get_config
    B, H, N, D = v.shape
    if mp_cfg is None and not _scl.USE_NOISE_MODEL:
        out = sc_matmul(attn.reshape(B * H, N, N), v.transpose(-1, -2).reshape(B * H, D, N),
                        granularity="per_row", group_a=1, group_b=1, mode=mode,
                        sc_prec=sc_prec, config=cfg_for(N, sc_prec), out_dtype=out_dtype)
        return out.reshape(B, H, N, D)
    a_flat = attn.float().reshape(B * H, N, N)
    b_flat = v.float().transpose(-1, -2).reshape(B * H, D, N)
    if mp_cfg is None:
        out = _noisy_matmul_core(a_flat, b_flat, L=2 ** sc_prec, mode=mode, per_row_scale=True)
        return out.reshape(B, H, N, D)
    score = av_row_score(a_flat)  # [BH, N]
    if isinstance(mp_cfg, AdaptiveMPConfig):
        t, T = _scl.get_vit_timestep()
        rows = [adaptive_classify_rows(score[i], t, T, mp_cfg, operator="av").row_levels
                for i in range(B * H)]
        row_L = torch.stack(rows)
    else:
        row_L = quantile_levels_batched(score, mp_cfg.stoc_len_levels, mp_cfg.level_fractions)
    row_L = row_L.reshape(-1).to(torch.int32)
    if not _scl.USE_NOISE_MODEL:  # reference order: per (b, h), longest level first (:217-240)
        _create_pools_in_first_use_order(
            cfg_for, N, mp_cfg.stoc_len_levels,
            lambda: _levels_in_slice_order(row_L.reshape(B * H, N), mp_cfg.stoc_len_levels))
    if AutoMPBudgetLogger.enabled:
        maxL = max(int(x) for x in mp_cfg.stoc_len_levels)
        AutoMPBudgetLogger.record(get_current_block_idx(), "av", B * H * N * D * maxL,
                                  row_L.clamp(min=0).to(torch.float64).sum() * D)
    out = torch.empty(B * H, N, D, dtype=torch.float32, device=v.device)
    if (not isinstance(mp_cfg, AdaptiveMPConfig) and not _scl.USE_NOISE_MODEL
            and len(_levels_by_prec(mp_cfg.stoc_len_levels)) > 1):
        counts = quantile_counts(N, mp_cfg.stoc_len_levels, mp_cfg.level_fractions)
        _av_rows_by_prec(a_flat, b_flat, row_L.reshape(B * H, N), mp_cfg.stoc_len_levels, counts,
                         mode=mode, D_pool=N, cfg_for=cfg_for, out=out)
        return out.reshape(B, H, N, D)
    if _scl.USE_NOISE_MODEL:
        out.zero_()
        flat_a = a_flat.reshape(B * H * N, N)
        for L in sorted({int(x) for x in mp_cfg.stoc_len_levels if int(x) > 0}):
            sel = (row_L == L).reshape(B * H, N)
            for i in range(B * H):
                r = sel[i]
                if bool(r.any()):
                    out[i, r] = _noisy_matmul_core(a_flat[i][r], b_flat[i], L=L, mode=mode,
                                                   per_row_scale=True)
        del flat_a
        return out.reshape(B, H, N, D)
    _run_levels(a_flat, b_flat, row_L, mp_cfg.stoc_len_levels, "row", granularity="per_row",
                mode=mode, D_pool=N, cfg_for=cfg_for, out=out)
    return out.reshape(B, H, N, D)


# Whether the attention forward fuses `* scale`, the softmax and the Attn@V
# a-operand quantisation into one pass (scmp_softmax_quantize) where the
# result is bit-identical to the unfused steps: fp32 glue, uniform Attn@V
# stream length, rows of 33 to 1024 tokens.
FUSED_SOFTMAX = True


def set_fused_softmax(flag: bool) -> None:
    """Turn the fused softmax + Attn@V quantisation on or off (results are
    identical either way; off runs torch.softmax and quantises its output)."""
    global FUSED_SOFTMAX
    FUSED_SOFTMAX = bool(flag)


def sc_softmax_av(scores: torch.Tensor, scale: float, v: torch.Tensor, sc_prec: int, *,
                  mode: str = "bipolar", cfg_for: Optional[CfgFor] = None) -> torch.Tensor:
    """``sc_av(softmax(scores * scale), v)`` for fp32 scores ``[B, H, N, N]``
    and v ``[B, H, N, D]``, with the softmax and the per-row quantisation of
    its probabilities in one engine pass: the probabilities are never
    stored, and the result equals the unfused steps bit for bit."""
    cfg_for = cfg_for or _scl._get_config
    B, H, N, D = v.shape
    qa = softmax_quantize(scores.reshape(B * H, N, N), scale, mode=mode, sc_prec=sc_prec)
    out = sc_matmul(qa, v.transpose(-1, -2).reshape(B * H, D, N), granularity="per_row",
                    group_a=1, group_b=1, mode=mode, sc_prec=sc_prec, config=cfg_for(N, sc_prec))
    return out.reshape(B, H, N, D)


def _fused_softmax_applies(scores: torch.Tensor, x: torch.Tensor, av_mp_cfg) -> bool:
    return (FUSED_SOFTMAX and av_mp_cfg is None and not _scl.USE_NOISE_MODEL
            and sc_av_fn is sc_av and x.dtype == torch.float32 and scores.is_cuda
            and scores.dtype == torch.float32 and 32 < scores.shape[-1] <= 1024)


def _glue_dtype(x: torch.Tensor) -> Optional[torch.dtype]:
    """bf16 models take SC results in bf16 straight from the engine (the same
    values ``.to(torch.bfloat16)`` gives); otherwise fp32."""
    return torch.bfloat16 if x.dtype == torch.bfloat16 else None


def split_qkv(qkv: torch.Tensor, num_heads: int):
    """``qkv`` [B, N, 3 C] (the fused projection output, C = H D) -> q, k
    [B, H, N, D] contiguous and v [B, H, N, D] as the transposed view of a
    contiguous v^T [B, H, D, N]: the layouts the per-head Q@K^T and per-row
    Attn@V engine calls read without further copies.  One engine pass
    (``scmp_split_qkv``), bit-identical to unbind + transpose."""
    from . import _lib
    B, N, C3 = qkv.shape
    H = num_heads
    D = C3 // (3 * H)
    src = qkv.contiguous()
    q = torch.empty(B, H, N, D, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty_like(q)
    vt = torch.empty(B, H, D, N, dtype=qkv.dtype, device=qkv.device)
    stream = torch.cuda.current_stream(qkv.device).cuda_stream
    _lib.check(_lib.load().scmp_split_qkv(src.data_ptr(), B, N, H, D, src.element_size(),
                                          q.data_ptr(), k.data_ptr(), vt.data_ptr(), stream))
    return q, k, vt.transpose(-1, -2)


def make_sc_attention_forward(sc_prec: int, sc_av: bool, sc_qk: bool = True,
                              qk_mp_cfg: MPConfig | None = None,
                              av_mp_cfg: MPConfig | None = None, *,
                              av_mode: str = "bipolar", cfg_for: Optional[CfgFor] = None):
    """``forward(self, x)`` for a DINOv2-style attention module with
    ``qkv``, ``proj``, ``proj_drop``, ``num_heads``, ``scale`` attributes
    (same signature and numerics as ``cls/sc_attention_patch.py:248-328``)."""
    do_av = sc_av

    def forward(self, x, attn_bias=None):
        B, N, C = x.shape
        H = self.num_heads
        D = C // H
        qkv = self.qkv(x)
        if qkv.is_cuda and qkv.element_size() in (2, 4) and B * H <= 65535 and D <= 256:
            q, k, v = split_qkv(qkv, H)
        else:
            q, k, v = torch.unbind(qkv.reshape(B, N, 3, H, D), 2)
            q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if sc_qk:
            attn = sc_qk_fn(q, k, sc_prec, mp_cfg=qk_mp_cfg, cfg_for=cfg_for,
                            out_dtype=_glue_dtype(x))
            if do_av and _fused_softmax_applies(attn, x, av_mp_cfg):
                out = sc_softmax_av(attn, self.scale, v, sc_prec, mode=av_mode, cfg_for=cfg_for)
                out = out.transpose(1, 2).reshape(B, N, C)
                return self.proj_drop(self.proj(out))
            attn = attn.to(x.dtype) * self.scale
        else:
            attn = (q @ k.transpose(-2, -1)) * self.scale
        attn = attn.softmax(dim=-1)
        if do_av:
            out = sc_av_fn(attn, v, sc_prec, mode=av_mode, mp_cfg=av_mp_cfg,
                           cfg_for=cfg_for, out_dtype=_glue_dtype(x)).to(x.dtype)
        else:
            out = attn @ v
        out = out.transpose(1, 2).reshape(B, N, C)
        out = self.proj(out)
        return self.proj_drop(out)

    return forward


sc_qk_fn = sc_qk
sc_av_fn = sc_av


class SCMatMul(nn.Module):
    """EVA ``MatMul`` replacement: ``A @ B`` (``A (..., M, K)``, ``B (..., K, N)``)
    through SC in one batched launch (reference ``det/sc_patch/sc_matmul.py``)."""

    def __init__(self, sc_prec: int = 8, mode: str = "bipolar", mp_cfg=None,
                 adaptive_mp_cfg=None, op: str | None = None, stoc_len: int | None = None):
        super().__init__()
        if mode not in ("bipolar", "unipolar"):
            raise ValueError(mode)
        self.sc_prec = sc_prec
        self.stoc_len = stoc_len
        self.mode = mode
        self.mp_cfg = mp_cfg
        self.adaptive_mp_cfg = adaptive_mp_cfg
        self.op = op

    def _mp(self):
        return self.adaptive_mp_cfg or self.mp_cfg

    def forward(self, A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
        if A.dim() < 2 or B.dim() < 2:
            raise ValueError(f"SCMatMul expects >=2-D, got A={tuple(A.shape)} B={tuple(B.shape)}")
        if A.shape[-1] != B.shape[-2]:
            raise ValueError(f"Inner-dim mismatch: A.shape[-1]={A.shape[-1]} "
                             f"B.shape[-2]={B.shape[-2]}")
        M, K = A.shape[-2], A.shape[-1]
        N = B.shape[-1]
        lead = A.shape[:-2]
        if B.shape[:-2] != lead:
            B = B.expand(*lead, K, N)
        A_flat = A.reshape(-1, M, K).float().contiguous()
        B_rm = B.reshape(-1, K, N).float().transpose(1, 2).contiguous()  # (BH, N, K)
        BH = A_flat.shape[0]
        cfg = self._mp()
        out = torch.empty(BH, M, N, dtype=torch.float32, device=A.device)
        if cfg is not None and self.op == "qk":
            metric = A_flat.abs().amax(dim=(1, 2))
            if isinstance(cfg, AdaptiveMPConfig):
                t, T = _scl.get_vit_timestep()
                sl = adaptive_classify_rows(metric, t, T, cfg, operator="qk").row_levels
            else:
                sl = classify_rows_by_metric(metric, cfg.stoc_len_levels,
                                             cfg.level_fractions).row_levels
            # reference order: the assignment's levels, longest first (:113-136)
            _create_pools_in_first_use_order(
                _det_get_config, K, cfg.stoc_len_levels,
                lambda: _levels_in_slice_order(sl.reshape(1, -1), cfg.stoc_len_levels))
            _run_levels(A_flat, B_rm, sl.to(torch.int32), cfg.stoc_len_levels, "slice",
                        granularity="per_row", mode=self.mode, D_pool=K,
                        cfg_for=_det_get_config, out=out)
        elif cfg is not None and self.op == "av":
            row_max = A_flat.amax(dim=-1)  # (BH, M)
            if isinstance(cfg, AdaptiveMPConfig):
                t, T = _scl.get_vit_timestep()
                rl = torch.stack([adaptive_classify_rows(row_max[i], t, T, cfg,
                                                         operator="av").row_levels
                                  for i in range(BH)])
            else:
                rl = quantile_levels_batched(row_max, cfg.stoc_len_levels, cfg.level_fractions)
            # reference order: per slice, its levels longest first (:139-160)
            _create_pools_in_first_use_order(
                _det_get_config, K, cfg.stoc_len_levels,
                lambda: _levels_in_slice_order(rl.reshape(BH, M), cfg.stoc_len_levels))
            _run_levels(A_flat, B_rm, rl.reshape(-1).to(torch.int32), cfg.stoc_len_levels,
                        "row", granularity="per_row", mode=self.mode, D_pool=K,
                        cfg_for=_det_get_config, out=out)
        else:
            sc_matmul(A_flat, B_rm, granularity="per_row", group_a=1, group_b=1, mode=self.mode,
                      sc_prec=self.sc_prec, config=_det_get_config(K, self.sc_prec),
                      stoc_len=self.stoc_len, out=out)
        return out.reshape(*lead, M, N).to(A.dtype)
