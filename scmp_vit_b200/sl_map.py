"""Per-(op, block) stream-length maps ("sl_map") from the MP budget search.

An sl_map is ``{op_name: [entry per block]}`` over the op names
``mlp_fc1, mlp_fc2, qk, av, proj`` (``cls/sc_attention_patch.py:332``).
An entry is an ``int`` stream length for the whole (op, block), or a list of
per-row / per-head stream lengths ("bins") whose distinct values and shares
become an ``MPConfig`` at inference; a length <= 0 means the op stays FP in
that block. The JSON written by the search holds the map either bare or
under ``"sl_map"`` (``cls/experiments/mp_budget_swap_search.py:241-246,1368``).

``patch_model_with_sl_map`` installs the SC operators block by block the way
the reference does (``cls/experiments/mp_budget_swap_search.py:613-660``):
``qk`` / ``av`` entries drive the batched attention core, ``proj`` drives
``qkv`` and ``proj`` as ``SCLinear``, ``mlp_fc1`` / ``mlp_fc2`` the MLP
linears. Each MP level runs as one grouped launch per precision class.
"""
from __future__ import annotations

import json
from collections import Counter
from typing import Optional, Sequence

import torch.nn as nn

from .attention import make_sc_attention_forward
from .mp import MPConfig
from .sc_linear import SCLinear

SC_OP_NAMES = ("mlp_fc1", "mlp_fc2", "qk", "av", "proj")


def entry_bins(entry) -> list[int]:
    """Stream lengths of an entry as a list (a scalar entry is one bin)."""
    if isinstance(entry, (list, tuple)):
        return [int(x) for x in entry]
    return [int(entry)]


def entry_avg_sl(entry) -> float:
    bins = entry_bins(entry)
    return float(sum(bins)) / float(len(bins))


def entry_levels_fractions(entry) -> tuple[list[int], list[float]]:
    """Distinct stream lengths, longest first, and the share of bins at each
    (``mp_budget_swap_search.py:259-265``)."""
    bins = entry_bins(entry)
    counts = Counter(bins)
    levels = sorted(counts, reverse=True)
    return levels, [counts[sl] / len(bins) for sl in levels]


def entry_to_mpconfig(entry) -> Optional[MPConfig]:
    """``MPConfig`` of the entry's positive levels with their shares
    renormalised, or None when every bin is <= 0 (the op stays FP)
    (``mp_budget_swap_search.py:330-342``)."""
    levels, fracs = entry_levels_fractions(entry)
    kept = [(sl, fr) for sl, fr in zip(levels, fracs) if sl > 0]
    total = sum(fr for _, fr in kept)
    if not kept or total <= 0:
        return None
    return MPConfig([sl for sl, _ in kept], [fr / total for _, fr in kept])


def make_entry(level: int, n_bins: int):
    return int(level) if n_bins <= 1 else [int(level)] * int(n_bins)


def load_sl_map_json(path: str, op_names: Sequence[str] = SC_OP_NAMES) -> dict[str, list]:
    """Read a search result (``{"sl_map": {...}, ...}``) or a bare map; keeps
    ``op_names`` (each must be present, one entry per block)."""
    with open(path) as f:
        data = json.load(f)
    if isinstance(data, dict) and "sl_map" in data:
        data = data["sl_map"]
    if not isinstance(data, dict):
        raise ValueError(f"{path}: an sl_map is a JSON object of op -> entries")
    missing = [op for op in op_names if op not in data]
    if missing:
        raise ValueError(f"{path}: sl_map lacks ops {missing}")
    lens = {len(data[op]) for op in op_names}
    if len(lens) != 1:
        raise ValueError(f"{path}: ops have different block counts {sorted(lens)}")
    return {op: list(data[op]) for op in op_names}


def save_sl_map_json(path: str, sl_map: dict[str, list], **meta) -> None:
    """Write ``{"sl_map": ..., **meta}`` in the layout ``load_sl_map_json`` reads."""
    with open(path, "w") as f:
        json.dump({**meta, "sl_map": sl_map}, f, indent=2)


def _blocks(model: nn.Module):
    if hasattr(model, "backbone") and hasattr(model.backbone, "blocks"):
        return list(model.backbone.blocks)
    if hasattr(model, "blocks"):
        return list(model.blocks)
    raise RuntimeError("cannot find transformer blocks (model.backbone.blocks or model.blocks)")


def _attention_of(block: nn.Module):
    for m in block.modules():
        if hasattr(m, "qkv") and hasattr(m, "proj") and hasattr(m, "num_heads"):
            return m
    return None


def patch_model_with_sl_map(model: nn.Module, sc_prec: int, sl_map: dict[str, list],
                            mode: str = "bipolar") -> dict[str, int]:
    """Install SC operators per (op, block) from ``sl_map`` (in place).
    Returns how many modules of each kind were patched."""
    blocks = _blocks(model)
    nb = len(blocks)
    for op, entries in sl_map.items():
        if len(entries) != nb:
            raise ValueError(f"sl_map[{op!r}] has {len(entries)} entries for {nb} blocks")
    stats: Counter = Counter()
    for i, blk in enumerate(blocks):
        if hasattr(blk, "block_idx"):
            blk.block_idx = i
        attn = _attention_of(blk)
        qk_mp = entry_to_mpconfig(sl_map.get("qk", [0] * nb)[i])
        av_mp = entry_to_mpconfig(sl_map.get("av", [0] * nb)[i])
        if attn is not None and (qk_mp is not None or av_mp is not None):
            fwd = make_sc_attention_forward(sc_prec, sc_av=av_mp is not None,
                                            sc_qk=qk_mp is not None,
                                            qk_mp_cfg=qk_mp, av_mp_cfg=av_mp)
            attn.forward = fwd.__get__(attn, type(attn))
            stats["attn"] += 1
        mp = entry_to_mpconfig(sl_map.get("proj", [0] * nb)[i])
        if attn is not None and mp is not None:
            if isinstance(attn.qkv, nn.Linear):
                attn.qkv = SCLinear(attn.qkv, sc_prec, mode=mode, mp_cfg=mp, operator="qkv_proj")
                stats["qkv_proj"] += 1
            if isinstance(attn.proj, nn.Linear):
                attn.proj = SCLinear(attn.proj, sc_prec, mode=mode, mp_cfg=mp, operator="out_proj")
                stats["out_proj"] += 1
        mlp = getattr(blk, "mlp", None)
        if mlp is not None:
            for op in ("mlp_fc1", "mlp_fc2"):
                mp = entry_to_mpconfig(sl_map.get(op, [0] * nb)[i])
                attr = op.replace("mlp_", "")
                lin = getattr(mlp, attr, None)
                if mp is not None and isinstance(lin, nn.Linear):
                    setattr(mlp, attr, SCLinear(lin, sc_prec, mode=mode, mp_cfg=mp, operator=op))
                    stats[op] += 1
    return dict(stats)
