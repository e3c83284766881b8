"""Host logic of the mixed-precision maps and the reference-facing API (CPU).

The free-boundary counts restate the reference's own smoke assertions
(experiments/test_free_boundary_classifier.py: 25/25/25/25 at default
boundaries, 10/10/30/50 +-1 at custom ones, fall-back to default for an
unset block, a flat metric going wholly to the top level)."""
import torch

from scmp_vit_b200 import mp
from scmp_vit_b200.mp_linear import (DispatchEntry, RangeMPConfig, build_range_dispatch,
                                     classify_input_rows, sc_prec_for_stoc_len)


def _counts(a):
    return {sl: int(idx.numel()) for sl, idx in a.level_row_indices.items()}


def test_free_boundary_default_equal_spacing():
    cfg = mp.FreeBoundaryMPConfig(stoc_len_levels=[256, 128, 64, 32])
    mp.set_current_block_idx(0)
    a = mp.adaptive_classify_rows(torch.linspace(0.0, 1.0, 100), 0, 1, cfg, operator="qk")
    assert _counts(a) == {256: 25, 128: 25, 64: 25, 32: 25}


def test_free_boundary_custom_then_fallback():
    cfg = mp.FreeBoundaryMPConfig(stoc_len_levels=[256, 128, 64, 32])
    cfg.set_boundaries("av", block_idx=3, boundaries=torch.tensor([0.90, 0.80, 0.50]))
    metric = torch.linspace(0.0, 1.0, 100)
    mp.set_current_block_idx(3)
    c = _counts(mp.adaptive_classify_rows(metric, 0, 1, cfg, operator="av"))
    for sl, want in ((256, 10), (128, 10), (64, 30), (32, 50)):
        assert abs(c[sl] - want) <= 1, c
    mp.set_current_block_idx(0)
    c = _counts(mp.adaptive_classify_rows(metric, 0, 1, cfg, operator="av"))
    assert c == {256: 25, 128: 25, 64: 25, 32: 25}


def test_free_boundary_flat_metric():
    cfg = mp.FreeBoundaryMPConfig(stoc_len_levels=[256, 64, 16])
    mp.set_current_block_idx(0)
    c = _counts(mp.adaptive_classify_rows(torch.full((50,), 0.5), 0, 1, cfg, operator="qk"))
    assert c == {256: 50, 64: 0, 16: 0}


def test_fixed_quantile_split_higher_metric_longer_stream():
    metric = torch.arange(10, dtype=torch.float32)
    a = mp.classify_rows_by_metric(metric, [128, 256], [0.5, 0.5])  # ascending levels given
    assert a.row_levels.tolist() == [128] * 5 + [256] * 5
    a = mp.classify_rows_by_metric(metric, [256, 192, 128], [0.2, 0.3, 0.5])
    assert _counts(a) == {256: 2, 192: 3, 128: 5}
    assert set(a.level_row_indices[256].tolist()) == {8, 9}


def test_target_fractions_exact_up_to_rounding():
    cfg = mp.AdaptiveMPConfig([256, 128, 64, 32], target_fractions=[0.05, 0.35, 0.40, 0.20])
    c = _counts(mp.adaptive_classify_rows(torch.rand(1000), 9, 10, cfg, operator="qkv_proj"))
    assert c == {256: 50, 128: 350, 64: 400, 32: 200}


def test_adaptive_progress_moves_boundaries():
    cfg = mp.AdaptiveMPConfig([256, 64], alpha=0.5, beta=0.0)
    metric = torch.linspace(0, 1, 101)
    early = _counts(mp.adaptive_classify_rows(metric, 0, 10, cfg))
    late = _counts(mp.adaptive_classify_rows(metric, 9, 10, cfg))
    assert late[256] < early[256]


def test_batched_quantile_matches_per_slice():
    metric = torch.rand(6, 17)
    out = mp.quantile_levels_batched(metric, [128, 256], [0.5, 0.5])
    for i in range(6):
        ref = mp.classify_rows_by_metric(metric[i], [128, 256], [0.5, 0.5]).row_levels
        assert torch.equal(out[i], ref)


def test_seeded_random_assignment_is_deterministic():
    cfg = mp.SeededRandomMPConfig([128, 192, 256], None, seed=3)
    a, b = cfg.assign(300, "cpu", salt=5), cfg.assign(300, "cpu", salt=5)
    assert torch.equal(a, b)
    assert sorted(set(a.tolist())) == [128, 192, 256]
    assert not torch.equal(a, cfg.assign(300, "cpu", salt=6))


def test_sc_prec_for_stoc_len():
    assert [sc_prec_for_stoc_len(v) for v in (1, 2, 64, 128, 129, 192, 256)] == [1, 1, 6, 7, 8, 8, 8]


def test_range_dispatch_merges_groups_by_level():
    w = torch.zeros(8, 4)
    w[0:2] = torch.tensor([1.0, -1.0, 0.5, 0.0])   # wide range -> longest
    w[2:4] = 0.05 * torch.randn(2, 4)
    w[4:6] = torch.tensor([1.0, -1.0, 0.0, 0.0])
    w[6:8] = 0.001
    entries = build_range_dispatch(w, RangeMPConfig([256, 128, 64], base_threshold=0.5),
                                   group_size=2)
    assert all(isinstance(e, DispatchEntry) for e in entries)
    rows = sorted(int(i) for e in entries for i in e.out_indices)
    assert rows == list(range(8))
    by = {e.stoc_len: sorted(e.out_indices.tolist()) for e in entries}
    assert by[256] == [0, 1, 4, 5]
    for e in entries:
        assert torch.equal(e.weight, w.index_select(0, e.out_indices))
        assert e.sc_prec == sc_prec_for_stoc_len(e.stoc_len)


def test_classify_input_rows_uses_abs_max():
    x = torch.tensor([[0.1, -3.0], [0.2, 0.1], [-1.0, 0.0], [0.0, 0.05]])
    a = classify_input_rows(x, mp.MPConfig([256, 128], [0.5, 0.5]))
    assert a.row_levels.tolist() == [256, 128, 256, 128]


def test_budget_logger_accumulates_without_sync():
    mp.AutoMPBudgetLogger.reset()
    mp.AutoMPBudgetLogger.record(2, "qk", 100, torch.tensor(40.0))
    mp.AutoMPBudgetLogger.record(2, "qk", 100, 60)
    s = mp.AutoMPBudgetLogger.summary()[(2, "qk")]
    assert s["baseline"] == 200 and s["actual"] == 100 and s["calls"] == 2
    mp.AutoMPBudgetLogger.reset()
