"""CPU checks of the oracle and of the host-side pool generation.

The reference ships no golden vectors for the SC path (its kernel package is
an empty submodule), so the oracle is pinned here by (1) the literal
(m, n, d, t) definition of the enable-signal count, (2) the Sobol
stratification property of every pool prefix, (3) independent C and numpy
generators of every pool kind, (4) committed fixtures in tests/golden/, and
(5) the statistical behaviour of the estimate (error shrinking ~1/L).
"""
import json
import random
from pathlib import Path

import numpy as np
import pytest

from oracle import sc_oracle as so
from scmp_vit_b200 import config_helpers as ch

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("p", [1, 3, 6, 7, 8])
def test_sobol_pool_c_matches_numpy(p):
    random.seed(p)
    cfg = ch.make_sobol_simple_config(33, 33, p)
    np.testing.assert_array_equal(so.pool_from_config(cfg), cfg["table"])


@pytest.mark.parametrize("p", [7, 8])
def test_sobol_prefixes_are_stratified(p):
    """Every aligned 2^j-prefix of a dimension hits each value bin once."""
    random.seed(1)
    R = ch.make_sobol_simple_config(16, 16, p)["table"].astype(np.int64)
    T = 1 << p
    for j in range(p + 1):
        n = 1 << j
        bins = R[:, :n] >> (p - j)
        for row in bins:
            assert sorted(row.tolist()) == list(range(n))
    assert R.shape == (16, T)


def test_pool_variants_c_matches_numpy():
    random.seed(3)
    for cfg in (ch.make_sobol_antithetic_config(20, 20, 8),
                ch.make_sobol_altseed_config(20, 20, 5, [1, 3, 7, 9, 31]),
                ch.make_lfsr_config(20, 20, 8, seed=11),
                ch.make_lfsr_config(20, 20, 6, seed=0)):
        np.testing.assert_array_equal(so.pool_from_config(cfg), cfg["table"])


def test_python_random_controls_scramble():
    random.seed(0)
    a = ch.make_sobol_simple_config(8, 8, 7)["table"]
    random.seed(0)
    b = ch.make_sobol_simple_config(8, 8, 7)["table"]
    c = ch.make_sobol_simple_config(8, 8, 7)["table"]
    assert np.array_equal(a, b) and not np.array_equal(a, c)


def test_altseed_validation():
    with pytest.raises(ValueError):
        ch.make_sobol_altseed_config(4, 4, 3, [1, 2, 5])
    with pytest.raises(ValueError):
        ch.make_sobol_altseed_config(4, 4, 3, [1, 3])


@pytest.mark.parametrize("mode,p,L", [("bipolar", 7, 128), ("bipolar", 8, 192),
                                      ("bipolar", 2, 3), ("unipolar", 6, 64),
                                      ("unipolar", 8, 97)])
def test_bitpacked_counts_match_literal_loop(mode, p, L):
    rng = np.random.default_rng(p * 100 + L)
    a = rng.standard_normal((4, 11)).astype(np.float32)
    b = rng.standard_normal((5, 11)).astype(np.float32)
    random.seed(2)
    R = ch.make_sobol_simple_config(11, 11, p)["table"]
    ga, nga = so.row_groups("per_row", 1, 4, 1)
    gb, ngb = so.row_groups("per_row", 1, 5, 1)
    ca = so.quantize(a, ga, nga, mode, p)[0]
    cb = so.quantize(b, gb, ngb, mode, p)[0]
    np.testing.assert_array_equal(so.counts(ca, cb, R, p, L), so.count_naive(ca, cb, R, p, L))


def test_quantisation_rules():
    x = np.array([[0.0, 1.0, -2.0, 0.5, -0.25]], dtype=np.float32)
    g, ng = so.row_groups("per_row", 1, 1, 1)
    code, s, z, rs = so.quantize(x, g, ng, "bipolar", 8)
    # q_max = 127, scale = 2/127; codes are 2|x_int| with sign
    assert s[0] == np.float32(2.0) / np.float32(127.0)
    np.testing.assert_array_equal(code[0], [0, 128, -254, 64, -32])
    assert rs[0] == 0 + 128 + 254 + 64 + 32
    code, s, z, rs = so.quantize(x, g, ng, "unipolar", 8)
    # range 3 -> scale 3/255, zero point rint(2 * 255/3) = 170
    assert z[0] == 170
    assert code[0].min() >= 0 and code[0].max() <= 255 and code[0][2] == 0


def test_zero_rows_quantise_to_zero():
    x = np.zeros((2, 7), dtype=np.float32)
    g, ng = so.row_groups("per_row", 1, 2, 1)
    code, s, _, _ = so.quantize(x, g, ng, "bipolar", 7)
    assert not code.any() and np.all(s == np.float32(1e-6) / np.float32(63.0))


def test_group_ids():
    g, n = so.row_groups("per_row", 2, 5, 2)
    assert n == 6 and g.tolist() == [0, 0, 1, 1, 2, 3, 3, 4, 4, 5]
    g, n = so.row_groups("per_head", 3, 2, 1)
    assert n == 3 and g.tolist() == [0, 0, 1, 1, 2, 2]
    g, n = so.row_groups("per_tensor", 3, 2, 1)
    assert n == 1 and not g.any()


def test_error_shrinks_with_stream_length():
    """Sobol SC error scales ~1/L (reference sc_integration/noise_matmul.py:
    12-23: halving L doubles the RMSE)."""
    rng = np.random.default_rng(0)
    a = rng.standard_normal((64, 256)).astype(np.float32)
    b = (rng.standard_normal((96, 256)) * 0.05).astype(np.float32)
    exact = a @ b.T
    errs = {}
    for p in (5, 6, 7, 8):
        random.seed(0)
        R = ch.make_sobol_simple_config(256, 256, p)["table"]
        _, y = so.sc_matmul_ref(a, b, sc_prec=p, pool=R)
        errs[p] = float(np.sqrt(np.mean((y[0] - exact) ** 2)))
    for p in (5, 6, 7):
        assert errs[p + 1] < 0.75 * errs[p], errs
    assert errs[8] / np.abs(exact).mean() < 0.05


def test_early_termination_is_prefix_exact():
    """L < 2^p reuses the 2^p pool: rows at L=192 equal the reference-style
    bucket computation, and L=2^p equals the default."""
    rng = np.random.default_rng(1)
    a = rng.standard_normal((10, 32)).astype(np.float32)
    b = rng.standard_normal((12, 32)).astype(np.float32)
    random.seed(0)
    R = ch.make_sobol_simple_config(32, 32, 8)["table"]
    acc_full, _ = so.sc_matmul_ref(a, b, sc_prec=8, pool=R)
    acc_def, _ = so.sc_matmul_ref(a, b, sc_prec=8, pool=R, stoc_len=256)
    np.testing.assert_array_equal(acc_full, acc_def)
    rowL = np.array([192] * 5 + [256] * 5)
    acc_mp, _ = so.sc_matmul_ref(a, b, sc_prec=8, pool=R, L_row=rowL)
    acc_b, _ = so.sc_matmul_rows_ref(a, b, rowL, {8: R})
    np.testing.assert_array_equal(acc_mp[0], acc_b)
    np.testing.assert_array_equal(acc_mp[0][5:], acc_full[0][5:])


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("sc_case_*.json")))
def test_golden_fixtures(name):
    """Committed fixtures (tests/golden/make_golden.py) still reproduce."""
    case = json.loads((GOLDEN / f"{name}.json").read_text())
    data = np.load(GOLDEN / f"{name}.npz")
    random.seed(case["seed"])
    if case["kind"] == "lfsr16":
        cfg = ch.make_lfsr_config(case["K"], case["K"], case["sc_prec"], seed=case["seed"])
    else:
        cfg = ch.make_sobol_simple_config(case["K"], case["K"], case["sc_prec"])
    np.testing.assert_array_equal(cfg["table"], data["pool"])
    acc, y = so.sc_matmul_ref(data["a"], data["b"], granularity=case["granularity"],
                              mode=case["mode"], sc_prec=case["sc_prec"], pool=cfg["table"],
                              stoc_len=case["stoc_len"])
    np.testing.assert_array_equal(acc, data["acc"])
    np.testing.assert_array_equal(y, data["y"])
