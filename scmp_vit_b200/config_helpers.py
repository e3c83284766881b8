"""Stream-pool configurations (the ``scmp_kernels.sc.config_helpers`` surface).

A *pool* is the random-number table ``R[d, t]`` (``d`` = stream dimension,
``t`` = position in the stream, ``t < 2**sc_prec``, values in ``[0, 2**p)``)
that the SC engine compares each operand magnitude against.  The reference
builds one pool per ``(D, sc_prec)`` with ``make_sobol_simple_config(D, D, p)``
and caches it on first use (reference ``sc_integration/sc_linear.py:85-92``);
its scramble seeds come from Python's global ``random`` state
(``det/sc_eval.py:222-225``), so creation order is part of the result.

Configs are plain dicts, like the reference's.  Keys:

``kind``        ``"sobol"`` or ``"lfsr16"``
``sc_prec``     p (1..8)
``dims``        number of stream dimensions ``D`` (one per reduction index)
``dims_a``      first constructor argument, kept for API fidelity
``m``           (sobol) uint32 ``[D, p]`` odd direction-number seeds m_i < 2^i
``shift``       (sobol) uint32 ``[D]`` per-dimension digital shift
``antithetic``  (sobol) complement every value
``state0``      (lfsr16) uint16 ``[D]`` non-zero initial LFSR states
``table``       uint8 ``[D, 2**p]`` the pool ``R`` itself
``uid``         process-unique id; keys the device-side pool cache

Sequence definitions (restated in the CPU oracle, ``oracle/sc_oracle.c``):

* Sobol, Gray-code order: ``V_i = m_i << (p - i)``,
  ``x_t = XOR_{i : bit i-1 of gray(t)} V_i``, ``R = x_t ^ shift_d``
  (``^ (2**p - 1)`` when antithetic).  Any odd ``m_i < 2^i`` gives a
  stratified 1-D digital sequence, so every aligned prefix of ``2^j`` points
  hits each ``2^(p-j)``-wide value bin exactly once.
* LFSR-16, Galois form, polynomial x^16 + x^14 + x^13 + x^11 + 1 (mask
  0xB400): value ``t`` is the top ``p`` bits of the state after ``t + 1``
  steps.
"""
from __future__ import annotations

import contextlib
import itertools
import random

import numpy as np

__all__ = [
    "make_sobol_simple_config",
    "make_sobol_antithetic_config",
    "make_sobol_altseed_config",
    "make_lfsr_config",
    "pool_table",
    "config_from_table",
    "det_kernel_tuning",
]

_UID = itertools.count(1)
_MASK64 = (1 << 64) - 1


def _splitmix64(x: int) -> int:
    """SplitMix64 finaliser (Steele, Lea & Flood 2014), used as a fixed hash."""
    x = (x + 0x9E3779B97F4A7C15) & _MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _MASK64
    return x ^ (x >> 31)


def _check_prec(sc_prec: int) -> int:
    p = int(sc_prec)
    if not 1 <= p <= 8:
        raise ValueError(f"sc_prec must be in [1, 8], got {sc_prec}")
    return p


def default_direction_seeds(D: int, sc_prec: int) -> np.ndarray:
    """Default per-dimension direction-number seeds ``m[d, i-1]`` (odd, < 2^i).

    ``m_1 = 1``; for ``i >= 2`` the seed is a fixed hash of ``(d, i)``, so the
    default pool depends only on ``(D, p)`` and the ``random`` state that
    draws the scramble shifts.
    """
    p = _check_prec(sc_prec)
    m = np.empty((D, p), dtype=np.uint32)
    for d in range(D):
        m[d, 0] = 1
        for i in range(2, p + 1):
            h = _splitmix64((d << 8) | i)
            m[d, i - 1] = ((h % (1 << (i - 1))) << 1) | 1
    return m


def sobol_table(m: np.ndarray, shift: np.ndarray, sc_prec: int,
                antithetic: bool = False) -> np.ndarray:
    """Pool ``R[d, t]`` of the scrambled Gray-code Sobol sequence."""
    p = _check_prec(sc_prec)
    T = 1 << p
    full = T - 1
    m = np.asarray(m, dtype=np.uint32)
    D = m.shape[0]
    t = np.arange(T, dtype=np.uint32)
    gray = t ^ (t >> 1)
    V = (m << (p - np.arange(1, p + 1, dtype=np.uint32))[None, :]) & full  # [D, p]
    x = np.zeros((D, T), dtype=np.uint32)
    for i in range(p):
        bit = ((gray >> i) & 1).astype(bool)
        x[:, bit] ^= V[:, i:i + 1]
    x ^= (np.asarray(shift, dtype=np.uint32) & full)[:, None]
    if antithetic:
        x ^= full
    return x.astype(np.uint8)


def lfsr16_table(state0: np.ndarray, sc_prec: int) -> np.ndarray:
    """Pool ``R[d, t]`` of a Galois LFSR-16 per dimension (mask 0xB400)."""
    p = _check_prec(sc_prec)
    T = 1 << p
    s = np.asarray(state0, dtype=np.uint32).copy()
    if np.any(s == 0) or np.any(s > 0xFFFF):
        raise ValueError("LFSR states must be in [1, 65535]")
    out = np.empty((s.shape[0], T), dtype=np.uint8)
    for t in range(T):
        lsb = s & 1
        s >>= 1
        s ^= np.where(lsb == 1, np.uint32(0xB400), np.uint32(0))
        out[:, t] = (s >> (16 - p)).astype(np.uint8)
    return out


def _finish(cfg: dict) -> dict:
    cfg["uid"] = next(_UID)
    return cfg


def make_sobol_simple_config(D_a: int, D_b: int, sc_prec: int) -> dict:
    """Default scrambled-Sobol pool for a ``D_b``-wide reduction.

    Draws one ``sc_prec``-bit digital shift per dimension from Python's
    global ``random`` (so ``random.seed`` fixes the streams, as in the
    reference's ``--seed`` handling).
    """
    p = _check_prec(sc_prec)
    D = int(D_b)
    if D <= 0:
        raise ValueError(f"D must be positive, got {D_b}")
    m = default_direction_seeds(D, p)
    shift = np.array([random.getrandbits(p) for _ in range(D)], dtype=np.uint32)
    return _finish({
        "kind": "sobol", "sc_prec": p, "dims": D, "dims_a": int(D_a),
        "m": m, "shift": shift, "antithetic": False,
        "table": sobol_table(m, shift, p, False),
    })


def make_sobol_antithetic_config(D_a: int, D_b: int, sc_prec: int) -> dict:
    """Antithetic variant: every pool value complemented (``R' = 2^p-1-R``)."""
    cfg = make_sobol_simple_config(D_a, D_b, sc_prec)
    cfg["antithetic"] = True
    cfg["table"] = sobol_table(cfg["m"], cfg["shift"], cfg["sc_prec"], True)
    return cfg


def make_sobol_altseed_config(D_a: int, D_b: int, sc_prec: int, k_seed) -> dict:
    """Alternative direction numbers ``k_seed = [1, m_2, ..., m_p]`` (odd,
    ``m_i < 2^i``) shared by every dimension (reference
    ``cls/experiments/qwt_sc_overnight.py:185-202``)."""
    p = _check_prec(sc_prec)
    seed = [int(s) for s in k_seed]
    if len(seed) != p:
        raise ValueError(f"k_seed needs {p} entries, got {len(seed)}")
    for i, s in enumerate(seed, start=1):
        if s % 2 == 0 or not 0 < s < (1 << i):
            raise ValueError(f"k_seed[{i - 1}]={s} must be odd and < 2^{i}")
    cfg = make_sobol_simple_config(D_a, D_b, p)
    cfg["m"] = np.tile(np.array(seed, dtype=np.uint32), (cfg["dims"], 1))
    cfg["table"] = sobol_table(cfg["m"], cfg["shift"], p, False)
    return cfg


def lfsr_states(D: int, seed: int) -> np.ndarray:
    """Non-zero 16-bit initial states, one per dimension, hashed from seed."""
    out = np.empty(D, dtype=np.uint16)
    for d in range(D):
        h = _splitmix64(((int(seed) & 0xFFFFFFFF) << 32) | d)
        out[d] = 1 + (h % 0xFFFF)
    return out


def make_lfsr_config(D_a: int, D_b: int, sc_prec: int, seed: int = 0) -> dict:
    """16-bit LFSR pool seeded by ``seed`` (e.g. one seed per ViT block)."""
    p = _check_prec(sc_prec)
    D = int(D_b)
    state0 = lfsr_states(D, seed)
    return _finish({
        "kind": "lfsr16", "sc_prec": p, "dims": D, "dims_a": int(D_a),
        "seed": int(seed), "state0": state0,
        "table": lfsr16_table(state0, p),
    })


def config_from_table(table, sc_prec: int) -> dict:
    """A config around an explicit uint8 pool ``table`` ``[D, 2**sc_prec]``,
    e.g. a pool recorded from another run or generated elsewhere."""
    p = _check_prec(sc_prec)
    tab = np.ascontiguousarray(table, dtype=np.uint8)
    if tab.ndim != 2 or tab.shape[1] != (1 << p):
        raise ValueError(f"pool table must be [D, {1 << p}], got {tab.shape}")
    return _finish({"kind": "table", "sc_prec": p, "dims": int(tab.shape[0]),
                    "dims_a": int(tab.shape[0]), "table": tab})


def pool_table(cfg: dict) -> np.ndarray:
    """The uint8 ``[D, 2**p]`` pool of a config (validated)."""
    if not isinstance(cfg, dict) or "table" not in cfg:
        raise TypeError("config must be a dict made by scmp config helpers")
    tab = cfg["table"]
    p = int(cfg["sc_prec"])
    if tab.dtype != np.uint8 or tab.ndim != 2 or tab.shape[1] != (1 << p):
        raise ValueError("malformed pool table")
    return tab


_TUNING = {"det": False}


@contextlib.contextmanager
def det_kernel_tuning():
    """Context manager kept for the reference's det scripts
    (``det/experiments/_p8_breakdown.py:70-73``).  The sm_100a engine picks
    its tiles from the problem shape, so this only records that the caller
    asked for the det heuristic."""
    prev = _TUNING["det"]
    _TUNING["det"] = True
    try:
        yield
    finally:
        _TUNING["det"] = prev
