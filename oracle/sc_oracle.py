"""CPU oracle for the SC matmul -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module; it is the checker, never the thing measured or
shipped.  The product path (``scmp_vit_b200``) never imports it.

Parity status: UNPINNED.  The reference's SC kernels live in the un-vendored
``scmp_kernels`` submodule (reference ``.gitmodules:4-7``; the directory is
empty, the commit unrecoverable) and the reference ships no golden vectors
for this path.  ``oracle/sc_oracle.c`` restates the semantics the reference's
call sites and documents fix, with every free choice written down there.

Layers:
* ``lib()``            ctypes binding of ``oracle/libsc_oracle.so`` (built by
                       ``oracle/Makefile``; OpenMP for the CPU baseline).
* ``sc_matmul_ref``    the uniform SC matmul (quantise -> count -> rescale),
                       mirroring ``scmp_kernels.sc.sc_matmul``.
* ``sc_matmul_rows_ref`` the per-row stream-length form, restated as the
                       reference's bucket loop (``sc_integration/sc_linear.py:
                       255-265``): one uniform call per distinct level.
* ``count_naive``      pure-Python triple loop over (m, n, d, t) for tiny
                       cases, used to check the bit-packed C counter.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libsc_oracle.so"

_lib = None

_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i16p = ctypes.POINTER(ctypes.c_int16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_f32p = ctypes.POINTER(ctypes.c_float)


def build() -> Path:
    """Compile the C oracle (make -C oracle)."""
    res = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.sco_pool_sobol.argtypes = [ctypes.c_int, ctypes.c_int, _u32p, _u32p, ctypes.c_int, _u8p]
        L.sco_pool_lfsr16.argtypes = [ctypes.c_int, ctypes.c_int, _u16p, _u8p]
        L.sco_quantize.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, _i64p, ctypes.c_int64,
                                   ctypes.c_int, ctypes.c_int, _f32p, _i32p, _i16p, _i64p]
        L.sco_sc_counts.argtypes = [_i16p, _i16p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                    _u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p, _i32p,
                                    ctypes.c_int]
        L.sco_rescale.argtypes = [_i32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p, _i32p,
                                  _f32p, _i32p, _i64p, _f32p, _i32p, _i64p, _f32p, _f32p]
        L.sco_num_threads.restype = ctypes.c_int
        for f in ("sco_pool_sobol", "sco_pool_lfsr16", "sco_quantize", "sco_sc_counts",
                  "sco_rescale"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _p(arr, typ):
    return None if arr is None else arr.ctypes.data_as(typ)


def _check(rc: int, what: str):
    if rc != 0:
        raise ValueError(f"oracle {what} failed with status {rc}")


# ------------------------------------------------------------------- pools

def pool_sobol(m: np.ndarray, shift: np.ndarray, sc_prec: int, antithetic=False) -> np.ndarray:
    m = np.ascontiguousarray(m, dtype=np.uint32)
    shift = np.ascontiguousarray(shift, dtype=np.uint32)
    D = m.shape[0]
    R = np.empty((D, 1 << sc_prec), dtype=np.uint8)
    _check(lib().sco_pool_sobol(D, sc_prec, _p(m, _u32p), _p(shift, _u32p), int(antithetic),
                                _p(R, _u8p)), "pool_sobol")
    return R


def pool_lfsr16(state0: np.ndarray, sc_prec: int) -> np.ndarray:
    s = np.ascontiguousarray(state0, dtype=np.uint16)
    R = np.empty((s.shape[0], 1 << sc_prec), dtype=np.uint8)
    _check(lib().sco_pool_lfsr16(s.shape[0], sc_prec, _p(s, _u16p), _p(R, _u8p)), "pool_lfsr16")
    return R


def pool_from_config(cfg: dict) -> np.ndarray:
    """Recompute a config's pool from its parameters (independent of the
    product's numpy generator)."""
    if cfg["kind"] == "sobol":
        return pool_sobol(cfg["m"], cfg["shift"], cfg["sc_prec"], cfg.get("antithetic", False))
    if cfg["kind"] == "lfsr16":
        return pool_lfsr16(cfg["state0"], cfg["sc_prec"])
    raise ValueError(cfg["kind"])


# ------------------------------------------------------------ quantisation

def row_groups(gran: str, slices: int, rows_per_slice: int, group: int) -> tuple[np.ndarray, int]:
    """Group id per row (groups are contiguous row ranges)."""
    rows = slices * rows_per_slice
    if gran == "per_tensor":
        return np.zeros(rows, dtype=np.int64), 1
    g = rows_per_slice if gran == "per_head" else min(max(int(group), 1), rows_per_slice)
    gps = -(-rows_per_slice // g)
    r = np.arange(rows, dtype=np.int64)
    return (r // rows_per_slice) * gps + (r % rows_per_slice) // g, slices * gps


def quantize(x: np.ndarray, row_group: np.ndarray, ngroups: int, mode: str, p: int):
    """-> (code int16 [rows,K], scale per row, zero per row, rowsum per row)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    rg = np.ascontiguousarray(row_group, dtype=np.int64)
    gs = np.empty(ngroups, dtype=np.float32)
    gz = np.empty(ngroups, dtype=np.int32)
    code = np.empty((rows, K), dtype=np.int16)
    rs = np.empty(rows, dtype=np.int64)
    _check(lib().sco_quantize(_p(x, _f32p), rows, K, _p(rg, _i64p), ngroups,
                              0 if mode == "bipolar" else 1, p, _p(gs, _f32p), _p(gz, _i32p),
                              _p(code, _i16p), _p(rs, _i64p)), "quantize")
    return code, gs[rg], gz[rg], rs


# ------------------------------------------------------------------ counts

def counts(ca: np.ndarray, cb: np.ndarray, R: np.ndarray, p: int, L: int,
           L_row: np.ndarray | None = None, nthreads: int = 0) -> np.ndarray:
    ca = np.ascontiguousarray(ca, dtype=np.int16)
    cb = np.ascontiguousarray(cb, dtype=np.int16)
    R = np.ascontiguousarray(R, dtype=np.uint8)
    M, K = ca.shape
    N = cb.shape[0]
    acc = np.empty((M, N), dtype=np.int32)
    Lr = None if L_row is None else np.ascontiguousarray(L_row, dtype=np.int32)
    _check(lib().sco_sc_counts(_p(ca, _i16p), _p(cb, _i16p), M, N, K, _p(R, _u8p), R.shape[0],
                               p, int(L), _p(Lr, _i32p), _p(acc, _i32p), int(nthreads)), "counts")
    return acc


def count_naive(ca, cb, R, p: int, L: int) -> np.ndarray:
    """Literal (m, n, d, t) loop of the enable-signal count; tiny cases only."""
    M, K = ca.shape
    N = cb.shape[0]
    D = R.shape[0]
    acc = np.zeros((M, N), dtype=np.int64)
    for m in range(M):
        for n in range(N):
            tot = 0
            for d in range(K):
                a, b = int(ca[m, d]), int(cb[n, d])
                k = (abs(a) * L) >> p
                cnt = sum(1 for t in range(k) if int(R[d % D, t]) < abs(b))
                tot += (-1 if a < 0 else 1) * (-1 if b < 0 else 1) * cnt
            acc[m, n] = tot
    return acc


# ----------------------------------------------------------------- matmul

def _as3(x):
    x = np.asarray(x, dtype=np.float32)
    return x if x.ndim == 3 else x[None]


def sc_matmul_ref(a, b, *, granularity="per_row", mode="bipolar", sc_prec=8, pool=None,
                  pool_dims=None, group_a=1, group_b=1, stoc_len=None, bias=None,
                  L_row=None, nthreads: int = 0):
    """Uniform SC matmul.  Returns (acc int32 [BH,M,N], y fp32 [BH,M,N]).

    ``pool`` is the uint8 ``[D, 2**p]`` table; ``pool_dims`` the number of
    its rows used (``d`` reads row ``d % pool_dims``).  ``L_row`` (per
    flattened a-row, same-``p`` levels only) is the per-row stream length.
    """
    a3, b3 = _as3(a), _as3(b)
    BH, M, K = a3.shape
    BHb, N, _ = b3.shape
    p = int(sc_prec)
    L = int(stoc_len) if stoc_len is not None else (1 << p)
    R = np.ascontiguousarray(pool[: (pool_dims or K)], dtype=np.uint8)
    ga, nga = row_groups(granularity, BH, M, group_a)
    gb, ngb = row_groups(granularity, BHb, N, group_b)
    ca, sa, za, rsa = quantize(a3.reshape(BH * M, K), ga, nga, mode, p)
    cb, sb, zb, rsb = quantize(b3.reshape(BHb * N, K), gb, ngb, mode, p)
    acc = np.empty((BH, M, N), dtype=np.int32)
    y = np.empty((BH, M, N), dtype=np.float32)
    mcode = 0 if mode == "bipolar" else 1
    bias32 = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    for s in range(BH):
        sbi = 0 if BHb == 1 else s
        rows = slice(s * M, (s + 1) * M)
        cols = slice(sbi * N, (sbi + 1) * N)
        Lr = None if L_row is None else np.ascontiguousarray(L_row[rows], dtype=np.int32)
        acc[s] = counts(ca[rows], cb[cols], R, p, L, Lr, nthreads)
        prow = None
        if Lr is not None:
            prow = np.full(M, p, dtype=np.int32)
        ys = np.empty((M, N), dtype=np.float32)
        sa_s = np.ascontiguousarray(sa[rows]); za_s = np.ascontiguousarray(za[rows])
        rsa_s = np.ascontiguousarray(rsa[rows])
        sb_s = np.ascontiguousarray(sb[cols]); zb_s = np.ascontiguousarray(zb[cols])
        rsb_s = np.ascontiguousarray(rsb[cols])
        _check(lib().sco_rescale(_p(acc[s], _i32p), M, N, K, mcode, p, L, _p(Lr, _i32p),
                                 _p(prow, _i32p), _p(sa_s, _f32p), _p(za_s, _i32p),
                                 _p(rsa_s, _i64p), _p(sb_s, _f32p), _p(zb_s, _i32p),
                                 _p(rsb_s, _i64p), _p(bias32, _f32p), _p(ys, _f32p)), "rescale")
        y[s] = ys
    return acc, y


def sc_matmul_rows_ref(a, b, row_L, pools: dict, *, mode="bipolar", bias=None,
                       granularity="per_row", group_a=1, group_b=1, pool_dims=None,
                       nthreads: int = 0):
    """Per-row stream lengths, restated as the reference's bucket loop
    (``sc_integration/sc_linear.py:255-265``): rows at level ``L`` are computed
    by a uniform call at ``p = ceil(log2 L)`` with ``pools[p]``; rows with
    ``L == 0`` give zeros (+ bias).  2-D operands only.
    Returns (acc, y) with acc of pruned rows = 0."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    M, K = a.shape
    N = b.shape[0]
    row_L = np.asarray(row_L, dtype=np.int64)
    acc = np.zeros((M, N), dtype=np.int32)
    y = np.zeros((M, N), dtype=np.float32)
    if bias is not None:
        y += np.asarray(bias, dtype=np.float32)[None, :]
    for L in sorted(set(int(v) for v in row_L.tolist())):
        if L <= 0:
            continue
        idx = np.nonzero(row_L == L)[0]
        p = max(1, int(np.ceil(np.log2(L))))
        acc_s, y_s = sc_matmul_ref(a[idx], b, granularity=granularity, mode=mode, sc_prec=p,
                                   pool=pools[p], pool_dims=pool_dims or K, group_a=group_a,
                                   group_b=group_b, stoc_len=L, bias=bias, nthreads=nthreads)
        acc[idx] = acc_s[0]
        y[idx] = y_s[0]
    return acc, y


def sc_matmul_segments_ref(a, b, k_segment: int, *, mode="bipolar", sc_prec=8, pool=None,
                           stoc_len=None, bias=None, L_row=None, nthreads: int = 0):
    """Segmented K (head-aligned compensation, chunk-D summation): each
    segment is a per-row SC matmul with pool rows ``0..k_segment-1``; the fp32
    results are summed in segment order (reference
    ``sc_integration/head_aligned_comp.py:128-144``), then the bias is added.
    Returns (sum of segment accumulators, y)."""
    a3, b3 = _as3(a), _as3(b)
    K = a3.shape[-1]
    if K % k_segment:
        raise ValueError("k_segment must divide K")
    acc_tot, y = None, None
    for s0 in range(0, K, k_segment):
        acc_s, y_s = sc_matmul_ref(a3[..., s0:s0 + k_segment], b3[..., s0:s0 + k_segment],
                                   mode=mode, sc_prec=sc_prec, pool=pool, pool_dims=k_segment,
                                   stoc_len=stoc_len, L_row=L_row, nthreads=nthreads)
        if y is None:
            acc_tot, y = acc_s.astype(np.int64), y_s
        else:
            acc_tot += acc_s
            y = (y + y_s).astype(np.float32)
    if bias is not None:
        y = (y + np.asarray(bias, dtype=np.float32)[None, None, :]).astype(np.float32)
    return acc_tot.astype(np.int32), y


def num_threads() -> int:
    return int(lib().sco_num_threads())
