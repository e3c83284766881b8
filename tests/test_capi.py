"""CPU checks of the C ABI: the library loads, exports every symbol that
include/*.h declares, and rejects bad arguments before touching a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from scmp_vit_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names.update(re.findall(r"SCMP_API\s+[\w\s\*]+?\b(scmp_\w+)\s*\(", text))
    return names


def test_header_declares_the_binding_surface():
    assert set(_lib.EXPORTED_SYMBOLS) <= _declared_symbols()


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_struct_layout_matches_header():
    # 2*i32 + 2 ptr + 5 i64 + 4 i32 + 3 i64 + ptr + 2 i32 + 6 ptr + size_t
    assert ctypes.sizeof(_lib.MatmulArgs) == 8 + 16 + 40 + 16 + 16 + 8 + 8 + 8 + 48 + 8
    assert _lib.MatmulArgs.workspace_bytes.offset == ctypes.sizeof(_lib.MatmulArgs) - 8


def _args(**kw):
    a = _lib.MatmulArgs()
    a.abi_version = _lib.ABI_VERSION
    a.batch, a.batch_b, a.M, a.N, a.K = 1, 1, 4, 5, 8
    a.sc_prec, a.stoc_len = 7, 128
    a.group_a = a.group_b = 1
    a.pool_dims = 8
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,msg", [
    (dict(abi_version=99), "abi_version"),
    (dict(K=0), "bad shape"),
    (dict(batch=2, batch_b=3), "batch_b"),
    (dict(granularity=7), "granularity"),
    (dict(mode=3), "mode"),
    (dict(sc_prec=9), "sc_prec"),
    (dict(sc_prec=1, mode=0), "sc_prec"),
    (dict(stoc_len=129), "stoc_len"),
    (dict(stoc_len=0), "stoc_len"),
    (dict(group_a=0), "group"),
    (dict(pool_dims=0), "pool_dims"),
    (dict(engine=5), "engine"),
    (dict(io_flags=32), "io_flags"),
    (dict(io_flags=16, granularity=1), "SCMP_IO_A_QUANT"),
    (dict(io_flags=16 | 1), "SCMP_IO_A_QUANT"),
    (dict(io_flags=16, K=8, k_segment=4), "SCMP_IO_A_QUANT"),
])
def test_invalid_arguments_are_rejected(kw, msg):
    lib = _lib.load()
    args = _args(**kw)
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(args)) == 0
    rc = lib.scmp_sc_matmul(ctypes.byref(args), None)
    assert rc == -1
    assert msg in _lib.last_error()


def test_null_pointers_and_workspace_are_rejected():
    lib = _lib.load()
    args = _args()
    need = lib.scmp_sc_matmul_workspace_size(ctypes.byref(args))
    assert need > 0
    assert lib.scmp_sc_matmul(ctypes.byref(args), None) == -1  # NULL operands
    args.a = args.b = args.pool = args.out = 16  # non-NULL placeholders, never dereferenced
    assert lib.scmp_sc_matmul(ctypes.byref(args), None) == -3
    assert "workspace" in _lib.last_error()


def test_empty_problem_is_a_no_op():
    lib = _lib.load()
    args = _args(M=0)
    assert lib.scmp_sc_matmul(ctypes.byref(args), None) == 0


def test_workspace_grows_with_problem():
    lib = _lib.load()
    small = lib.scmp_sc_matmul_workspace_size(ctypes.byref(_args()))
    big = lib.scmp_sc_matmul_workspace_size(ctypes.byref(_args(M=400, N=500, K=64, pool_dims=64)))
    assert big > small


def test_softmax_quantize_rejects_bad_arguments():
    """Sizes and arguments of scmp_softmax_quantize are checked before any
    launch (no GPU needed)."""
    lib = _lib.load()
    assert lib.scmp_softmax_quantize_size(-1, 257) == 0
    assert lib.scmp_softmax_quantize_size(4, 0) == 0
    assert lib.scmp_softmax_quantize_size(514, 257) >= 514 * 264 * 2 + 3 * 514 * 4
    for rows, K, mode, prec, code in ((4, 32, 0, 8, -4), (4, 1025, 0, 8, -4), (4, 257, 3, 8, -1),
                                      (4, 257, 0, 9, -1), (-1, 257, 0, 8, -1)):
        rc = lib.scmp_softmax_quantize(None, rows, K, 0.125, mode, prec, None, 0, None, None)
        assert rc == code, (rows, K, mode, prec, rc)
    rc = lib.scmp_softmax_quantize(None, 4, 257, 0.125, 0, 8, None, 0, None, None)
    assert rc == -1 and "non-NULL" in _lib.last_error()


def test_block_glue_rejects_bad_arguments():
    """Argument checks of the fused block glue (no launch, no GPU needed)."""
    lib = _lib.load()
    assert lib.scmp_bias_gelu(None, None, -1, 4, None) == -1
    assert lib.scmp_bias_gelu(None, None, 0, 4, None) == 0
    assert lib.scmp_bias_gelu(None, None, 2, 4, None) == -1
    assert "non-NULL" in _lib.last_error()
    assert lib.scmp_scale_residual(None, None, None, None, None, None, 3, -2, None) == -1
    assert lib.scmp_scale_residual(None, None, None, None, None, None, 3, 4, None) == -1
    assert "non-NULL" in _lib.last_error()
