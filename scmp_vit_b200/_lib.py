"""ctypes binding of the engine's C ABI (``include/scmp_b200.h``).

The library is built in-tree (``scmp_vit_b200/libscmp_b200.so``).  There is
no fallback: if it is missing or fails to load, every SC call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libscmp_b200.so"

ABI_VERSION = 1
NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024  # SCMP_NOALLOC_SCRATCH_BYTES

SCMP_OK = 0
STATUS_NAMES = {
    -1: "SCMP_EINVAL", -2: "SCMP_ECUDA", -3: "SCMP_EWORKSPACE",
    -4: "SCMP_EUNSUPPORTED", -5: "SCMP_ETIMEOUT",
}
GRANULARITY = {"per_row": 0, "per_head": 1, "per_tensor": 2}
MODE = {"bipolar": 0, "unipolar": 1}
ENGINE = {"auto": 0, "popc": 1, "tcgen05": 2}
IO_A_BF16, IO_B_BF16, IO_OUT_BF16, IO_B_PACKED, IO_A_QUANT = 1, 2, 4, 8, 16  # io_flags bits

EXPORTED_SYMBOLS = (
    "scmp_sc_matmul_workspace_size",
    "scmp_sc_matmul",
    "scmp_sc_matmul_noalloc",
    "scmp_last_error",
    "scmp_abi_version",
    "scmp_kernel_launches",
    "scmp_engine_status",
    "scmp_probe_int_peak",
    "scmp_debug_set_wait_limit",
    "scmp_debug_hold_producers",
    "scmp_prepack_b_size",
    "scmp_prepack_b",
    "scmp_split_qkv",
    "scmp_softmax_quantize_size",
    "scmp_softmax_quantize",
    "scmp_bias_gelu",
    "scmp_scale_residual",
)


class MatmulArgs(ctypes.Structure):
    """Mirror of ``scmp_matmul_args`` (field order and types must match)."""
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("engine", ctypes.c_int32),
        ("a", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("batch_b", ctypes.c_int64),
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("granularity", ctypes.c_int32),
        ("mode", ctypes.c_int32),
        ("sc_prec", ctypes.c_int32),
        ("stoc_len", ctypes.c_int32),
        ("group_a", ctypes.c_int64),
        ("group_b", ctypes.c_int64),
        ("k_segment", ctypes.c_int64),
        ("pool", ctypes.c_void_p),
        ("pool_dims", ctypes.c_int32),
        ("io_flags", ctypes.c_int32),
        ("row_stoc_len", ctypes.c_void_p),
        ("slice_stoc_len", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("acc_out", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class EngineError(RuntimeError):
    """A non-zero status returned by the engine."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the engine library once (raises if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"SC engine library {LIB_PATH} is missing; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'`. "
                "There is no CPU fallback.")
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.scmp_sc_matmul_workspace_size.argtypes = [ctypes.POINTER(MatmulArgs)]
        lib.scmp_sc_matmul_workspace_size.restype = ctypes.c_size_t
        lib.scmp_sc_matmul.argtypes = [ctypes.POINTER(MatmulArgs), ctypes.c_void_p]
        lib.scmp_sc_matmul.restype = ctypes.c_int
        lib.scmp_sc_matmul_noalloc.argtypes = [ctypes.POINTER(MatmulArgs), ctypes.c_void_p]
        lib.scmp_sc_matmul_noalloc.restype = ctypes.c_int
        lib.scmp_prepack_b_size.argtypes = [ctypes.POINTER(MatmulArgs)]
        lib.scmp_prepack_b_size.restype = ctypes.c_size_t
        lib.scmp_prepack_b.argtypes = [ctypes.POINTER(MatmulArgs), ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.c_void_p]
        lib.scmp_prepack_b.restype = ctypes.c_int
        lib.scmp_last_error.argtypes = []
        lib.scmp_last_error.restype = ctypes.c_char_p
        lib.scmp_abi_version.argtypes = []
        lib.scmp_abi_version.restype = ctypes.c_int
        lib.scmp_kernel_launches.argtypes = []
        lib.scmp_kernel_launches.restype = ctypes.c_uint64
        lib.scmp_engine_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint)]
        lib.scmp_engine_status.restype = ctypes.c_int
        lib.scmp_probe_int_peak.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
        lib.scmp_probe_int_peak.restype = ctypes.c_int
        lib.scmp_split_qkv.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p]
        lib.scmp_split_qkv.restype = ctypes.c_int
        lib.scmp_softmax_quantize_size.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.scmp_softmax_quantize_size.restype = ctypes.c_size_t
        lib.scmp_softmax_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                              ctypes.c_void_p]
        lib.scmp_softmax_quantize.restype = ctypes.c_int
        lib.scmp_bias_gelu.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_void_p]
        lib.scmp_bias_gelu.restype = ctypes.c_int
        lib.scmp_scale_residual.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64,
                                                                    ctypes.c_int64,
                                                                    ctypes.c_void_p]
        lib.scmp_scale_residual.restype = ctypes.c_int
        lib.scmp_debug_set_wait_limit.argtypes = [ctypes.c_uint64]
        lib.scmp_debug_set_wait_limit.restype = ctypes.c_int
        lib.scmp_debug_hold_producers.argtypes = [ctypes.c_int]
        lib.scmp_debug_hold_producers.restype = ctypes.c_int
        if lib.scmp_abi_version() != ABI_VERSION:
            raise RuntimeError(
                f"engine ABI {lib.scmp_abi_version()} != expected {ABI_VERSION}")
        _lib = lib
        return lib


def kernel_launches() -> int:
    """Kernels launched by the engine library so far in this process."""
    return int(load().scmp_kernel_launches())


def engine_status(reset: bool = False) -> int:
    """Sticky device error flags (bit 0: a bounded wait in the tensor-core
    engine gave up).  Synchronises the current device."""
    v = ctypes.c_uint(0)
    check(load().scmp_engine_status(int(reset), ctypes.byref(v)))
    return int(v.value)


def set_wait_limit(ns: int) -> None:
    """Limit of the engine's bounded device waits on the current device
    (default 2 s); a test hook for the give-up path."""
    check(load().scmp_debug_set_wait_limit(int(ns)))


def hold_producers(on: bool) -> None:
    """Test hook: make the e2m1 kernels' bounded waits run out (see
    ``scmp_debug_hold_producers`` in the header)."""
    check(load().scmp_debug_hold_producers(1 if on else 0))


def probe_int_peak(kind: int) -> float:
    """Measured rate of one instruction class on the current device
    (0: LOP3+POPC bit-products/s, 1: mma.sync b1 bit-products/s,
    2: mma.sync s8 MACs/s, 3 / 4: tcgen05 kind::mxf4 M128 x N256 / N64 MACs/s,
    i.e. e2m1 bit-products/s)."""
    v = ctypes.c_double(0.0)
    check(load().scmp_probe_int_peak(int(kind), ctypes.byref(v)))
    return float(v.value)


def last_error() -> str:
    msg = load().scmp_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    if status != SCMP_OK:
        raise EngineError(status, last_error())
