"""``sc_matmul`` -- the ``scmp_kernels.sc`` entry point, on the sm_100a engine.

Reference contract (the kernel package itself is not vendored; usage from
``sc_integration/sc_linear.py:137-147``, ``cls/sc_attention_patch.py:288-291,
314-318``, ``det/sc_patch/sc_matmul.py:187-194`` and the adapters at
``sc_integration/sc_attention.py:39-81``):

    sc_matmul(a, b, *, granularity="per_row"|"per_head"|"per_tensor",
              mode="bipolar"|"unipolar", sc_prec, config, group_a=1,
              group_b=1, chunk_d=0, stoc_len=None) -> fp32 tensor

``a`` is ``[M, K]`` or ``[BH, M, K]``, ``b`` is ``[N, K]`` or ``[BH, N, K]``
(a 2-D ``b`` is shared by every slice); the result is ``a @ b^T`` per slice,
estimated by SC.  ``stoc_len=None`` means ``2**sc_prec``.  ``per_head``
gives one scale per slice, ``per_tensor`` one per tensor, ``per_row`` one
per ``group_*`` rows.  With ``chunk_d > 0`` the reduction index ``d`` reads
pool row ``d % chunk_d`` of a ``(chunk_d, sc_prec)`` config.

There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional

import torch

from . import _lib
from .config_helpers import make_sobol_simple_config, pool_table

__all__ = ["sc_matmul", "device_pool", "default_config", "set_default_engine", "prepack_b",
           "PackedWeight", "softmax_quantize", "QuantizedRows"]

_DEFAULT_ENGINE = "auto"


def set_default_engine(engine: str) -> None:
    """Engine used when ``sc_matmul(engine=None)``: ``auto`` (the library
    picks), ``tcgen05`` (tensor cores) or ``popc`` (CUDA cores)."""
    global _DEFAULT_ENGINE
    engine = _DEFAULT_ENGINE if engine is None else engine
    if engine not in _lib.ENGINE:
        raise ValueError(f"unknown engine {engine!r}")
    _DEFAULT_ENGINE = engine


_POOL_LOCK = threading.Lock()
_POOLS: dict = {}
_DEFAULT_CFGS: dict = {}


def default_config(D: int, sc_prec: int) -> dict:
    """Process-wide ``(D, sc_prec)`` pool, created on first use."""
    key = (int(D), int(sc_prec))
    with _POOL_LOCK:
        if key not in _DEFAULT_CFGS:
            _DEFAULT_CFGS[key] = make_sobol_simple_config(D, D, sc_prec)
        return _DEFAULT_CFGS[key]


def device_pool(config: dict, device: torch.device) -> torch.Tensor:
    """The config's pool as a uint8 device tensor, uploaded once per device."""
    key = (config["uid"], device.index if device.index is not None else torch.cuda.current_device())
    with _POOL_LOCK:
        t = _POOLS.get(key)
        if t is None:
            tab = pool_table(config)
            t = torch.from_numpy(tab.copy()).to(device=device, non_blocking=False)
            _POOLS[key] = t
        return t


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class PackedWeight:
    """A weight ``b`` ([N, K]) quantised and expanded into its tensor-core
    operand bytes once (``scmp_prepack_b``); pass it as ``b`` to
    ``sc_matmul`` with the same granularity, mode, sc_prec, config and
    group_b.  Results are bit-identical to passing the weight itself; the
    engine loads the bytes with TMA instead of generating them in every call.
    Holds about ``N * K * 2**sc_prec / 2`` bytes of device memory for
    sc_prec 7 / 8 with N > 128 (e2m1 nibbles for the e2m1 CTA pairs), else
    ``N * K * 2**sc_prec`` (int8 bytes)."""

    def __init__(self, buf: torch.Tensor, N: int, K: int, granularity: str, mode: str,
                 sc_prec: int, config: dict, group_b: int, source: Optional[torch.Tensor] = None,
                 k_segment: int = 0):
        self.buf = buf
        self.k_segment = int(k_segment)  # > 0: packed for calls with this k_segment
        self.source = source  # the weight it was packed from (not read by the engine)
        self.N, self.K = N, K
        self.granularity, self.mode, self.sc_prec = granularity, mode, sc_prec
        self.config = config
        self.group_b = group_b
        self.device = buf.device

    @property
    def shape(self):
        return (self.N, self.K)

    def matches(self, *, granularity: str, mode: str, sc_prec: int, config: dict,
                group_b: int, k_segment: int = 0) -> bool:
        return (granularity == self.granularity and mode == self.mode and
                sc_prec == self.sc_prec and config["uid"] == self.config["uid"] and
                int(k_segment) == self.k_segment and
                (granularity != "per_row" or max(int(group_b), 1) == self.group_b))


class QuantizedRows:
    """Softmax probabilities already quantised as the a operand of a per-row
    ``sc_matmul`` (``softmax_quantize``): int16 codes and per-row scale /
    zero point / row sum in the engine's layout.  Pass it as ``a`` with
    ``granularity="per_row"``, ``group_a=1`` and the same ``mode`` and
    ``sc_prec``; the result is bit-identical to passing the probabilities.
    ``probs`` holds the probabilities when they were asked for."""

    def __init__(self, buf: torch.Tensor, shape, mode: str, sc_prec: int,
                 probs: Optional[torch.Tensor] = None):
        self.buf = buf
        self.shape = tuple(int(d) for d in shape)
        self.mode, self.sc_prec = mode, int(sc_prec)
        self.probs = probs
        self.device = buf.device
        self.is_cuda = buf.is_cuda

    def dim(self) -> int:
        return len(self.shape)


@torch.no_grad()
def softmax_quantize(scores: torch.Tensor, scale: float, *, mode: str = "bipolar",
                     sc_prec: int = 8, keep_probs: bool = False) -> QuantizedRows:
    """``softmax(scores * scale, dim=-1)`` quantised per row for the a operand
    of ``sc_matmul``, in one pass (``scmp_softmax_quantize``): the
    probabilities carry torch.softmax's fp32 bits and their codes are those
    ``sc_matmul`` would compute, without storing the probabilities
    (``keep_probs`` stores them in ``.probs`` as well).  ``scores``: fp32
    CUDA ``[..., K]`` with 32 < K <= 1024."""
    if mode not in _lib.MODE:
        raise ValueError(f"unknown mode {mode!r}")
    if not scores.is_cuda or scores.dtype != torch.float32:
        raise ValueError("softmax_quantize takes fp32 CUDA scores")
    x = scores.contiguous()
    K = x.shape[-1]
    rows = x.numel() // K if K else 0
    lib = _lib.load()
    nbytes = lib.scmp_softmax_quantize_size(rows, K)
    if nbytes == 0:
        raise ValueError(f"bad softmax_quantize shape {tuple(x.shape)}")
    buf = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    probs = torch.empty_like(x) if keep_probs else None
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(lib.scmp_softmax_quantize(
            ctypes.c_void_p(x.data_ptr()), rows, K, float(scale), _lib.MODE[mode], int(sc_prec),
            ctypes.c_void_p(buf.data_ptr()), nbytes, ctypes.c_void_p(_ptr(probs)),
            ctypes.c_void_p(stream)))
    return QuantizedRows(buf, x.shape, mode, sc_prec, probs)


def _base_args(engine: str, granularity: str, mode: str, p: int, L: int, group_a: int,
               group_b: int) -> "_lib.MatmulArgs":
    args = _lib.MatmulArgs()
    args.abi_version = _lib.ABI_VERSION
    args.engine = _lib.ENGINE[engine]
    args.granularity = _lib.GRANULARITY[granularity]
    args.mode = _lib.MODE[mode]
    args.sc_prec = p
    args.stoc_len = L
    args.group_a = max(int(group_a), 1)
    args.group_b = max(int(group_b), 1)
    return args


@torch.no_grad()
def prepack_b(b: torch.Tensor, *, granularity: str = "per_row", mode: str = "bipolar",
              sc_prec: int = 8, config: Optional[dict] = None,
              group_b: int = 1, k_segment: int = 0) -> PackedWeight:
    """Quantise the weight ``b`` ([N, K], fp32 or bf16, CUDA) and expand its
    SC operand bytes once (see ``PackedWeight``).  ``k_segment > 0`` packs it
    for segmented calls (each segment quantised on its own, pool rows per
    index inside the segment; sc_prec 7 or 8)."""
    if granularity not in _lib.GRANULARITY or mode not in _lib.MODE:
        raise ValueError(f"unknown granularity / mode {granularity!r} / {mode!r}")
    if b.dim() != 2 or not b.is_cuda:
        raise ValueError("prepack_b needs a 2-D CUDA weight [N, K]")
    N, K = b.shape
    p = int(sc_prec)
    kseg = int(k_segment) if 0 < int(k_segment) < K else 0
    if kseg and K % kseg:
        raise ValueError(f"k_segment={kseg} must divide K={K}")
    if config is None:
        config = default_config(kseg or K, p)
    if int(config["sc_prec"]) != p or int(config["dims"]) < (kseg or K):
        raise ValueError("config must be (>= K or k_segment dims, sc_prec) for prepacking")
    bt = b.contiguous() if b.dtype in (torch.float32, torch.bfloat16) else b.float().contiguous()
    dev = b.device
    pool = device_pool(config, dev)
    args = _base_args("auto", granularity, mode, p, 1 << p, 1, group_b)
    args.b = bt.data_ptr()
    args.batch, args.batch_b, args.M, args.N, args.K = 1, 1, 1, N, K
    args.pool = pool.data_ptr()
    args.pool_dims = kseg or K
    args.k_segment = kseg
    args.io_flags = _lib.IO_B_BF16 if bt.dtype == torch.bfloat16 else 0
    lib = _lib.load()
    nbytes = lib.scmp_prepack_b_size(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(lib.scmp_prepack_b(ctypes.byref(args), None, 0, None))  # raises the reason
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.scmp_prepack_b(ctypes.byref(args), ctypes.c_void_p(buf.data_ptr()),
                                      nbytes, ctypes.c_void_p(stream)))
    return PackedWeight(buf, N, K, granularity, mode, p, config, max(int(group_b), 1), source=b,
                        k_segment=kseg)


@torch.no_grad()
def sc_matmul(a: torch.Tensor, b: torch.Tensor, *, granularity: str = "per_row",
              mode: str = "bipolar", sc_prec: int = 8, config: Optional[dict] = None,
              group_a: int = 1, group_b: int = 1, chunk_d: int = 0,
              stoc_len: Optional[int] = None, bias: Optional[torch.Tensor] = None,
              row_stoc_len: Optional[torch.Tensor] = None,
              slice_stoc_len: Optional[torch.Tensor] = None,
              out: Optional[torch.Tensor] = None,
              acc_out: Optional[torch.Tensor] = None,
              k_segment: int = 0,
              engine: Optional[str] = None,
              out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """SC estimate of ``a @ b^T`` (see module docstring).

    Extra keyword arguments beyond the reference signature:
    ``bias`` ([N], fused into the rescale), ``row_stoc_len`` (int32 per
    a-row stream length, ``[BH*M]``; 0 = pruned row, < 0 = leave ``out``
    row untouched), ``slice_stoc_len`` (int32 per slice), ``out``,
    ``acc_out`` (int32 signed popcount sums, for parity checks),
    ``k_segment`` (split K into equal segments, each quantised and rescaled
    on its own, fp32 results summed in order), ``engine``, ``out_dtype``
    (``torch.float32``, the default, or ``torch.bfloat16``: the fp32 result
    with bias rounded to nearest even, as ``.to(torch.bfloat16)`` would).
    bf16 operands are read as they are (widening to fp32 is exact); other
    dtypes are converted to fp32.

    ``chunk_d > 0`` (bipolar, ``K > chunk_d``) runs the chunked form of the
    reference's chunk-D summation (``sc_integration/sc_attention.py:337-376``):
    ``k_segment = chunk_d`` with the ``(chunk_d, sc_prec)`` pool reused by
    every chunk; a ragged last chunk is zero-padded, which leaves bipolar
    scales and counts unchanged.
    """
    if granularity not in _lib.GRANULARITY:
        raise ValueError(f"unknown granularity {granularity!r}")
    if mode not in _lib.MODE:
        raise ValueError(f"unknown mode {mode!r}")
    engine = _DEFAULT_ENGINE if engine is None else engine
    if engine not in _lib.ENGINE:
        raise ValueError(f"unknown engine {engine!r}")
    packed = b if isinstance(b, PackedWeight) else None
    qa = a if isinstance(a, QuantizedRows) else None
    if a.dim() not in (2, 3) or (packed is None and b.dim() not in (2, 3)):
        raise ValueError(f"sc_matmul expects 2-D or 3-D operands, got {tuple(a.shape)} "
                         f"and {tuple(b.shape)}")
    if not a.is_cuda or (packed is None and not b.is_cuda):
        raise RuntimeError("sc_matmul runs on the CUDA engine only (no CPU path); "
                           f"got devices {a.device} and {b.device}")
    if a.device != b.device:
        raise ValueError(f"operands on different devices: {a.device} vs {b.device}")
    batched = a.dim() == 3
    if qa is not None:
        a3 = None
        BH, M, K = qa.shape if batched else (1,) + qa.shape
        if (granularity != "per_row" or max(int(group_a), 1) != 1 or mode != qa.mode
                or int(sc_prec) != qa.sc_prec or chunk_d or int(k_segment or 0) not in (0, K)):
            raise ValueError("a quantised a runs per_row with group_a=1, its own mode and "
                             "sc_prec, and no chunk_d / k_segment")
    else:
        a3 = a if batched else a.unsqueeze(0)
        BH, M, K = a3.shape
    if packed is not None:
        BHb, N, Kb = 1, packed.N, packed.K
        b3 = None
    else:
        b3 = b if b.dim() == 3 else b.unsqueeze(0)
        BHb, N, Kb = b3.shape
    if Kb != K:
        raise ValueError(f"inner-dim mismatch: a K={K}, b K={Kb}")
    if BHb not in (1, BH):
        raise ValueError(f"b batch {BHb} must be 1 or {BH}")
    p = int(sc_prec)
    L = int(stoc_len) if stoc_len is not None else (1 << p)
    if config is None:
        config = default_config(chunk_d if chunk_d > 0 else K, p)
    if int(config["sc_prec"]) != p:
        raise ValueError(f"config sc_prec={config['sc_prec']} != sc_prec={p}")
    dims = int(config["dims"])
    dev = a.device
    def _operand(t):
        if t.dtype not in (torch.float32, torch.bfloat16):
            t = t.float()
        return t.contiguous()
    if qa is None:
        a3 = _operand(a3)
    if packed is not None:
        if chunk_d:
            raise ValueError("a prepacked b runs without chunk_d")
        kseg_call = int(k_segment) if 0 < int(k_segment) < K else 0
        if not packed.matches(granularity=granularity, mode=mode, sc_prec=p, config=config,
                              group_b=group_b, k_segment=kseg_call):
            raise ValueError("prepacked b was built with other granularity / mode / sc_prec / "
                             "config / group_b / k_segment")
    else:
        b3 = _operand(b3)
    if chunk_d and 0 < int(chunk_d) < K and mode == "bipolar":
        chunk_d = int(chunk_d)
        if dims < chunk_d:
            raise ValueError(f"config has {dims} stream dims < chunk_d={chunk_d}")
        pad = (-K) % chunk_d
        if pad:
            a3 = torch.nn.functional.pad(a3, (0, pad))
            b3 = torch.nn.functional.pad(b3, (0, pad))
            K += pad
        k_segment = chunk_d
        pool_dims = chunk_d
    elif k_segment and int(k_segment) > 0:
        k_segment = int(k_segment)
        if K % k_segment:
            raise ValueError(f"k_segment={k_segment} must divide K={K}")
        if dims < k_segment:
            raise ValueError(f"config has {dims} stream dims < k_segment={k_segment}")
        pool_dims = k_segment
    else:
        k_segment = 0
        if dims < K:
            raise ValueError(f"config has {dims} stream dims < K={K}; pass chunk_d")
        pool_dims = K
    if out is None:
        odt = torch.float32 if out_dtype is None else out_dtype
        if odt not in (torch.float32, torch.bfloat16):
            raise ValueError(f"out_dtype must be float32 or bfloat16, got {odt}")
        out = torch.empty(BH, M, N, dtype=odt, device=dev)
    else:
        out = out.view(BH, M, N)
        if out.dtype not in (torch.float32, torch.bfloat16) or not out.is_contiguous():
            raise ValueError("out must be a contiguous float32 or bfloat16 tensor")
    if acc_out is not None:
        if acc_out.dtype != torch.int32 or acc_out.numel() != BH * M * N or not acc_out.is_contiguous():
            raise ValueError("acc_out must be a contiguous int32 tensor of BH*M*N elements")
    if bias is not None:
        bias = bias.to(device=dev, dtype=torch.float32).contiguous()
        if bias.numel() != N:
            raise ValueError(f"bias has {bias.numel()} elements, expected {N}")
    if row_stoc_len is not None:
        row_stoc_len = row_stoc_len.to(device=dev, dtype=torch.int32).contiguous()
        if row_stoc_len.numel() != BH * M:
            raise ValueError("row_stoc_len needs BH*M entries")
    if slice_stoc_len is not None:
        slice_stoc_len = slice_stoc_len.to(device=dev, dtype=torch.int32).contiguous()
        if slice_stoc_len.numel() != BH:
            raise ValueError("slice_stoc_len needs BH entries")
    pool = device_pool(config, dev)

    args = _lib.MatmulArgs()
    args.abi_version = _lib.ABI_VERSION
    args.engine = _lib.ENGINE[engine]
    args.a = qa.buf.data_ptr() if qa is not None else a3.data_ptr()
    args.b = packed.buf.data_ptr() if packed is not None else b3.data_ptr()
    args.batch, args.batch_b, args.M, args.N, args.K = BH, BHb, M, N, K
    args.granularity = _lib.GRANULARITY[granularity]
    args.mode = _lib.MODE[mode]
    args.sc_prec = p
    args.stoc_len = L
    args.group_a = max(int(group_a), 1)
    args.group_b = max(int(group_b), 1)
    args.k_segment = k_segment
    args.pool = pool.data_ptr()
    args.pool_dims = pool_dims
    args.row_stoc_len = _ptr(row_stoc_len)
    args.slice_stoc_len = _ptr(slice_stoc_len)
    args.bias = _ptr(bias)
    args.out = out.data_ptr()
    args.acc_out = _ptr(acc_out)
    args.io_flags = ((_lib.IO_A_BF16 if a3 is not None and a3.dtype == torch.bfloat16 else 0)
                     | (_lib.IO_A_QUANT if qa is not None else 0)
                     | (_lib.IO_B_BF16 if b3 is not None and b3.dtype == torch.bfloat16 else 0)
                     | (_lib.IO_B_PACKED if packed is not None else 0)
                     | (_lib.IO_OUT_BF16 if out.dtype == torch.bfloat16 else 0))
    lib = _lib.load()
    nbytes = lib.scmp_sc_matmul_workspace_size(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(lib.scmp_sc_matmul(ctypes.byref(args), None))  # raises with the reason
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    args.workspace = ws.data_ptr()
    args.workspace_bytes = nbytes
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.scmp_sc_matmul(ctypes.byref(args), ctypes.c_void_p(stream)))
    return out if batched else out[0]
