"""Golden vectors of the reference's own patchers (test infrastructure).

Runs the reference's unmodified Python -- ``cls/sc_attention_patch.py``
(``patch_model`` and the attention forward it installs),
``sc_integration/sc_linear.py`` (``SCLinear`` with fixed, range and chunked
forms) and ``det/sc_patch/sc_matmul.py`` (``SCMatMul``) -- on the CPU, with
the ``scmp_kernels`` import surface served by ``scmp_vit_b200.shim`` and every
``scmp_kernels.sc.sc_matmul`` call answered by the oracle (``oracle/``) and
recorded: operands, keyword arguments, pool, result.  The reference tree
cannot travel to the GPU machine, so its behaviour travels as these
fixtures: ``tests/test_dropin_gpu.py`` replays every recorded call through
the engine, runs this package's modules configured as the reference's
patcher configures them, and compares bit for bit.

The CPU glue (layer norm, softmax, GELU, the patch convolution) is pinned to
one thread and the AVX2 code paths so that it gives the same bits on any
x86-64 machine with AVX2.

    python tests/golden/make_dropin.py [REFERENCE_DIR [OUT_DIR]]
        # defaults: /root/reference, this directory
"""
from __future__ import annotations

import os

# pin the CPU glue before torch loads (see module docstring)
import sys  # noqa: E402
from pathlib import Path  # noqa: E402

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from dropin_cases import (IMAGES, MODEL, PINNED_ENV, cls_cases, det_cases,  # noqa: E402
                          det_mp, linear_cases, tiny_images, tiny_model)

for _k, _v in PINNED_ENV.items():
    os.environ[_k] = _v

import hashlib  # noqa: E402
import importlib  # noqa: E402
import json  # noqa: E402
import random  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle import sc_oracle  # noqa: E402
from scmp_vit_b200 import config_helpers as ch  # noqa: E402


class Recorder:
    """``scmp_kernels.sc.sc_matmul`` answered by the oracle, every call kept."""

    def __init__(self):
        self.calls: list = []
        self.arrays: dict = {}
        self.case = None

    def _put(self, arr: np.ndarray) -> str:
        arr = np.ascontiguousarray(arr)
        h = hashlib.sha1(arr.tobytes() + str(arr.shape).encode() + arr.dtype.str.encode())
        name = "t" + h.hexdigest()[:16]
        self.arrays.setdefault(name, arr)
        return name

    def __call__(self, a, b, *, granularity="per_row", mode="bipolar", sc_prec=8, config=None,
                 group_a=1, group_b=1, chunk_d=0, stoc_len=None):
        A = a.detach().float().cpu().numpy()
        B = b.detach().float().cpu().numpy()
        p = int(sc_prec)
        L = int(stoc_len) if stoc_len is not None else (1 << p)
        table = ch.pool_table(config)
        K = A.shape[-1]
        if chunk_d and 0 < int(chunk_d) < K and mode == "bipolar":
            cd = int(chunk_d)
            pad = (-K) % cd
            if pad:
                A = np.concatenate([A, np.zeros(A.shape[:-1] + (pad,), np.float32)], -1)
                B = np.concatenate([B, np.zeros(B.shape[:-1] + (pad,), np.float32)], -1)
            _, y = sc_oracle.sc_matmul_segments_ref(A, B, cd, mode=mode, sc_prec=p, pool=table,
                                                    stoc_len=L)
        else:
            _, y = sc_oracle.sc_matmul_ref(A, B, granularity=granularity, mode=mode, sc_prec=p,
                                           pool=table, pool_dims=K, group_a=group_a,
                                           group_b=group_b, stoc_len=L)
        out = y if a.dim() == 3 else y[0]
        self.calls.append({
            "case": self.case, "a": self._put(a.detach().float().cpu().numpy()),
            "b": self._put(b.detach().float().cpu().numpy()), "out": self._put(out),
            "pool": self._put(table), "granularity": granularity, "mode": mode,
            "sc_prec": p, "stoc_len": stoc_len, "group_a": int(group_a),
            "group_b": int(group_b), "chunk_d": int(chunk_d)})
        return torch.from_numpy(np.ascontiguousarray(out))


def load_reference(ref: Path, recorder: Recorder):
    """Import the reference's modules against the shim, with the recorder as
    ``scmp_kernels.sc.sc_matmul`` (bound by their ``from ... import``)."""
    from scmp_vit_b200 import shim
    shim.install()
    sys.modules["scmp_kernels.sc"].sc_matmul = recorder
    for p in (str(ref), str(ref / "cls")):
        if p not in sys.path:
            sys.path.insert(0, p)
    patch = importlib.import_module("sc_attention_patch")
    scl = importlib.import_module("sc_integration.sc_linear")
    mpl = importlib.import_module("sc_integration.mp_linear")
    det = importlib.import_module("det.sc_patch.sc_matmul")
    for mod in (patch, scl, det):
        assert mod.sc_matmul is recorder, f"{mod.__name__} did not bind the recorder"
    return patch, scl, mpl, det


def generate(ref: Path) -> tuple[dict, dict]:
    rec = Recorder()
    patch, scl, mpl, det = load_reference(ref, rec)
    meta = {"model": MODEL, "images": list(IMAGES), "env": PINNED_ENV, "cases": {}}
    x = tiny_images()
    for name, seed, kw in cls_cases(mpl):
        rec.case = name
        scl._CFG_CACHE.clear()
        random.seed(seed)
        model = tiny_model()
        stats = patch.patch_model(model, **kw)
        n0 = len(rec.calls)
        with torch.no_grad():
            logits = model(x)
        meta["cases"][name] = {"kind": "cls", "seed": seed, "stats": stats,
                               "calls": [n0, len(rec.calls)], "images": rec._put(x.numpy()),
                               "logits": rec._put(logits.numpy())}
    for name, seed, kw, sa, sb, soft in det_cases():
        rec.case = name
        det._CFG_CACHE.clear()
        random.seed(seed)
        g = torch.Generator().manual_seed(seed)
        A = torch.randn(*sa, generator=g)
        if soft:
            A = (A * 3).softmax(-1)
        B = torch.randn(*sb, generator=g)
        kw = dict(kw)
        if "op" in kw:
            kw["mp_cfg"] = det_mp(mpl)
        n0 = len(rec.calls)
        with torch.no_grad():
            y = det.SCMatMul(**kw)(A, B)
        meta["cases"][name] = {"kind": "det", "seed": seed,
                               "kwargs": {k: v for k, v in kw.items() if k != "mp_cfg"},
                               "mp": "op" in kw, "calls": [n0, len(rec.calls)],
                               "A": rec._put(A.numpy()), "B": rec._put(B.numpy()),
                               "out": rec._put(y.numpy())}
    for name, seed, kw, din, dout, rows in linear_cases(mpl):
        rec.case = name
        scl._CFG_CACHE.clear()
        random.seed(seed)
        g = torch.Generator().manual_seed(seed)
        lin = torch.nn.Linear(din, dout)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(dout, din, generator=g) * 0.05)
            lin.bias.copy_(torch.randn(dout, generator=g) * 0.1)
        xin = torch.randn(rows, din, generator=g)
        n0 = len(rec.calls)
        with torch.no_grad():
            y = scl.SCLinear(lin, **kw)(xin)
        meta["cases"][name] = {
            "kind": "linear", "seed": seed, "in": din, "out_features": dout,
            "kwargs": {k: (v if isinstance(v, (int, str)) else repr(v)) for k, v in kw.items()},
            "calls": [n0, len(rec.calls)], "weight": rec._put(lin.weight.detach().numpy()),
            "bias": rec._put(lin.bias.detach().numpy()), "x": rec._put(xin.numpy()),
            "out": rec._put(y.numpy())}
    meta["calls"] = rec.calls
    return meta, rec.arrays


def main(argv):
    ref = Path(argv[1]) if len(argv) > 1 else Path("/root/reference")
    out = Path(argv[2]) if len(argv) > 2 else HERE
    meta, arrays = generate(ref)
    np.savez_compressed(out / "dropin.npz", **arrays)
    (out / "dropin.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"{len(meta['calls'])} recorded calls, {len(arrays)} arrays, "
          f"{(out / 'dropin.npz').stat().st_size} bytes")


if __name__ == "__main__":
    main(sys.argv)
