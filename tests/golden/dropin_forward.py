"""One cls drop-in case with this package's modules (test infrastructure).

Builds the tiny model of ``dropin_cases``, installs this package's SC modules
where the reference's ``patch_model`` puts its own, and runs the forward with
the FP glue on the CPU -- pinned like the fixture run, so it gives the same
bits -- and every SC matmul on the GPU engine (operands copied to the device
and back).  Prints the logits as JSON hex words for the caller to compare
with the reference's.

    python tests/golden/dropin_forward.py CASE [engine|oracle]
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from dropin_cases import PINNED_ENV, cls_cases, patch_like_reference, tiny_model  # noqa: E402

for _k, _v in PINNED_ENV.items():
    os.environ[_k] = _v

import json  # noqa: E402
import random  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402


def engine_on_device(real):
    """``sc_matmul`` for CPU tensors: run the call on cuda:0, copy back."""
    from scmp_vit_b200.sc import PackedWeight
    dev = torch.device("cuda", 0)

    def call(a, b, **kw):
        out = kw.pop("out", None)
        kw = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in kw.items()}
        out_d = None if out is None else out.to(dev)
        y = real(a.to(dev), b if isinstance(b, PackedWeight) else b.to(dev), out=out_d, **kw)
        if out is not None:
            out.copy_(out_d.view(out.shape))
            return out if y.dim() == out.dim() else out.view(y.shape)
        return y.cpu()
    return call


def run(case: str, backend: str = "engine") -> np.ndarray:
    """Logits of ``case``; ``backend`` "engine" runs the SC matmuls on the GPU,
    "oracle" on the CPU restatement (no GPU; the Python layers alone under
    test)."""
    from dropin_cases import oracle_sc_matmul

    from scmp_vit_b200 import attention, mp_linear
    from scmp_vit_b200 import sc_linear as scl
    wrapped = engine_on_device(scl.sc_matmul) if backend == "engine" else oracle_sc_matmul
    attention.sc_matmul = wrapped
    scl.sc_matmul = wrapped
    spec = {name: (seed, kw) for name, seed, kw in cls_cases(mp_linear)}
    seed, kw = spec[case]
    fix = np.load(HERE / "dropin.npz")
    meta = json.loads((HERE / "dropin.json").read_text())
    x = torch.from_numpy(fix[meta["cases"][case]["images"]])
    scl._CFG_CACHE.clear()
    random.seed(seed)
    model = tiny_model()
    patch_like_reference(model, mp_linear, **kw)
    with torch.no_grad():
        return model(x).numpy()


if __name__ == "__main__":
    y = run(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "engine")
    print(json.dumps({"shape": list(y.shape),
                      "bits": y.astype(np.float32).view(np.uint32).ravel().tolist()}))
