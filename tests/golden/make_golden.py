"""Regenerate the SC matmul fixtures in this directory.

Each case stores seeded inputs, the pool, and the oracle's accumulators and
outputs, so the spec (oracle/sc_oracle.c) and the engine can both be checked
against fixed bytes.  The reference ships no golden data for this path (its
kernel package is an un-vendored submodule), so these vectors pin this
project's written spec, not the reference's kernel.

    python tests/golden/make_golden.py
"""
import json
import random
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import sc_oracle as so  # noqa: E402
from scmp_vit_b200 import config_helpers as ch  # noqa: E402

CASES = [
    dict(name="sc_case_qkv_p7", M=9, N=12, K=64, sc_prec=7, stoc_len=128, mode="bipolar",
         granularity="per_tensor", kind="sobol", seed=0, batch=0),
    dict(name="sc_case_p8_l192", M=7, N=10, K=40, sc_prec=8, stoc_len=192, mode="bipolar",
         granularity="per_row", kind="sobol", seed=1, batch=0),
    dict(name="sc_case_qk_head", M=6, N=6, K=64, sc_prec=7, stoc_len=128, mode="bipolar",
         granularity="per_head", kind="sobol", seed=2, batch=3),
    dict(name="sc_case_av_unipolar", M=5, N=8, K=17, sc_prec=7, stoc_len=128, mode="unipolar",
         granularity="per_row", kind="sobol", seed=3, batch=2),
    dict(name="sc_case_lfsr_p8", M=6, N=9, K=64, sc_prec=8, stoc_len=256, mode="bipolar",
         granularity="per_row", kind="lfsr16", seed=4, batch=0),
]


def main():
    for c in CASES:
        rng = np.random.default_rng(c["seed"])
        shape_a = (c["batch"], c["M"], c["K"]) if c["batch"] else (c["M"], c["K"])
        shape_b = (c["batch"], c["N"], c["K"]) if c["batch"] else (c["N"], c["K"])
        a = rng.standard_normal(shape_a).astype(np.float32)
        b = rng.standard_normal(shape_b).astype(np.float32)
        if c["mode"] == "unipolar":
            a = np.abs(a)
        random.seed(c["seed"])
        if c["kind"] == "lfsr16":
            cfg = ch.make_lfsr_config(c["K"], c["K"], c["sc_prec"], seed=c["seed"])
        else:
            cfg = ch.make_sobol_simple_config(c["K"], c["K"], c["sc_prec"])
        acc, y = so.sc_matmul_ref(a, b, granularity=c["granularity"], mode=c["mode"],
                                  sc_prec=c["sc_prec"], pool=cfg["table"],
                                  stoc_len=c["stoc_len"])
        np.savez_compressed(HERE / f"{c['name']}.npz", a=a, b=b, pool=cfg["table"], acc=acc, y=y)
        (HERE / f"{c['name']}.json").write_text(json.dumps(c, indent=1) + "\n")
        print(c["name"], acc.shape)


if __name__ == "__main__":
    main()
