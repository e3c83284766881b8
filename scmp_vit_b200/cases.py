"""Run one SC matmul case of the ViT-L/14 workloads, for profiling.

    python -m scmp_vit_b200.cases qk --heads 512 --prec 8
    python -m scmp_vit_b200.cases av --heads 512 --prec 8 [--mode unipolar]
    python -m scmp_vit_b200.cases linear --rows 16448 --n 3072 --k 1024 --prec 8 [--kseg 64]
        [--prepack]
    python -m scmp_vit_b200.cases vit --config 5 --images 64

Each case builds seeded inputs on cuda:0 (257 tokens, head dim 64, the
benchmark's pools), runs the call ``--iters`` times (default 2: one warm-up,
one to capture), checks the engine's error word, and prints the time of the
last call from CUDA events.  A profiler capture (``ncu -k ... -s 1 -c 1``)
then sees exactly one warm launch of each kernel.
"""
from __future__ import annotations

import argparse
import json
import random
import sys


def _args(argv):
    p = argparse.ArgumentParser(prog="python -m scmp_vit_b200.cases")
    p.add_argument("case", choices=["qk", "av", "linear", "vit"])
    p.add_argument("--heads", type=int, default=512, help="(batch, head) slices of 257 tokens")
    p.add_argument("--prec", type=int, default=8)
    p.add_argument("--mode", default="bipolar")
    p.add_argument("--rows", type=int, default=257 * 64)
    p.add_argument("--n", type=int, default=3072)
    p.add_argument("--k", type=int, default=1024)
    p.add_argument("--kseg", type=int, default=0)
    p.add_argument("--prepack", action="store_true")
    p.add_argument("--config", type=int, default=5)
    p.add_argument("--images", type=int, default=64)
    p.add_argument("--iters", type=int, default=2)
    return p.parse_args(argv)


def main(argv=None) -> int:
    a = _args(sys.argv[1:] if argv is None else argv)
    import torch

    from . import _lib
    from . import config_helpers as ch
    from .sc import prepack_b, sc_matmul
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False  # fp32 convolutions, as the benchmark runs them
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    random.seed(0)
    L = 1 << a.prec
    if a.case == "qk":
        q = torch.randn(a.heads, 257, 64, generator=g).to(dev)
        k = torch.randn(a.heads, 257, 64, generator=g).to(dev)
        cfg = ch.make_sobol_simple_config(64, 64, a.prec)
        run = lambda: sc_matmul(q, k, granularity="per_head", sc_prec=a.prec,  # noqa: E731
                                config=cfg, stoc_len=L)
    elif a.case == "av":
        s = torch.randn(a.heads, 257, 257, generator=g).to(dev)
        probs = (s * 64 ** -0.5 * 8).softmax(dim=-1)
        vt = torch.randn(a.heads, 64, 257, generator=g).to(dev)
        cfg = ch.make_sobol_simple_config(257, 257, a.prec)
        run = lambda: sc_matmul(probs, vt, granularity="per_row", mode=a.mode,  # noqa: E731
                                sc_prec=a.prec, config=cfg, stoc_len=L)
    elif a.case == "linear":
        x = torch.randn(a.rows, a.k, generator=g).to(dev)
        w = (torch.randn(a.n, a.k, generator=g) * 0.02).to(dev)
        D = a.kseg or a.k
        cfg = ch.make_sobol_simple_config(D, D, a.prec)
        b = prepack_b(w, sc_prec=a.prec, config=cfg, k_segment=a.kseg) if a.prepack else w
        run = lambda: sc_matmul(x, b, sc_prec=a.prec, config=cfg, k_segment=a.kseg)  # noqa: E731
    else:
        import bench
        model = bench.build_model(a.config, dev, torch.float32)
        x = torch.randn(a.images, 3, 224, 224, generator=g).to(dev)

        def run():
            with torch.no_grad():
                return model(x)
    for _ in range(a.iters - 1):
        run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    status = _lib.engine_status()
    print(json.dumps({"case": a.case, "ms": e0.elapsed_time(e1), "engine_status": status,
                      "args": vars(a)}))
    return 0 if status == 0 else 3


if __name__ == "__main__":
    sys.exit(main())
