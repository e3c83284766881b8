#!/usr/bin/env python
"""Benchmark: SC-patched ViT-L/14 forward throughput (images/s) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3|4|5]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N
    python bench.py --impl reference     # CPU restatement of the SC path

Workloads (synthetic 224x224 images ~ N(0,1), random-init weights, seed 0):
  3  p7_uniform: qkv_proj, Q@K^T, Attn@V, out_proj through SC at L=128,
     256 images per GPU (weak scaling)                                [default]
  4  MP avg L~192: QK per head {128,256}, AV per row {128,256}, linears
     (qkv/proj/fc1/fc2) per row {128,192,256} seeded random, 512 per GPU
  5  p8 + head-aligned compensation on blocks 1-22 + LFSR-16 per block,
     2048 images sharded across the GPUs (strong scaling)

One step = one forward of the rank's image batch (plus, for N > 1, an NCCL
all-gather of the fp32 logits).  ``value`` is device-timed with CUDA events
(inputs resident in HBM, max over ranks); ``e2e`` is the same forward through
the public API with pinned-host images copied in and logits copied out
inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "SC ViT-L/14 images/sec"
UNIT = "images/s"
TOKENS = 257
SC_BITOPS_PER_IMAGE_L128 = 24 * (257 * 1024 * 3072 + 2 * 16 * 257 * 257 * 64
                                 + 257 * 1024 * 1024) * 128


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, choices=[3, 4, 5], default=3)
    p.add_argument("--batch", type=int, default=0, help="override images per step")
    p.add_argument("--engine", default="auto")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


WORKLOADS = {
    3: dict(name="vit_l14_p7_uniform", batch=256, scaling="weak", sc_prec=7,
            ops=("qk", "av", "proj")),
    4: dict(name="vit_l14_mp_avg192", batch=512, scaling="weak", sc_prec=8,
            ops=("qk", "av", "proj", "mlp_fc1", "mlp_fc2")),
    5: dict(name="vit_l14_p8_headaligned_lfsr16", batch=2048, scaling="strong", sc_prec=8,
            ops=("qk", "av", "proj")),
}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ----------------------------------------------------------- CPU baseline

def cpu_baseline(sc_prec: int = 7, L: int = 128, budget_s: float = 10.0) -> dict:
    """The CPU restatement (oracle, OpenMP over the host cores) on a bounded
    sample: one image's qkv_proj SC matmul, extrapolated to a whole image by
    SC bit-operations (the FP parts of the forward are not counted)."""
    import random

    import numpy as np

    from oracle import sc_oracle
    from scmp_vit_b200 import config_helpers as ch

    rng = np.random.default_rng(0)
    a = rng.standard_normal((TOKENS, 1024)).astype(np.float32)
    b = (rng.standard_normal((3072, 1024)) * 0.02).astype(np.float32)
    random.seed(0)
    cfg = ch.make_sobol_simple_config(1024, 1024, sc_prec)
    sc_oracle.sc_matmul_ref(a[:8], b[:64], sc_prec=sc_prec, pool=cfg["table"], stoc_len=L)
    reps, t0 = 0, time.perf_counter()
    while True:
        sc_oracle.sc_matmul_ref(a, b, sc_prec=sc_prec, pool=cfg["table"], stoc_len=L)
        reps += 1
        if time.perf_counter() - t0 > budget_s or reps >= 20:
            break
    dt = (time.perf_counter() - t0) / reps
    bitops = TOKENS * 1024 * 3072 * L
    per_image_s = dt * SC_BITOPS_PER_IMAGE_L128 / (bitops * (128 / L))
    return {"value": 1.0 / per_image_s, "unit": UNIT, "cores": sc_oracle.num_threads(),
            "kind": "port",
            "sample": (f"qkv_proj SC matmul of one image ([257,1024]x[3072,1024]^T, L={L}) "
                       f"x{reps} in {dt * reps:.1f}s, extrapolated by SC bit-ops per image "
                       f"({SC_BITOPS_PER_IMAGE_L128:.3g}); own CPU restatement, not reference code"),
            "bitops_per_s": bitops / dt}


# --------------------------------------------------------------- roofline

def int8_tensor_peak(dev) -> float:
    """Measured dense int8 tensor-core rate (ops/s, 2 per multiply-add):
    cuBLAS int8 GEMM 8192^3 through torch._int_mm, best of 10."""
    import torch
    n = 8192
    a = torch.randint(-3, 3, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-3, 3, (n, n), dtype=torch.int8, device=dev).t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1) / 1e3)
    del a, b
    return 2.0 * n ** 3 / best


# DRAM bytes (read + write) of one qkv_proj e2m1 pair-kernel launch per image
# (prepacked weight), from the ncu capture of 64 images
# (profiles/gemm_tc_pair_fp4_vit_l14_qkv_b64.md); traffic grows with the a
# rows, i.e. per image.
QKV_DRAM_BYTES_PER_IMAGE = (585.3e6 + 77.1e6) / 64
QKV_DRAM_SOURCE = ("ncu dram__bytes_read+write of the e2m1 pair kernel at 64 images, "
                   "scaled per image")


def _tensor_peak_alt(mult: int) -> dict:
    """Tensor-core denominator from the driver's measured bf16 GEMM rate
    (x2 for int8, x4 for e2m1: the dense rates are 2x / 4x bf16), or the
    recipe's fallback."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            bf16 = float(json.load(f)["bf16_tflops"])
        return {"value": mult * bf16,
                "source": f"of measured: MEASURED_PEAKS.json bf16_tflops x{mult}"}
    except (OSError, KeyError, ValueError, TypeError):
        return {"value": mult * 1590.0, "source": f"of fallback: 1.59 PFLOP/s bf16 x{mult}"}


def roofline(on_tc, achieved, peak_i8, peak_popc, qkv_ms, qkv_bitops, images=None,
             e2m1=False) -> dict:
    """Roofline of the dominant kernel (the qkv_proj SC matmul).  One SC
    bit-product = one multiply-add on the tensor-core engine (2 ops: int8,
    or e2m1 with unit block scales on the e2m1 CTA pairs, whose dense rate is
    twice int8's) and one counted AND bit on the CUDA-core engine."""
    base = {"kernel": "sc_matmul qkv_proj", "per_launch_ms": qkv_ms,
            "algorithmic_per_launch": qkv_bitops, "algorithmic_unit": "bit-products",
            "traffic": (QKV_DRAM_BYTES_PER_IMAGE * images) if (images and on_tc) else None,
            "traffic_source": QKV_DRAM_SOURCE,
            "int_pipe_peak_tbitops": peak_popc / 1e12,
            "x_int_pipe_roofline": (achieved / peak_popc) if achieved else None}
    if on_tc:
        mult = 2 if e2m1 else 1
        base.update({"bound": "tensor",
                     "engine": ("tcgen05 kind::mxf4 (e2m1 operands, unit block scales), "
                                "prepacked weight by TMA") if e2m1 else "tcgen05 kind::i8",
                     "achieved": 2 * achieved / 1e12 if achieved else None,
                     "peak": mult * peak_i8 / 1e12,
                     "unit": "TOP/s (e2m1)" if e2m1 else "TOP/s (int8)",
                     "frac": (2 * achieved / (mult * peak_i8)) if achieved else None,
                     "peak_source": ("2 x " if e2m1 else "") +
                                    "measured cuBLAS int8 GEMM 8192^3 (torch._int_mm), best of 10"
                                    + (" (dense e2m1 = 2 x int8 rate)" if e2m1 else "")})
        alt = _tensor_peak_alt(4 if e2m1 else 2)
        if achieved:
            alt["frac"] = 2 * achieved / 1e12 / alt["value"]
        base["peak_alt_tops"] = alt
    else:
        base.update({"bound": "int", "engine": "CUDA-core LOP3+POPC",
                     "achieved": achieved / 1e12 if achieved else None,
                     "peak": peak_popc / 1e12, "unit": "Tbit-op/s",
                     "frac": (achieved / peak_popc) if achieved else None,
                     "peak_source": "measured LOP3+POPC probe (scmp_probe_int_peak kind 0)"})
    return base


# ------------------------------------------------------------ reference arm

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t_all = time.perf_counter()
    wl = WORKLOADS[args.config]
    L = 2 ** wl["sc_prec"]
    samples = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(sc_prec=wl["sc_prec"], L=L, budget_s=2.0)
        if i >= args.warmup:
            samples.append(cb["value"])
    v = statistics.mean(samples)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": wl["scaling"],
            "vs_baseline": None, "dtype": "int32-count", "data": "synthetic",
            "config": {"workload": wl["name"], "global_batch": 1, "seq_len": TOKENS,
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cb["cores"], "kind": "port",
                             "sample": cb["sample"]},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": ("The reference has no CPU SC path and its Triton kernel package is not "
                     "vendored; this arm times the CPU restatement in oracle/."),
            "wall_s": time.perf_counter() - t_all}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm

def build_model(cfg_id: int, dev, dtype):
    import torch

    from scmp_vit_b200 import config_helpers as ch
    from scmp_vit_b200 import vit
    from scmp_vit_b200.mp import MPConfig, SeededRandomMPConfig

    wl = WORKLOADS[cfg_id]
    model = vit.vit_l14(seed=0).to(dev, dtype)
    p = wl["sc_prec"]
    if cfg_id == 3:
        vit.patch_vit(model, p, wl["ops"])
    elif cfg_id == 4:
        vit.patch_vit(model, p, wl["ops"],
                      attn_mp_spec={"qk": MPConfig([128, 256], [0.5, 0.5]),
                                    "av": MPConfig([128, 256], [0.5, 0.5])},
                      linear_random_mp=SeededRandomMPConfig([128, 192, 256], None, seed=0),
                      linear_ops=("qkv_proj", "out_proj", "mlp_fc1", "mlp_fc2"))
    else:
        caches: dict = {}

        def block_cfg_for(i):
            def cfg_for(D, prec, i=i):
                key = (i, D, prec)
                if key not in caches:
                    caches[key] = ch.make_lfsr_config(D, D, prec, seed=1000 + i)
                return caches[key]
            return cfg_for
        vit.patch_vit(model, p, wl["ops"], block_cfg_for=block_cfg_for,
                      comp_blocks=range(1, 23), comp_sc_prec=p)
    return model


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # stdout carries exactly one JSON line: keep NCCL's version banner off it
        # unless verbose NCCL logging was asked for
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=600))

    from scmp_vit_b200 import _lib
    from scmp_vit_b200.sc import set_default_engine

    set_default_engine(args.engine)

    wl = WORKLOADS[args.config]
    if args.batch:
        gbatch = args.batch * (world if wl["scaling"] == "weak" else 1)
    else:
        gbatch = wl["batch"] * (world if wl["scaling"] == "weak" else 1)
    from scmp_vit_b200.dist import gather_logits, shard_range
    lo, hi = shard_range(gbatch, rank, world)
    bl = hi - lo
    dtype = torch.bfloat16
    t_build = time.perf_counter()
    model = build_model(args.config, dev, dtype)
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    x_host = torch.randn(bl, 3, 224, 224, generator=g).pin_memory()
    x_dev = x_host.to(dev)
    logits_all = torch.empty(gbatch, 1000, dtype=torch.float32, device=dev)
    logits_host = torch.empty(bl, 1000, dtype=torch.float32).pin_memory()
    build_s = time.perf_counter() - t_build

    # events around every qkv_proj SC call: the dominant SC matmul
    qkv_events = []
    recording = {"on": False}

    def pre(mod, inp):
        if recording["on"]:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            qkv_events.append([e, None])

    def post(mod, inp, out):
        if recording["on"]:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            qkv_events[-1][1] = e

    for blk in model.backbone.blocks:
        blk.attn.qkv.register_forward_pre_hook(pre)
        blk.attn.qkv.register_forward_hook(post)

    # per-operator time split (CUDA events around modules, timed region only)
    split_events: dict = {"qkv_proj": [], "out_proj": [], "attention": []}

    def timed(name):
        def pre_h(mod, inp):
            if recording["on"]:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                split_events[name].append([e, None])

        def post_h(mod, inp, out):
            if recording["on"]:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                split_events[name][-1][1] = e
        return pre_h, post_h

    for blk in model.backbone.blocks:
        for name, mod in (("qkv_proj", blk.attn.qkv), ("out_proj", blk.attn.proj),
                          ("attention", blk.attn)):
            h0, h1 = timed(name)
            mod.register_forward_pre_hook(h0)
            mod.register_forward_hook(h1)

    def step(x):
        with torch.no_grad():
            y = model(x.to(dtype)).float()
        gather_logits(y, gbatch, world, out=logits_all)
        return y

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(x_dev)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    l0 = _lib.kernel_launches()
    recording["on"] = True
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step(x_dev)
    t1.record()
    barrier()
    recording["on"] = False
    launches = _lib.kernel_launches() - l0
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    value = gbatch * args.steps / (ms / 1000.0)

    split = {k: sum(a.elapsed_time(b) for a, b in v if b is not None) / args.steps
             for k, v in split_events.items()}
    split["attention_core"] = split.pop("attention") - split["qkv_proj"] - split["out_proj"]
    split["rest_of_forward"] = ms / args.steps - sum(split.values())

    # roofline of the dominant SC matmul (qkv_proj): bit-products per call
    durs = [a.elapsed_time(b) for a, b in qkv_events if b is not None]
    qkv_ms = statistics.mean(durs) if durs else float("nan")
    L_qkv = 2 ** WORKLOADS[args.config]["sc_prec"]
    if args.config == 4:
        L_qkv = 192  # expected stream length of the seeded random {128,192,256} split
    qkv_bitops = bl * TOKENS * 1024 * 3072 * L_qkv
    achieved = qkv_bitops / (qkv_ms * 1e-3) if durs else None
    peak_popc = _lib.probe_int_peak(0)
    peak_i8 = int8_tensor_peak(dev)
    on_tc = args.engine in ("auto", "tcgen05") and 5 <= WORKLOADS[args.config]["sc_prec"] <= 8
    # qkv_proj runs on the e2m1 CTA pairs at p = 7 / 8 (Lp = 128 / 256)
    e2m1 = on_tc and WORKLOADS[args.config]["sc_prec"] in (7, 8)

    # end to end: pinned host images in, logits out, through the public API
    e2e = None
    if not args.no_e2e:
        step(x_dev)
        barrier()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            xd = x_host.to(dev, non_blocking=True)
            y = step(xd)
            logits_host.copy_(y, non_blocking=True)
        s1.record()
        barrier()
        ems = torch.tensor([s0.elapsed_time(s1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e = {"value": gbatch * args.steps / (float(ems.item()) / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
               "d2h_bytes_per_step": logits_host.numel() * logits_host.element_size()}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(sc_prec=WORKLOADS[args.config]["sc_prec"], L=min(L_qkv, 256))
        cpu.pop("bitops_per_s", None)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": wl["scaling"], "vs_baseline": None,
            "dtype": "int32-count", "data": "synthetic",
            "config": {"workload": wl["name"], "global_batch": gbatch, "seq_len": TOKENS,
                       "parallelism": f"dp{world}", "sc_prec": wl["sc_prec"],
                       "engine": args.engine, "fp_glue": "bf16",
                       "l2": "inputs larger than L2 (154 MB of images per 256, GB-scale "
                             "activations per step)"},
            "e2e": e2e,
            "gpu_launches": int(launches),
            "roofline": roofline(on_tc, achieved, peak_i8, peak_popc, qkv_ms, qkv_bitops,
                                 images=bl, e2m1=e2m1),
            "ms_per_step_split": split,
            "cpu_baseline": cpu,
            "clocks": clk,
            "build_s": build_s,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
