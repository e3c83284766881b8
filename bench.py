#!/usr/bin/env python
"""Benchmark: SC-patched ViT-L/14 forward throughput (images/s) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3|4|5]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N
    python bench.py --impl reference     # the CPU restatement, block by block

Workloads (synthetic 224x224 images ~ N(0,1), random-init weights, seed 0,
fp32 FP glue with TF32 off, as the reference evaluates):
  5  p8 + head-aligned compensation on blocks 1-22 + LFSR-16 pool per block:
     qkv_proj, Q@K^T, Attn@V, out_proj through SC at L=256, 2048 images
     sharded across the GPUs (strong scaling)                          [default]
  3  p7_uniform: qkv_proj, Q@K^T, Attn@V, out_proj through SC at L=128,
     256 images per GPU (weak scaling)
  4  MP avg L~192: QK per head {128,256}, AV per row {128,256}, linears
     (qkv/proj/fc1/fc2) per row {128,192,256} seeded random, 512 per GPU

One step = one forward of the rank's image batch (plus, for N > 1, an NCCL
all-gather of the fp32 logits).  ``value`` is device-timed with CUDA events
(inputs resident in HBM, max over ranks); ``e2e`` is the same forward through
the public API with pinned-host images copied in and logits copied out
inside the timed region.  On one GPU the line also carries standalone
numbers for the other workloads (``configs``): the single per-tensor qkv SC
matmul (1), the attention core (2) and the ViT forwards of 3 and 4.
"""
from __future__ import annotations

import argparse
import json
import math
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
DEPTH = 24


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, choices=[3, 4, 5], default=5)
    p.add_argument("--batch", type=int, default=0, help="override images per step")
    p.add_argument("--engine", default="auto")
    p.add_argument("--fp-glue", choices=["fp32", "bf16"], default="fp32",
                   help="dtype of the FP ops around the SC matmuls (fp32 = the reference's)")
    p.add_argument("--e2e-steps", type=int, default=3,
                   help="steps of the end-to-end leg (at most --steps)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the standalone numbers of the other workloads (N=1 only)")
    return p.parse_args()


WORKLOADS = {
    3: dict(name="vit_l14_p7_uniform", batch=256, scaling="weak", sc_prec=7,
            ops=("qk", "av", "proj")),
    4: dict(name="vit_l14_mp_avg192", batch=512, scaling="weak", sc_prec=8,
            ops=("qk", "av", "proj", "mlp_fc1", "mlp_fc2")),
    5: dict(name="vit_l14_p8_headaligned_lfsr16", batch=2048, scaling="strong", sc_prec=8,
            ops=("qk", "av", "proj")),
}


def sc_bitops_per_image(cfg_id: int) -> float:
    """SC bit-products of one image's forward (the algorithmic work)."""
    lin = 257 * 1024 * 3072 + 257 * 1024 * 1024          # qkv_proj + out_proj
    attn = 2 * 16 * 257 * 257 * 64                        # Q@K^T + Attn@V
    mlp = 2 * 257 * 1024 * 4096                           # fc1 + fc2
    if cfg_id == 3:
        return DEPTH * (lin + attn) * 128.0
    if cfg_id == 4:  # linears at the expected L of {128,192,256}; attention {128,256}
        return DEPTH * ((lin + mlp) * 192.0 + attn * 192.0)
    comp = 257 * 1024 * 1024                              # head-aligned comp, blocks 1-22
    return (DEPTH * (lin + attn) + 22 * comp) * 256.0


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
        pw = [num(r[3]) for r in rows if num(r[3]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "power_w_max": max(pw) if pw else None, "samples": len(rows)}


# -------------------------------------------- CPU restatement, block by block

def host_cores() -> int:
    """Host threads this process may run on (overrides the OMP_NUM_THREADS=1
    that torchrun exports)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class OracleViT:
    """One image through the SC-patched ViT-L/14 of a workload, one block per
    step, on the host cores: the SC matmuls by the C restatement in
    ``oracle/`` (OpenMP over every core), the FP glue by torch in fp32.
    Same pools, stream lengths and op set as the GPU workload."""

    def __init__(self, cfg_id: int, nthreads: int):
        import random

        import numpy as np
        import torch

        from scmp_vit_b200 import config_helpers as ch
        from scmp_vit_b200 import vit
        from scmp_vit_b200.mp import SeededRandomMPConfig

        torch.set_num_threads(nthreads)
        self.np, self.torch = np, torch
        self.cfg_id = cfg_id
        self.p = WORKLOADS[cfg_id]["sc_prec"]
        self.nthreads = nthreads
        self.model = vit.vit_l14(seed=0).float()
        random.seed(0)
        self._pools: dict = {}
        self._ch = ch
        self.rand_mp = SeededRandomMPConfig([128, 192, 256], None, seed=0) if cfg_id == 4 else None
        g = torch.Generator().manual_seed(1)
        self.comp = {}
        if cfg_id == 5:
            for i in range(1, 23):
                self.comp[i] = (torch.randn(1024, 1024, generator=g) * 0.002, torch.zeros(1024))
        img = torch.randn(1, 3, 224, 224, generator=torch.Generator().manual_seed(1234))
        with torch.no_grad():
            bb = self.model.backbone
            x = bb.patch_embed(img).flatten(2).transpose(1, 2)
            self.x0 = torch.cat([bb.cls_token.expand(1, -1, -1), x], dim=1) + bb.pos_embed
        self.x = self.x0.clone()
        self.block = 0
        self.calls = 0

    def pool(self, D: int, p: int, block: int):
        key = (D, p, block if self.cfg_id == 5 else -1)
        if key not in self._pools:
            if self.cfg_id == 5:
                cfg = self._ch.make_lfsr_config(D, D, p, seed=1000 + block)
            else:
                cfg = self._ch.make_sobol_simple_config(D, D, p)
            self._pools[key] = self._ch.pool_table(cfg)
        return self._pools[key]

    def _linear(self, x2, lin, block, salt):
        """SC linear (per-row scales), uniform or seeded-random per-row levels."""
        from oracle import sc_oracle
        np = self.np
        a = x2.numpy()
        w = lin.weight.detach().numpy()
        bias = lin.bias.detach().numpy()
        K = a.shape[1]
        if self.rand_mp is None:
            _, y = sc_oracle.sc_matmul_ref(a, w, sc_prec=self.p, pool=self.pool(K, self.p, block),
                                           stoc_len=1 << self.p, bias=bias,
                                           nthreads=self.nthreads)
            return self.torch.from_numpy(y[0])
        row_L = self.rand_mp.assign(a.shape[0], "cpu", salt=salt).numpy()
        pools = {p: self.pool(K, p, block) for p in (7, 8)}
        _, y = sc_oracle.sc_matmul_rows_ref(a, w, row_L, pools, bias=bias, nthreads=self.nthreads)
        return self.torch.from_numpy(np.ascontiguousarray(y))

    def step(self) -> None:
        """Run the next block of the current image (a new image after 24)."""
        from oracle import sc_oracle
        from scmp_vit_b200.mp import classify_rows_by_metric, quantile_levels_batched
        torch, np = self.torch, self.np
        i = self.block
        blk = self.model.backbone.blocks[i]
        p = self.p
        with torch.no_grad():
            x = self.x
            h = blk.norm1(x)[0]                                          # [257, 1024]
            qkv = self._linear(h, blk.attn.qkv, i, 4 * i)
            q, k, v = qkv.reshape(TOKENS, 3, 16, 64).permute(1, 2, 0, 3).unbind(0)  # [16,257,64]
            if self.cfg_id == 4:
                metric = q.abs().amax(dim=(1, 2))
                head_L = classify_rows_by_metric(metric, [128, 256], [0.5, 0.5]).row_levels
                att = torch.empty(16, TOKENS, TOKENS)
                for L in (128, 256):
                    idx = torch.nonzero(head_L == L).flatten()
                    pp = 7 if L == 128 else 8
                    _, y = sc_oracle.sc_matmul_ref(q[idx].numpy(), k[idx].numpy(),
                                                   granularity="per_head", sc_prec=pp,
                                                   pool=self.pool(64, pp, i), stoc_len=L,
                                                   nthreads=self.nthreads)
                    att[idx] = torch.from_numpy(y)
            else:
                _, y = sc_oracle.sc_matmul_ref(q.contiguous().numpy(), k.contiguous().numpy(),
                                               granularity="per_head", sc_prec=p,
                                               pool=self.pool(64, p, i), stoc_len=1 << p,
                                               nthreads=self.nthreads)
                att = torch.from_numpy(y)
            att = (att * blk.attn.scale).softmax(dim=-1)
            vt = v.transpose(-1, -2).contiguous()                        # [16, 64, 257]
            if self.cfg_id == 4:
                from scmp_vit_b200.attention import av_row_score
                row_L = quantile_levels_batched(av_row_score(att), [128, 256], [0.5, 0.5])
                o = torch.empty(16, TOKENS, 64)
                pools = {pp: self.pool(TOKENS, pp, i) for pp in (7, 8)}
                for s in range(16):
                    _, y = sc_oracle.sc_matmul_rows_ref(att[s].numpy(), vt[s].numpy(),
                                                        row_L[s].numpy(), pools,
                                                        nthreads=self.nthreads)
                    o[s] = torch.from_numpy(np.ascontiguousarray(y))
            else:
                _, y = sc_oracle.sc_matmul_ref(att.numpy(), vt.numpy(), sc_prec=p,
                                               pool=self.pool(TOKENS, p, i), stoc_len=1 << p,
                                               nthreads=self.nthreads)
                o = torch.from_numpy(y)
            o = o.transpose(0, 1).reshape(TOKENS, 1024)
            y = x + blk.ls1(self._linear(o, blk.attn.proj, i, 4 * i + 1)[None])
            h2 = blk.norm2(y)[0]
            if self.cfg_id == 4:
                hid = blk.mlp.act(self._linear(h2, blk.mlp.fc1, i, 4 * i + 2))
                mlp = self._linear(hid, blk.mlp.fc2, i, 4 * i + 3)
            else:
                mlp = blk.mlp(h2)
            y = y + blk.ls2(mlp[None])
            if i in self.comp:
                w, b = self.comp[i]
                _, c = sc_oracle.sc_matmul_segments_ref(x[0].numpy(), w.numpy(), 64, sc_prec=p,
                                                        pool=self.pool(64, p, i),
                                                        stoc_len=1 << p, bias=b.numpy(),
                                                        nthreads=self.nthreads)
                y = y + torch.from_numpy(c)
            self.x = y
        self.block += 1
        if self.block == DEPTH:
            self.block = 0
            self.x = self.x0.clone()


def cpu_blocks(cfg_id: int, warmup: int, steps: int, nthreads: int) -> dict:
    """Time ``steps`` block-steps of one image on the host cores (after
    ``warmup`` untimed ones); images/s = (steps / 24) / time."""
    ov = OracleViT(cfg_id, nthreads)
    for _ in range(warmup):
        ov.step()
    durs = []
    for _ in range(steps):
        t0 = time.perf_counter()
        ov.step()
        durs.append(time.perf_counter() - t0)
    total = sum(durs)
    return {"value": (steps / DEPTH) / total, "unit": UNIT, "cores": nthreads, "kind": "port",
            "ms_per_step": 1000.0 * total / steps,
            "sample": (f"{steps} transformer blocks of one image of the {WORKLOADS[cfg_id]['name']} "
                       f"forward (blocks {warmup % DEPTH}..), each a step: SC matmuls by the C "
                       "restatement in oracle/ (OpenMP), FP glue by torch fp32; images/s = "
                       "blocks / 24 / time; own CPU restatement, not reference code")}


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


def measured_peaks() -> dict:
    """e2m1 tensor-core denominators: the dense e2m1 rate is 4x the dense
    bf16 rate, so 4 x the driver's measured bf16 GEMM rate (burst for a
    kernel timed alone, sustained for one inside a long step), or the
    recipe's fallback."""
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(path.read_text())
        return {"burst": 4 * float(d["bf16_tflops"]),
                "sustained": 4 * float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "of measured: MEASURED_PEAKS.json bf16 TF/s x4 (dense e2m1 = 4 x bf16)"}
    except (OSError, KeyError, ValueError, TypeError):
        return {"burst": 4 * 1590.0, "sustained": 4 * 1400.0,
                "source": "of fallback: 1.59 (burst) / 1.4 (sustained) PFLOP/s bf16 x4"}


# DRAM bytes (read + write) of one qkv_proj e2m1 pair-kernel launch
# (prepacked weight): at p = 7 from the ncu capture of 64 images
# (profiles/gemm_tc_pair_fp4_vit_l14_qkv_b64.md), scaled per image; at p = 8
# the two-point fit of captures at 128 and 512 images
# (profiles/gemm_tc_pair_fp4_qkv_p8_prepacked_dram.md): traffic is linear in
# the images with a fixed part (the weight's reads).
QKV_DRAM_BYTES_PER_IMAGE = (585.3e6 + 77.1e6) / 64
QKV_DRAM_SOURCE = ("ncu dram__bytes_read+write of the e2m1 pair kernel at 64 images (p=7), "
                   "scaled per image; an estimate: weight re-reads do not scale with images")
QKV_P8_DRAM_FIXED = 759_570_048
QKV_P8_DRAM_PER_IMAGE = 17_689_163
QKV_P8_DRAM_SOURCE = ("ncu dram__bytes_read+write of the prepacked e2m1 pair kernel (p=8) at 128 "
                      "and 512 images: 3.02e9 and 9.82e9 B; linear fit 0.760 GB + 17.69 MB per "
                      "image, evaluated at this launch's images")


def roofline(kind: str, ms: float, bitops: float, peaks: dict, peak_i8: float, peak_popc: float,
             images: int | None, sc_prec: int, uniform: bool = True) -> dict:
    """Roofline of one SC matmul kind.  One SC bit-product is one multiply-add
    on the tensor-core engine (2 ops: e2m1 operands with unit block scales)."""
    ach = 2 * bitops / (ms * 1e-3) / 1e12 if ms and ms > 0 else None
    out = {"kernel": kind, "per_launch_ms": ms, "algorithmic_per_launch": bitops,
           "algorithmic_unit": "bit-products (x2 ops)", "bound": "tensor",
           "engine": "tcgen05 kind::mxf4 (e2m1 operands in {-1,0,+1}, unit block scales)",
           "achieved": ach, "peak": peaks["burst"], "unit": "TOP/s (e2m1)",
           "frac": ach / peaks["burst"] if ach else None, "peak_source": peaks["source"] +
           " (burst)", "frac_of_sustained": ach / peaks["sustained"] if ach else None,
           "frac_of_int8_cublas_x2": ach / (2 * peak_i8 / 1e12) if (ach and peak_i8) else None,
           "x_int_pipe_roofline": (bitops / (ms * 1e-3)) / peak_popc if (ms and peak_popc)
           else None,
           # the e2m1 MMA itself (scmp_probe_int_peak kind 3: M128 x N256 x K64
           # kind::mxf4, back to back on every SM) runs faster than 4 x the
           # bf16 GEMM; this is the fraction of that raw issue rate
           "frac_of_mxf4_probe": (ach / (2 * peaks["mxf4_probe"] / 1e12)
                                  if (ach and peaks.get("mxf4_probe")) else None),
           "mxf4_probe_tops": (2 * peaks["mxf4_probe"] / 1e12 if peaks.get("mxf4_probe")
                               else None),
           "int_pipe_peak_tbitops": peak_popc / 1e12 if peak_popc else None}
    if images and kind.startswith("sc_matmul qkv_proj") and sc_prec == 7:
        out["traffic"] = QKV_DRAM_BYTES_PER_IMAGE * images
        out["traffic_source"] = QKV_DRAM_SOURCE
    elif (images and uniform and sc_prec == 8
          and kind.startswith("sc_matmul qkv_proj (SCLinear, prepacked")):
        out["traffic"] = float(QKV_P8_DRAM_FIXED + QKV_P8_DRAM_PER_IMAGE * images)
        out["traffic_source"] = QKV_P8_DRAM_SOURCE
    else:
        out["traffic"] = None
    return out


# ------------------------------------------------------------ reference arm

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t_all = time.perf_counter()
    wl = WORKLOADS[args.config]
    cores = host_cores()
    cb = cpu_blocks(args.config, args.warmup, args.steps, cores)
    v = cb["value"]
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cb["ms_per_step"], "higher_is_better": True,
            "scaling": wl["scaling"], "vs_baseline": None, "dtype": "int32-count",
            "data": "synthetic",
            "config": {"workload": wl["name"], "global_batch": 1, "seq_len": TOKENS,
                       "parallelism": f"cpu x{cores} threads", "sc_prec": wl["sc_prec"],
                       "fp_glue": "fp32", "step": "one transformer block of one image"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": cb["sample"]},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": ("The reference has no CPU SC path and its Triton kernel package is not "
                     "vendored; this arm times the CPU restatement in oracle/ block by block."),
            "wall_s": time.perf_counter() - t_all}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm

def build_model(cfg_id: int, dev, dtype, depth: int = DEPTH, comp_blocks=None):
    """The workload's SC-patched ViT-L/14 (``depth`` blocks of full width;
    config 5's compensation on ``comp_blocks``, default blocks 1-22)."""
    from scmp_vit_b200 import config_helpers as ch
    from scmp_vit_b200 import vit
    from scmp_vit_b200.mp import MPConfig, SeededRandomMPConfig

    wl = WORKLOADS[cfg_id]
    model = vit.vit_l14(seed=0, depth=depth).to(dev, dtype)
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
                      comp_blocks=range(1, 23) if comp_blocks is None else comp_blocks,
                      comp_sc_prec=p)
    return model


def engine_status_or_fail(where: str) -> int:
    """The engine's sticky error word after a timed region; a non-zero word
    (a bounded device wait gave up) invalidates the measurement."""
    from scmp_vit_b200 import _lib
    st = _lib.engine_status()
    if st != 0:
        print(json.dumps({"error": f"engine error word 0x{st:x} after {where}: a bounded "
                                   "device wait gave up; the measurement is invalid"}),
              file=sys.stderr, flush=True)
    return st


def flush_l2(buf) -> None:
    buf.add_(1.0)  # 256 MB read + write: evicts the 126 MB L2


def measure_config1(dev, peaks, peak_i8, peak_popc) -> dict:
    """One SC linear of the qkv_proj shape, per-tensor scales: X fp32
    [257,1024] ~ N(0,1), W [3072,1024] ~ trunc_normal(std 0.02), scrambled
    Sobol pool (seed 0), L=128.  Each of 20 timed calls follows an L2 flush."""
    import random

    import torch

    from scmp_vit_b200 import config_helpers as ch
    from scmp_vit_b200.sc import sc_matmul
    torch.manual_seed(0)
    x = torch.randn(257, 1024).to(dev)
    w = torch.nn.init.trunc_normal_(torch.empty(3072, 1024), std=0.02).to(dev)
    random.seed(0)
    cfg = ch.make_sobol_simple_config(1024, 1024, 7)
    flush = torch.zeros(64 * 1024 * 1024, device=dev)
    call = lambda: sc_matmul(x, w, granularity="per_tensor", sc_prec=7, config=cfg,  # noqa: E731
                             stoc_len=128)
    for _ in range(3):
        call()
    durs = []
    for _ in range(20):
        flush_l2(flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        e1.synchronize()
        durs.append(e0.elapsed_time(e1))
    ms = statistics.mean(durs)
    bitops = 257 * 3072 * 1024 * 128
    return {"workload": "sc_linear_qkv_per_tensor_L128", "shape": "[257,1024]x[3072,1024]^T",
            "ms_per_call": ms, "ms_min": min(durs), "calls": len(durs),
            "bitops_per_s": bitops / (ms * 1e-3), "l2": "flushed before every call",
            "roofline": roofline("sc_matmul per_tensor qkv shape", ms, bitops, peaks, peak_i8,
                                 peak_popc, None, 7)}


def measure_config2(dev, peaks, peak_i8, peak_popc) -> dict:
    """Attention core: Q, K, V fp32 [64,16,257,64] ~ N(0,1); SC Q@K^T
    (per_head, pool (64,7), L=128), x scale, fp32 softmax, SC Attn@V (per_row,
    probabilities unipolar, pool (257,7), L=128).  The scale, the softmax and
    the quantisation of the probabilities run as one fused pass (the same
    bits as torch.softmax followed by sc_matmul on the probabilities)."""
    import torch

    from scmp_vit_b200 import sc_linear as scl
    from scmp_vit_b200.attention import sc_qk, sc_softmax_av
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(64, 16, 257, 64, generator=g).to(dev) for _ in range(3))
    scale = 64 ** -0.5
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def core(rec=None):
        e = [ev() for _ in range(3)]
        e[0].record()
        a = sc_qk(q, k, 7, cfg_for=scl._get_config)
        e[1].record()
        o = sc_softmax_av(a, scale, v, 7, mode="unipolar", cfg_for=scl._get_config)
        e[2].record()
        if rec is not None:
            rec.append(e)
        return o
    for _ in range(3):
        core()
    rec: list = []
    for _ in range(10):
        core(rec)
    torch.cuda.synchronize()
    tot = statistics.mean(e[0].elapsed_time(e[2]) for e in rec)
    qk = statistics.mean(e[0].elapsed_time(e[1]) for e in rec)
    bit = 1024 * 257 * 257 * 64 * 128
    return {"workload": "attention_core_b64_h16_L128", "shape": "[64,16,257,64]",
            "ms_per_call": tot, "qk_ms": qk, "softmax_av_ms": tot - qk, "calls": len(rec),
            "bitops_per_s": 2 * bit / (tot * 1e-3), "l2": "inputs and scores larger than L2",
            "roofline_qk": roofline("sc_matmul per_head Q@K^T", qk, bit, peaks, peak_i8,
                                    peak_popc, None, 7)}


def measure_vit(cfg_id: int, dev, dtype, batch: int, warmup: int, steps: int) -> dict:
    """Images/s of a whole SC ViT forward at ``batch`` images (inputs resident)."""
    import torch
    model = build_model(cfg_id, dev, dtype)
    x = torch.randn(batch, 3, 224, 224, generator=torch.Generator().manual_seed(1234)).to(dev,
                                                                                           dtype)
    with torch.no_grad():
        for _ in range(warmup):
            model(x)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            y = model(x)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    st = engine_status_or_fail(f"config {cfg_id}")
    del model, x, y
    torch.cuda.empty_cache()
    return {"workload": WORKLOADS[cfg_id]["name"], "images_per_step": batch, "warmup": warmup,
            "steps": steps, "ms_per_step": ms / steps, "value": batch * steps / (ms / 1000.0),
            "unit": UNIT, "engine_status": st,
            "sc_bitops_per_s": sc_bitops_per_image(cfg_id) * batch * steps / (ms / 1000.0)}


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    # fp32 FP glue as the reference evaluates it: no TF32 anywhere
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False

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
    _lib.engine_status(reset=True)

    wl = WORKLOADS[args.config]
    per_rank = args.batch or wl["batch"]
    gbatch = per_rank * (world if wl["scaling"] == "weak" else 1)
    from scmp_vit_b200.dist import gather_logits, shard_range
    lo, hi = shard_range(gbatch, rank, world)
    bl = hi - lo
    dtype = torch.float32 if args.fp_glue == "fp32" else torch.bfloat16
    t_build = time.perf_counter()
    model = build_model(args.config, dev, dtype)
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    x_host = torch.randn(bl, 3, 224, 224, generator=g).pin_memory()
    x_dev = x_host.to(dev)
    logits_all = torch.empty(gbatch, 1000, dtype=torch.float32, device=dev)
    logits_host = torch.empty(bl, 1000, dtype=torch.float32).pin_memory()
    build_s = time.perf_counter() - t_build

    recording = {"on": False}
    # per-operator CUDA events around modules, timed region only
    split_events: dict = {"qkv_proj": [], "out_proj": [], "attention": [], "comp": []}

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
        mods = [("qkv_proj", blk.attn.qkv), ("out_proj", blk.attn.proj), ("attention", blk.attn)]
        if blk.comp is not None:
            mods.append(("comp", blk.comp))
        for name, mod in mods:
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
    status = engine_status_or_fail("the timed region")
    ms = t0.elapsed_time(t1)
    ms_t = torch.tensor([ms, float(status)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t[0].item())
    status = int(ms_t[1].item())
    value = gbatch * args.steps / (ms / 1000.0)

    def mean_ms(name):
        d = [a.elapsed_time(b) for a, b in split_events[name] if b is not None]
        return (statistics.mean(d) if d else float("nan")), d
    qkv_ms, _ = mean_ms("qkv_proj")
    split = {k: sum(a.elapsed_time(b) for a, b in v if b is not None) / args.steps
             for k, v in split_events.items()}
    split["attention_core"] = split.pop("attention") - split["qkv_proj"] - split["out_proj"]
    split["rest_of_forward"] = ms / args.steps - sum(split.values())
    comp_ms, comp_d = mean_ms("comp")
    out_ms, _ = mean_ms("out_proj")

    p = wl["sc_prec"]
    L_qkv = 192 if args.config == 4 else (1 << p)  # config 4: expected L of {128,192,256}
    qkv_bitops = bl * TOKENS * 1024 * 3072 * L_qkv
    peak_popc = _lib.probe_int_peak(0)
    peak_i8 = int8_tensor_peak(dev)
    peaks = measured_peaks()
    peaks["mxf4_probe"] = _lib.probe_int_peak(3)
    roof = roofline("sc_matmul qkv_proj (SCLinear, prepacked weight by TMA)", qkv_ms, qkv_bitops,
                    peaks, peak_i8, peak_popc, bl, p, uniform=args.config != 4)
    if comp_d:
        roof["comp_head_aligned"] = {
            "per_launch_ms": comp_ms, "vs_out_proj": comp_ms / out_ms if out_ms else None,
            "achieved": 2 * bl * TOKENS * 1024 * 1024 * (1 << p) / (comp_ms * 1e-3) / 1e12,
            "unit": "TOP/s (e2m1)"}

    # end to end: pinned host images in, logits out, through the public API
    e2e = None
    if not args.no_e2e and status == 0:
        n_e2e = max(1, min(args.e2e_steps, args.steps))
        step(x_dev)
        barrier()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(n_e2e):
            xd = x_host.to(dev, non_blocking=True)
            y = step(xd)
            logits_host.copy_(y, non_blocking=True)
        s1.record()
        barrier()
        ems = torch.tensor([s0.elapsed_time(s1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e = {"value": gbatch * n_e2e / (float(ems.item()) / 1000.0), "unit": UNIT,
               "steps": n_e2e,
               "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
               "d2h_bytes_per_step": logits_host.numel() * logits_host.element_size()}
        st2 = engine_status_or_fail("the end-to-end region")
        status = status or st2

    # standalone numbers of the other workloads (one GPU only)
    extras = None
    if world == 1 and not args.no_extras and status == 0:
        del model, x_dev, logits_all
        torch.cuda.empty_cache()
        extras = {}
        for key, fn in (("1", lambda: measure_config1(dev, peaks, peak_i8, peak_popc)),
                        ("2", lambda: measure_config2(dev, peaks, peak_i8, peak_popc)),
                        ("3", lambda: measure_vit(3, dev, dtype, 256, 3, 5)),
                        ("4", lambda: measure_vit(4, dev, dtype, 512, 2, 2))):
            if str(args.config) == key:
                continue
            try:
                extras[key] = fn()
            except Exception as exc:  # reported in the line, never hidden
                extras[key] = {"error": f"{type(exc).__name__}: {exc}"}
        st3 = engine_status_or_fail("the standalone workloads")
        status = status or st3

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_blocks(args.config, 1, 6, host_cores())
        cpu.pop("ms_per_step", None)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": wl["scaling"], "vs_baseline": None,
            "dtype": "int32-count", "data": "synthetic",
            "config": {"workload": wl["name"], "global_batch": gbatch, "seq_len": TOKENS,
                       "parallelism": f"dp{world}", "sc_prec": p, "engine": args.engine,
                       "fp_glue": args.fp_glue, "tf32": False,
                       "sc_bitops_per_image": sc_bitops_per_image(args.config),
                       "l2": "inputs larger than L2 (602 KB per image, GB-scale activations "
                             "per step)"},
            "e2e": e2e,
            "gpu_launches": int(launches),
            "engine_status": status,
            "roofline": roof,
            "ms_per_step_split": split,
            "cpu_baseline": cpu,
            "configs": extras,
            "clocks": clk,
            "build_s": build_s,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0 if status == 0 else 3


if __name__ == "__main__":
    sys.exit(main())
