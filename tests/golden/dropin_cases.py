"""Cases of the drop-in fixtures (``make_dropin.py``) and this package's side
of them (test infrastructure, no import-time side effects).

Each case names its seed, which both sides pass to ``random.seed`` after
clearing the pool cache, so pools drawn from Python's ``random`` come out the
same when created in the same order.  ``mp`` is the module that provides
``MPConfig`` / ``RangeMPConfig``: the reference's ``sc_integration.mp_linear``
when recording, ``scmp_vit_b200.mp_linear`` when replaying.
"""
from __future__ import annotations

# tiny DINOv2-style model: 2 blocks, d=64, 2 heads of 32, MLP 128, 42x42
# images (9 patches + CLS = 10 tokens), 10 classes, 2 images
MODEL = dict(seed=0, dim=64, depth=2, heads=2, hidden=128, img=42, num_classes=10)
IMAGES = (2, 3, 42, 42)
IMAGE_SEED = 7
PINNED_ENV = {"ATEN_CPU_CAPABILITY": "avx2", "OMP_NUM_THREADS": "1", "MKL_NUM_THREADS": "1",
              "MKL_CBWR": "AVX2", "DNNL_MAX_CPU_ISA": "AVX2"}


def tiny_model():
    import torch

    from scmp_vit_b200 import vit
    torch.set_num_threads(1)
    return vit.vit_l14(**MODEL)


def tiny_images():
    import torch
    return torch.randn(*IMAGES, generator=torch.Generator().manual_seed(IMAGE_SEED))


def cls_cases(mp):
    """(name, seed, ``patch_model`` keyword arguments) of the cls forwards."""
    MPConfig, RangeMPConfig = mp.MPConfig, mp.RangeMPConfig
    return [
        ("cls_uniform_p7", 11, dict(sc_prec=7, sc_qk=True, sc_av=True, sc_mlp=True,
                                    sc_qkv_proj=True, sc_out_proj=True, sc_mlp_mode="unipolar")),
        ("cls_mp_p8", 12, dict(
            sc_prec=8,
            sc_ops_per_block={"qk": [1, 1], "av": [1, 1], "proj": [1, 1],
                              "mlp_fc1": [1, 0], "mlp_fc2": [0, 1]},
            linear_mp_spec={
                "proj": MPConfig([128, 192, 256]),
                "mlp_fc1": {"fixed": MPConfig([128, 256], [0.25, 0.75]),
                            "range": RangeMPConfig([256, 128], base_threshold=0.6),
                            "range_group_size": 32},
                "mlp_fc2": RangeMPConfig([256, 192, 128], base_threshold=0.5)},
            attn_mp_spec={"qk": MPConfig([128, 256], [0.5, 0.5]),
                          "av": MPConfig([128, 256], [0.5, 0.5])})),
    ]


def det_cases():
    """(name, seed, ``SCMatMul`` kwargs, A shape, B shape, A softmaxed)."""
    return [
        ("det_uniform_p8", 21, dict(sc_prec=8), (2, 2, 12, 16), (2, 2, 16, 12), False),
        ("det_stoc_len_192", 22, dict(sc_prec=8, stoc_len=192), (1, 3, 12, 16), (1, 3, 16, 12),
         False),
        ("det_qk_mp", 23, dict(sc_prec=8, op="qk"), (2, 4, 12, 16), (2, 4, 16, 12), False),
        ("det_av_mp_unipolar", 24, dict(sc_prec=8, op="av", mode="unipolar"), (2, 2, 12, 12),
         (2, 2, 12, 16), True),
    ]


def det_mp(mp):
    return mp.MPConfig([128, 256], [0.5, 0.5])


def linear_cases(mp):
    """(name, seed, ``SCLinear`` kwargs, in_features, out_features, rows)."""
    return [
        ("linear_chunk_d", 31, dict(sc_prec=7, chunk_d=16), 72, 40, 30),
        ("linear_range_and_rows", 32,
         dict(sc_prec=8, mp_cfg=mp.MPConfig([128, 192, 256], [0.2, 0.3, 0.5]),
              range_mp_cfg=mp.RangeMPConfig([256, 128], base_threshold=0.6),
              range_mp_group_size=16, operator="mlp_fc1"), 48, 64, 40),
    ]


# ------------------------------------------------ this package's side (cls)

LINEAR_OPS = ("mlp_fc1", "mlp_fc2", "qkv_proj", "out_proj")


def _linear_mp(spec, mp):
    """{op: SCLinear MP keyword arguments} from a ``linear_mp_spec`` (the
    reference's spelling: an MP config, or a dict of fixed / adaptive / range
    / range_group_size; ``proj`` = qkv_proj and out_proj)."""
    out = {}
    for key, v in (spec or {}).items():
        ops = ("qkv_proj", "out_proj") if key == "proj" else (key,)
        if isinstance(v, mp.MPConfig):
            kw = dict(mp_cfg=v)
        elif isinstance(v, mp.AdaptiveMPConfig):
            kw = dict(adaptive_mp_cfg=v)
        elif isinstance(v, mp.RangeMPConfig):
            kw = dict(range_mp_cfg=v)
        else:
            kw = dict(mp_cfg=v.get("fixed"), adaptive_mp_cfg=v.get("adaptive"),
                      range_mp_cfg=v.get("range"),
                      range_mp_group_size=int(v.get("range_group_size", 0)))
        for op in ops:
            out[op] = dict(kw, operator=op)
    return out


def patch_like_reference(model, mp, *, sc_prec, sc_qk=True, sc_av=False, sc_mlp=False,
                         sc_qkv_proj=False, sc_out_proj=False, sc_mlp_mode="bipolar",
                         sc_proj_mode="bipolar", sc_ops_per_block=None, linear_mp_spec=None,
                         attn_mp_spec=None):
    """Install this package's SC modules where the reference's ``patch_model``
    (``cls/sc_attention_patch.py:459-636``) installs its own, for the options
    the cases use: per-block op vectors or uniform op flags, linear and
    attention MP specs, linear modes."""
    from scmp_vit_b200.attention import make_sc_attention_forward
    from scmp_vit_b200.sc_linear import SCLinear

    blocks = list(model.backbone.blocks)
    n = len(blocks)
    if sc_ops_per_block is not None:
        def vec(k):
            v = sc_ops_per_block.get(k, 0)
            v = [v] * n if isinstance(v, (int, bool)) else list(v)
            return [int(bool(x)) for x in (v * n if len(v) == 1 else v)]
        on = {k: vec(k) for k in ("qk", "av", "proj", "mlp_fc1", "mlp_fc2")}
    else:
        on = {"qk": [int(sc_qk)] * n, "av": [int(sc_av)] * n,
              "proj": [int(sc_qkv_proj or sc_out_proj)] * n,
              "mlp_fc1": [int(sc_mlp)] * n, "mlp_fc2": [int(sc_mlp)] * n}
    lmp = _linear_mp(linear_mp_spec, mp)
    qk_mp = (attn_mp_spec or {}).get("qk")
    av_mp = (attn_mp_spec or {}).get("av")
    for i, blk in enumerate(blocks):
        attn = blk.attn
        if on["qk"][i] or on["av"][i]:
            fwd = make_sc_attention_forward(sc_prec, sc_av=bool(on["av"][i]),
                                            sc_qk=bool(on["qk"][i]),
                                            qk_mp_cfg=qk_mp if on["qk"][i] else None,
                                            av_mp_cfg=av_mp if on["av"][i] else None)
            attn.forward = fwd.__get__(attn, type(attn))
        if on["proj"][i]:
            if sc_ops_per_block is not None or sc_qkv_proj:
                attn.qkv = SCLinear(attn.qkv, sc_prec, mode=sc_proj_mode,
                                    **lmp.get("qkv_proj", {}))
            if sc_ops_per_block is not None or sc_out_proj:
                attn.proj = SCLinear(attn.proj, sc_prec, mode=sc_proj_mode,
                                     **lmp.get("out_proj", {}))
        if on["mlp_fc1"][i]:
            blk.mlp.fc1 = SCLinear(blk.mlp.fc1, sc_prec, mode=sc_mlp_mode,
                                   **lmp.get("mlp_fc1", {}))
        if on["mlp_fc2"][i]:
            blk.mlp.fc2 = SCLinear(blk.mlp.fc2, sc_prec, mode=sc_mlp_mode,
                                   **lmp.get("mlp_fc2", {}))
    return model


# --------------------------------------- the oracle as the engine (CPU tests)

def oracle_sc_matmul(a, b, *, granularity="per_row", mode="bipolar", sc_prec=8, config=None,
                     group_a=1, group_b=1, chunk_d=0, stoc_len=None, bias=None,
                     row_stoc_len=None, slice_stoc_len=None, out=None, k_segment=0,
                     out_dtype=None, **unused):
    """``scmp_vit_b200.sc.sc_matmul`` restated on the oracle, for CPU tests
    of the Python layers: same keywords and conventions (per-row / per-slice
    stream length with 0 = pruned row -> bias, < 0 = row left as in ``out``;
    chunk_d / k_segment summed per segment; bias added after the rescale)."""
    import numpy as np
    import torch

    from oracle import sc_oracle
    from scmp_vit_b200 import config_helpers as ch
    if out_dtype not in (None, torch.float32) or unused.get("acc_out") is not None:
        raise NotImplementedError("the oracle stand-in returns fp32 results only")
    A = a.detach().float().cpu().numpy()
    B = b.detach().float().cpu().numpy()
    batched = A.ndim == 3
    A3 = A if batched else A[None]
    B3 = B if B.ndim == 3 else B[None]
    BH, M, K = A3.shape
    N = B3.shape[1]
    p = int(sc_prec)
    table = ch.pool_table(config)
    bias_np = None if bias is None else bias.detach().float().cpu().numpy()
    if row_stoc_len is not None:
        Lr = row_stoc_len.cpu().numpy().astype(np.int64).reshape(-1)
    elif slice_stoc_len is not None:
        Lr = np.repeat(slice_stoc_len.cpu().numpy().astype(np.int64), M)
    else:
        Lr = None
    L = int(stoc_len) if stoc_len is not None else (1 << p)
    Lcalc = None if Lr is None else np.where(Lr > 0, Lr, 1).astype(np.int32)
    seg = int(chunk_d) if (chunk_d and 0 < int(chunk_d) < K and mode == "bipolar") else int(k_segment)
    if seg and seg < K:
        pad = (-K) % seg
        if pad:
            A3 = np.concatenate([A3, np.zeros((BH, M, pad), np.float32)], -1)
            B3 = np.concatenate([B3, np.zeros(B3.shape[:2] + (pad,), np.float32)], -1)
        _, y = sc_oracle.sc_matmul_segments_ref(A3, B3, seg, mode=mode, sc_prec=p, pool=table,
                                                stoc_len=L, bias=bias_np, L_row=Lcalc)
    else:
        _, y = sc_oracle.sc_matmul_ref(A3, B3, granularity=granularity, mode=mode, sc_prec=p,
                                       pool=table, pool_dims=K, group_a=group_a,
                                       group_b=group_b, stoc_len=L, bias=bias_np, L_row=Lcalc)
    y = np.ascontiguousarray(y.reshape(BH * M, N), dtype=np.float32)
    keep = None
    if Lr is not None:
        pruned = Lr == 0
        y[pruned] = 0.0
        if bias_np is not None:
            y[pruned] = np.float32(0.0) + bias_np[None, :]
        keep = Lr >= 0
    res = torch.from_numpy(y)
    if out is None:
        if keep is not None and not keep.all():
            raise ValueError("rows left untouched need an out tensor")
        res = res.reshape(BH, M, N)
        return res if batched else res[0]
    o = out.view(BH * M, N)
    if keep is None:
        o.copy_(res)
    else:
        idx = torch.from_numpy(np.nonzero(keep)[0])
        o.index_copy_(0, idx, res.index_select(0, idx))
    o3 = out.view(BH, M, N)
    return o3 if batched else o3[0]
