"""DINOv2-style ViT-L/14 with a linear head, and the SC patcher the benchmark
uses.

The model carries the attribute names the reference's patchers rely on
(``cls/sc_attention_patch.py:335-341,459-636``): ``backbone.blocks[i].attn``
with ``qkv``, ``proj``, ``proj_drop``, ``num_heads``, ``scale``; an ``Mlp``
class with ``fc1`` / ``fc2``; and a 1000-way head on the concatenation of the
CLS token and the mean patch token (2048 -> 1000).  Weights are random
(seeded); there are no checkpoints in this environment.

``patch_vit`` installs the SC operators per block: ``qkv_proj`` /
``out_proj`` / ``mlp_fc1`` / ``mlp_fc2`` as ``SCLinear``, Q@K^T and Attn@V
through the batched attention core, optional per-block pools (e.g. an
LFSR-16 pool seeded per block) and optional head-aligned compensation
``out = block(x) + comp(x)``.
"""
from __future__ import annotations

from typing import Callable, Dict, Iterable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import make_sc_attention_forward
from .head_aligned_comp import HeadAlignedSCLinear
from .mp import SeededRandomMPConfig, quantile_counts, set_current_block_idx
from .sc_linear import PackedWeights, SCLinear, _get_config, sc_linear_rows


def _fp_linear(lin: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """``lin(x)``; a plain ``nn.Linear`` with a bias on a CUDA input runs as a
    matmul followed by an in-place bias add.  On B200 with fp32 operands that
    is the same cuBLAS GEMM kernel as ``F.linear`` and the same single
    rounding of ``acc + bias`` as its bias epilogue (identical bits), without
    the epilogue's extra pass: ViT-L/14 fc1 at 128 images 5.07 -> 4.72 ms,
    fc2 4.42 -> 4.33 ms.  CPU inputs keep ``F.linear``, whose ``addmm`` adds
    the bias inside the GEMM, and so do 16-bit ones (the epilogue adds the
    bias before the output is rounded)."""
    if (type(lin) is not nn.Linear or lin.bias is None or not x.is_cuda
            or x.dtype != torch.float32 or lin.weight.dtype != torch.float32):
        return lin(x)
    x2 = x.reshape(-1, x.shape[-1])
    y = torch.mm(x2, lin.weight.t()).add_(lin.bias)
    return y.reshape(*x.shape[:-1], y.shape[-1])


# Whether the blocks run their fp32 elementwise steps fused on the engine
# (scmp_bias_gelu, scmp_scale_residual); identical bits either way.
FUSED_GLUE = True


def set_fused_glue(flag: bool) -> None:
    """Turn the fused fp32 block glue on or off (results are identical)."""
    global FUSED_GLUE
    FUSED_GLUE = bool(flag)


def _stream(t: torch.Tensor):
    import ctypes
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def bias_gelu_(t: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``t = gelu(t + bias)`` in place (fp32 CUDA ``[..., C]``, exact GELU):
    the bias add and torch's erf-form GELU in one pass, same bits."""
    from . import _lib
    C = t.shape[-1]
    _lib.check(_lib.load().scmp_bias_gelu(t.data_ptr(), bias.data_ptr(), t.numel() // C, C,
                                          _stream(t)))
    return t


def scale_residual(x: torch.Tensor, y: torch.Tensor, gamma: torch.Tensor,
                   bias: Optional[torch.Tensor] = None, extra: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``(x + (y [+ bias]) * gamma) [+ extra]`` (fp32 CUDA ``[..., C]``, all
    contiguous and of one shape): a block's layer-scaled residual add, with an
    unfused bias and a compensation term, in one pass; each step rounded as
    the separate torch ops round it.  ``out`` may be ``x`` or ``y``."""
    from . import _lib
    C = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _lib.check(_lib.load().scmp_scale_residual(
        out.data_ptr(), x.data_ptr(), y.data_ptr(), None if bias is None else bias.data_ptr(),
        gamma.data_ptr(), None if extra is None else extra.data_ptr(), x.numel() // C, C,
        _stream(x)))
    return out


def _plain_linear(m: nn.Module) -> bool:
    return (type(m) is nn.Linear and m.bias is not None and m.weight.dtype == torch.float32
            and m.weight.is_contiguous() and m.bias.is_contiguous())


class Mlp(nn.Module):
    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(hidden, dim)

    def forward(self, x):
        return _fp_linear(self.fc2, self.act(_fp_linear(self.fc1, x)))


class Attention(nn.Module):
    def __init__(self, dim: int, num_heads: int):
        super().__init__()
        self.num_heads = num_heads
        self.scale = (dim // num_heads) ** -0.5
        self.qkv = nn.Linear(dim, 3 * dim)
        self.proj = nn.Linear(dim, dim)
        self.attn_drop = nn.Identity()
        self.proj_drop = nn.Identity()

    def forward(self, x, attn_bias=None):
        B, N, C = x.shape
        H = self.num_heads
        qkv = self.qkv(x).reshape(B, N, 3, H, C // H).permute(2, 0, 3, 1, 4)
        q, k, v = qkv.unbind(0)
        out = F.scaled_dot_product_attention(q, k, v)
        return self.proj_drop(self.proj(out.transpose(1, 2).reshape(B, N, C)))


class LayerScale(nn.Module):
    def __init__(self, dim: int, init: float):
        super().__init__()
        self.gamma = nn.Parameter(torch.full((dim,), float(init)))

    def forward(self, x):
        return x * self.gamma


class Block(nn.Module):
    def __init__(self, dim: int, heads: int, hidden: int, ls_init: float):
        super().__init__()
        self.norm1 = nn.LayerNorm(dim, eps=1e-6)
        self.attn = Attention(dim, heads)
        self.ls1 = LayerScale(dim, ls_init)
        self.norm2 = nn.LayerNorm(dim, eps=1e-6)
        self.mlp = Mlp(dim, hidden)
        self.ls2 = LayerScale(dim, ls_init)
        self.comp: Optional[nn.Module] = None  # head-aligned compensation, if installed
        self.block_idx = 0

    def forward(self, x):
        set_current_block_idx(self.block_idx)
        if self._fused_glue_applies(x):
            return self._forward_fused_glue(x)
        y = x + self.ls1(self.attn(self.norm1(x)))
        y = y + self.ls2(self.mlp(self.norm2(y)))
        if self.comp is not None:
            y = y + self.comp(x).to(y.dtype)
        return y

    def _fused_glue_applies(self, x: torch.Tensor) -> bool:
        return (FUSED_GLUE and x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
                and not torch.is_grad_enabled() and type(self.ls1) is LayerScale
                and type(self.ls2) is LayerScale)

    def _forward_fused_glue(self, x: torch.Tensor) -> torch.Tensor:
        """The forward above with its fp32 elementwise steps on the engine:
        ``x + ls1(a)`` in one pass, fc1's bias with the GELU, fc2's bias with
        ``ls2``, the residual add and the compensation term in another (the
        matmuls stay cuBLAS fp32).  Bit-identical to the unfused forward."""
        a = self.attn(self.norm1(x)).contiguous()
        y = scale_residual(x, a, self.ls1.gamma)
        h = self.norm2(y)
        mlp = self.mlp
        ub = None
        if (type(mlp) is Mlp and _plain_linear(mlp.fc1) and _plain_linear(mlp.fc2)
                and type(mlp.act) is nn.GELU and mlp.act.approximate == "none"):
            h2 = h.reshape(-1, h.shape[-1])
            t = bias_gelu_(torch.mm(h2, mlp.fc1.weight.t()), mlp.fc1.bias)
            u = torch.mm(t, mlp.fc2.weight.t())
            ub = mlp.fc2.bias
        else:
            u = mlp(h)
        e = None
        if self.comp is not None:
            e = self.comp(x).to(torch.float32).contiguous()
        return scale_residual(y, u.reshape(y.shape).contiguous(), self.ls2.gamma, bias=ub,
                              extra=e, out=y)


class Backbone(nn.Module):
    def __init__(self, img: int = 224, patch: int = 14, dim: int = 1024, depth: int = 24,
                 heads: int = 16, hidden: int = 4096, ls_init: float = 1.0):
        super().__init__()
        self.patch_embed = nn.Conv2d(3, dim, kernel_size=patch, stride=patch)
        n = (img // patch) ** 2
        self.cls_token = nn.Parameter(torch.zeros(1, 1, dim))
        self.pos_embed = nn.Parameter(torch.zeros(1, n + 1, dim))
        self.blocks = nn.ModuleList([Block(dim, heads, hidden, ls_init) for _ in range(depth)])
        for i, b in enumerate(self.blocks):
            b.block_idx = i
        self.norm = nn.LayerNorm(dim, eps=1e-6)

    def forward(self, x):
        x = self.patch_embed(x).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.expand(x.shape[0], -1, -1), x], dim=1) + self.pos_embed
        for b in self.blocks:
            x = b(x)
        return self.norm(x)


class ViTClassifier(nn.Module):
    """ViT-L/14 backbone + linear head on [CLS, mean(patch)] (2048 -> 1000)."""

    def __init__(self, num_classes: int = 1000, **kw):
        super().__init__()
        self.backbone = Backbone(**kw)
        dim = self.backbone.norm.normalized_shape[0]
        self.linear_head = nn.Linear(2 * dim, num_classes)

    def forward(self, x):
        t = self.backbone(x)
        feat = torch.cat([t[:, 0], t[:, 1:].mean(dim=1)], dim=-1)
        return self.linear_head(feat)


def vit_l14(seed: int = 0, num_classes: int = 1000, **kw) -> ViTClassifier:
    """Random-initialised DINOv2-style ViT-L/14 (24 blocks, d=1024, 16 heads,
    MLP 4096, 257 tokens at 224x224)."""
    g = torch.Generator().manual_seed(seed)
    m = ViTClassifier(num_classes=num_classes, **kw)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("gamma"):
                continue
            if p.dim() >= 2:
                p.copy_(torch.nn.init.trunc_normal_(torch.empty_like(p), std=0.02, generator=g))
            elif "norm" in name and name.endswith("weight"):
                p.fill_(1.0)
            else:
                p.zero_()
        m.backbone.pos_embed.copy_(torch.randn(m.backbone.pos_embed.shape, generator=g) * 0.02)
        m.backbone.cls_token.copy_(torch.randn(m.backbone.cls_token.shape, generator=g) * 0.02)
    return m.eval()


class _RowMPLinear(nn.Module):
    """SC linear whose rows carry a seeded random level in each call."""

    def __init__(self, linear: nn.Linear, cfg: SeededRandomMPConfig, salt: int,
                 cfg_for: Callable[[int, int], dict]):
        super().__init__()
        self.weight = linear.weight
        self.bias = linear.bias
        self.cfg = cfg
        self.salt = salt
        self.cfg_for = cfg_for
        self.calls = 0
        self.packed = PackedWeights(self.weight, "bipolar")  # one per precision class

    def forward(self, x):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if x2.dtype not in (torch.float32, torch.bfloat16):
            x2 = x2.float()
        row_L = self.cfg.assign(x2.shape[0], x2.device, salt=(self.salt << 16) + self.calls)
        self.calls += 1
        counts = quantile_counts(x2.shape[0], self.cfg.stoc_len_levels, self.cfg.level_fractions)
        y = sc_linear_rows(x2, self.weight, row_L, self.cfg.stoc_len_levels, "bipolar",
                           bias=self.bias, cfg_for=self.cfg_for, host_counts=counts,
                           packed_for=self.packed)
        return y.to(x.dtype).reshape(*shp[:-1], -1)


def patch_vit(model: ViTClassifier, sc_prec: int, ops: Iterable[str] = ("qk", "av", "proj"), *,
              av_mode: str = "bipolar", attn_mp_spec: Optional[Dict] = None,
              linear_random_mp: Optional[SeededRandomMPConfig] = None,
              linear_ops: Iterable[str] = ("qkv_proj", "out_proj"),
              block_cfg_for: Optional[Callable[[int], Callable[[int, int], dict]]] = None,
              comp_blocks: Iterable[int] = (), comp_sc_prec: Optional[int] = None,
              comp_seed: int = 1) -> dict:
    """Install SC operators on every block (see module docstring).

    ``ops`` uses the reference's op names (``cls/sc_attention_patch.py:332``,
    with ``"proj"`` meaning qkv_proj + out_proj).  ``block_cfg_for(i)`` gives
    block ``i`` its own pool factory ``(D, p) -> config``.  ``comp_blocks``
    get a ``HeadAlignedSCLinear`` compensation (random weights) that reuses the
    block's ``(head_dim, p)`` pool.
    """
    ops = set(ops)
    stats = {"attn": 0, "qkv_proj": 0, "out_proj": 0, "mlp_fc1": 0, "mlp_fc2": 0, "comp": 0}
    attn_mp_spec = attn_mp_spec or {}
    linear_ops = set(linear_ops)
    if "proj" in ops:
        ops |= {"qkv_proj", "out_proj"}
    comp_blocks = set(comp_blocks)
    g = torch.Generator().manual_seed(comp_seed)
    for i, blk in enumerate(model.backbone.blocks):
        cfg_for = block_cfg_for(i) if block_cfg_for is not None else _get_config
        attn = blk.attn
        if "qk" in ops or "av" in ops:
            fwd = make_sc_attention_forward(
                sc_prec, sc_av="av" in ops, sc_qk="qk" in ops,
                qk_mp_cfg=attn_mp_spec.get("qk"), av_mp_cfg=attn_mp_spec.get("av"),
                av_mode=av_mode, cfg_for=cfg_for)
            attn.forward = fwd.__get__(attn, type(attn))
            stats["attn"] += 1

        def wrap(lin: nn.Linear, op: str, salt: int):
            if linear_random_mp is not None and op in linear_ops:
                return _RowMPLinear(lin, linear_random_mp, salt, cfg_for)
            cfg = None if block_cfg_for is None else cfg_for(lin.in_features, sc_prec)
            return SCLinear(lin, sc_prec, mode="bipolar", cfg_override=cfg, operator=op)

        if "qkv_proj" in ops:
            attn.qkv = wrap(attn.qkv, "qkv_proj", 4 * i)
            stats["qkv_proj"] += 1
        if "out_proj" in ops:
            attn.proj = wrap(attn.proj, "out_proj", 4 * i + 1)
            stats["out_proj"] += 1
        if "mlp_fc1" in ops:
            blk.mlp.fc1 = wrap(blk.mlp.fc1, "mlp_fc1", 4 * i + 2)
            stats["mlp_fc1"] += 1
        if "mlp_fc2" in ops:
            blk.mlp.fc2 = wrap(blk.mlp.fc2, "mlp_fc2", 4 * i + 3)
            stats["mlp_fc2"] += 1
        if i in comp_blocks:
            dim = attn.proj.weight.shape[0] if hasattr(attn.proj, "weight") else 1024
            lin = nn.Linear(dim, dim).to(next(model.parameters()).device)
            with torch.no_grad():
                lin.weight.copy_(torch.randn(dim, dim, generator=g) * 0.002)
                lin.bias.zero_()
            head_dim = dim // attn.num_heads
            p = comp_sc_prec or sc_prec
            blk.comp = HeadAlignedSCLinear(lin, p, n_heads=attn.num_heads,
                                           cfg_override=cfg_for(head_dim, p))
            stats["comp"] += 1
    return stats
