"""Import-time aliases that make the reference's Python modules run on this engine.

The reference imports its kernel package as ``scmp_kernels`` (an un-vendored
submodule, ``.gitmodules:4-7``):

    from scmp_kernels.sc import sc_matmul                       # sc_linear.py:32
    from scmp_kernels.sc.config_helpers import make_sobol_simple_config
    from scmp_kernels.mp import MPConfig, ...                   # mp_linear.py:37-48
    from scmp_kernels.sc import sc_matmul, det_kernel_tuning    # det/experiments/_p8_breakdown.py:25

``install()`` registers those module names, backed by this package, so the
reference's own ``sc_integration/*.py``, ``cls/sc_attention_patch.py`` and
``det/sc_patch/*`` import and run unmodified.  With
``replace_sc_integration=True`` the ``sc_integration.*`` modules named in
the reference (``sc_linear``, ``mp_linear``, ``mp_config``,
``head_aligned_comp``, ``noise_matmul``) are served by this package's
versions instead (grouped mixed-precision launches, one-launch head-aligned
compensation).
"""
from __future__ import annotations

import sys
import types

from . import config_helpers, mp, sc

__all__ = ["install", "uninstall"]

_INSTALLED: list[str] = []


def _module(name: str, **attrs) -> types.ModuleType:
    m = types.ModuleType(name)
    m.__dict__.update(attrs)
    return m


def install(replace_sc_integration: bool = False) -> None:
    """Register the ``scmp_kernels`` import surface (idempotent)."""
    sc_mod = _module("scmp_kernels.sc", sc_matmul=sc.sc_matmul,
                     det_kernel_tuning=config_helpers.det_kernel_tuning,
                     config_helpers=config_helpers, __path__=[])
    root = _module("scmp_kernels", sc=sc_mod, mp=mp, __path__=[])
    mods = {
        "scmp_kernels": root,
        "scmp_kernels.sc": sc_mod,
        "scmp_kernels.sc.config_helpers": config_helpers,
        "scmp_kernels.mp": mp,
    }
    if replace_sc_integration:
        from . import head_aligned_comp, mp_linear, noise_matmul, sc_linear
        pkg = _module("sc_integration", __path__=[])
        sub = {"sc_linear": sc_linear, "mp_linear": mp_linear, "mp_config": mp,
               "head_aligned_comp": head_aligned_comp, "noise_matmul": noise_matmul}
        for k, v in sub.items():
            setattr(pkg, k, v)
            mods[f"sc_integration.{k}"] = v
        mods["sc_integration"] = pkg
    for name, mod in mods.items():
        if sys.modules.get(name) is not mod:
            sys.modules[name] = mod
            _INSTALLED.append(name)


def uninstall() -> None:
    """Remove every alias ``install`` added."""
    while _INSTALLED:
        sys.modules.pop(_INSTALLED.pop(), None)
