"""Drop-in modules that let the unmodified upstream ``sparc3d`` code run on B200 kernels.

Same mechanism as the reference's ``hi3d_mac.torch_backend`` (src/hi3d_mac/torch_backend/__init__.py:24-64):
a module object registered in ``sys.modules`` under the name the upstream code imports.
:func:`register_flash_attn` installs ``flash_attn`` backed by the tcgen05 attention kernel.
"""

from __future__ import annotations

import importlib.machinery
import sys
import types


def _module(name: str) -> types.ModuleType:
    module = types.ModuleType(name)
    module.__spec__ = importlib.machinery.ModuleSpec(name, loader=None)
    module.__hi3d_b200_shim__ = True
    return module


def register_flash_attn() -> None:
    """Register ``flash_attn`` (varlen qkv-packed and kv-packed functions)."""
    from . import attention

    existing = sys.modules.get("flash_attn")
    if existing is not None and not getattr(existing, "__hi3d_b200_shim__", False):
        raise RuntimeError("a real flash_attn is already imported; refusing to shadow it")
    module = _module("flash_attn")
    module.flash_attn_varlen_qkvpacked_func = attention.flash_attn_varlen_qkvpacked_func
    module.flash_attn_varlen_kvpacked_func = attention.flash_attn_varlen_kvpacked_func
    sys.modules["flash_attn"] = module
