"""Drop-in modules that let the unmodified upstream ``sparc3d`` code run on B200 kernels.

Same mechanism as the reference's ``hi3d_mac.torch_backend`` (src/hi3d_mac/torch_backend/__init__.py:24-64):
a module object registered in ``sys.modules`` under the name the upstream code imports.
:func:`register_flash_attn` installs ``flash_attn`` backed by the tcgen05 attention kernel and
:func:`register_spconv` the ``spconv.pytorch`` subset backed by the GPU neighbour map and the
gather-GEMM convolution.
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


def register_spconv() -> None:
    """Register ``spconv``, ``spconv.pytorch`` (+ ``ops``, ``core``) backed by the B200 sparse kernels
    (the module set of src/hi3d_mac/torch_backend/__init__.py:34-55)."""
    from . import sparse_conv

    for name in ("spconv", "spconv.pytorch"):
        existing = sys.modules.get(name)
        if existing is not None and not getattr(existing, "__hi3d_b200_shim__", False):
            raise RuntimeError(f"a real {name} is already imported; refusing to shadow it")
    pytorch = _module("spconv.pytorch")
    for name in ("SubMConv3d", "SparseConvTensor", "ConvAlgo"):
        setattr(pytorch, name, getattr(sparse_conv, name))
    ops = _module("spconv.pytorch.ops")
    ops.get_indice_pairs = sparse_conv.get_indice_pairs
    core = _module("spconv.pytorch.core")
    core.IndiceData = sparse_conv.IndiceData
    pytorch.ops = ops
    pytorch.core = core
    root = _module("spconv")
    root.pytorch = pytorch
    sys.modules.update({"spconv": root, "spconv.pytorch": pytorch, "spconv.pytorch.ops": ops,
                        "spconv.pytorch.core": core})


def install() -> None:
    """Register both drop-in modules (``flash_attn`` and ``spconv``)."""
    register_flash_attn()
    register_spconv()


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
