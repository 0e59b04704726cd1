"""Operators of the sparse VAE decoder (``PTv3MeshDecoder``) on B200.

Mirrors the GPU-side pieces of ``SparconvVAEDecoderMLX`` (src/hi3d_mac/mlx_backend/vae.py) and
its helpers:

* :func:`group_stats`, :func:`group_norm_swish`, :func:`conv_gn_swish` -- ``conv(swish(GN(x)))``
  (vae.py:142-192, kernels.py:242-296): statistics by a deterministic two-stage reduction, the
  activated features written once, then the gathered tcgen05 convolution;
* :func:`child_neighbour_table` -- the octree child table from the parent table and the
  occupancy masks (sparse.py:46-95), on the GPU;
* :func:`serialization`, :func:`window_index`, :func:`window_attention` -- the serialized
  window attention of the mid attention blocks (vae.py:49-88, :249-266).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib, sparse

PATCH = 48
ORDERS = ("z", "z-trans")


def _groups(c: int) -> int:
    """Groups of ``PointGroupNorm``: 32, or ``c // 4`` for narrow layers (vae.py:150)."""
    return 32 if 4 * 32 <= c else c // 4


def group_stats(x: torch.Tensor, eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-channel ``mean`` and ``rsqrt(var + eps)`` of the channel groups (fp32 ``[C]`` each)."""
    _lib.require_cuda(x)
    if x.dtype not in (torch.float16, torch.float32):
        raise ValueError("group_stats takes float16/float32 features")
    x = x.contiguous()
    n, c = x.shape
    mean = torch.empty(c, dtype=torch.float32, device=x.device)
    inv = torch.empty_like(mean)
    lib = _lib.load()
    nb = ctypes.c_int64()
    _lib.check(lib.hi3d_group_norm_stats_workspace_size(n, c, ctypes.byref(nb)), "group_stats", launched=False)
    ws = torch.empty(nb.value, dtype=torch.uint8, device=x.device)
    rc = lib.hi3d_group_norm_stats(x.data_ptr(), n, c, _groups(c), float(eps), mean.data_ptr(), inv.data_ptr(),
                                   ws.data_ptr(), ws.numel(), _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "group_stats")
    return mean, inv


def group_norm_swish(x: torch.Tensor, mean: torch.Tensor, inv: torch.Tensor, weight: torch.Tensor,
                     bias: torch.Tensor, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """``swish((x - mean) * inv * weight + bias)`` in fp32, stored in ``out_dtype``."""
    _lib.require_cuda(x, mean, inv, weight, bias)
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    rc = _lib.load().hi3d_group_norm_swish(x.data_ptr(), x.shape[0], x.shape[1], mean.data_ptr(), inv.data_ptr(),
                                           weight.float().contiguous().data_ptr(),
                                           bias.float().contiguous().data_ptr(), out.data_ptr(),
                                           _lib.dtype_code(x), _lib.dtype_code(out), _lib.stream(x))
    _lib.check(rc, "group_norm_swish")
    return out


def conv_gn_swish(x: torch.Tensor, level: sparse.Level, norm_weight: torch.Tensor, norm_bias: torch.Tensor,
                  conv_weight: torch.Tensor, conv_bias: torch.Tensor | None,
                  dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """``conv(swish(GroupNorm(x)))`` (vae.py:166-192): ``conv_weight`` in spconv layout
    ``[Cout, 3, 3, 3, Cin]``; the GEMMs run in ``dtype`` (fp16/bf16)."""
    mean, inv = group_stats(x)
    act = group_norm_swish(x, mean, inv, norm_weight, norm_bias, out_dtype=torch.float16)
    return sparse.conv(act.to(dtype), level.table, conv_weight.to(dtype), conv_bias, n_in=level.n,
                       tap_mask=level.tap_mask)


def child_neighbour_table(parent_table: torch.Tensor, child_mask: torch.Tensor):
    """``(table [C, 27], parent [C], slot [C])`` of the kept children (parent-major, slot-minor)
    from the parent table ``[P, 27]`` and the occupancy ``child_mask [P, 8]`` (bool/uint8), as
    ``sparse.child_neighbour_table`` (sparse.py:64-95).  Synchronises once (the child count)."""
    _lib.require_cuda(parent_table, child_mask)
    p = parent_table.shape[0]
    mask = child_mask.to(torch.uint8).contiguous()
    if mask.shape != (p, 8):
        raise ValueError("child_mask must be [P, 8]")
    lib = _lib.load()
    nb = ctypes.c_int64()
    _lib.check(lib.hi3d_child_table_workspace_size(p, ctypes.byref(nb)), "child_table", launched=False)
    ws = torch.empty(nb.value, dtype=torch.uint8, device=mask.device)
    parent = torch.empty(8 * p, dtype=torch.int32, device=mask.device)
    slot = torch.empty_like(parent)
    num = torch.zeros(1, dtype=torch.int32, device=mask.device)
    rc = lib.hi3d_child_structure(mask.data_ptr(), p, parent.data_ptr(), slot.data_ptr(), num.data_ptr(),
                                  ws.data_ptr(), ws.numel(), _lib.stream(mask))
    _lib.check(rc, "child_structure")
    c = int(num.item())
    table = torch.empty((c, 27), dtype=torch.int32, device=mask.device)
    rc = lib.hi3d_child_table(parent_table.contiguous().data_ptr(), p, parent.data_ptr(), slot.data_ptr(), c,
                              ws.data_ptr(), table.data_ptr(), _lib.stream(mask))
    _lib.check(rc, "child_table")
    return table, parent[:c], slot[:c]


def serialization(coords) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """``(perm, inverse)`` of the Morton order and of its x/y-swapped variant (vae.py:58-69)."""
    c = sparse._coords_dev(coords)
    n = c.shape[0]
    depth = int(c.max().item()).bit_length() if n else 0
    lib = _lib.load()
    nb = ctypes.c_int64()
    _lib.check(lib.hi3d_serialize_workspace_size(n, ctypes.byref(nb)), "serialization", launched=False)
    ws = torch.empty(nb.value, dtype=torch.uint8, device=c.device)
    out = []
    for order in ORDERS:
        perm = torch.empty(n, dtype=torch.int32, device=c.device)
        inverse = torch.empty_like(perm)
        rc = lib.hi3d_serialize(c.data_ptr(), n, depth, 1 if order == "z-trans" else 0, perm.data_ptr(),
                                inverse.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream(c))
        _lib.check(rc, "serialization")
        out.append((perm, inverse))
    return out


def window_index(perm: torch.Tensor, patch: int = PATCH) -> torch.Tensor:
    """Rows in padded window order (vae.py:72-88): windows of ``patch`` serialized points, the
    last one completed with the points before it."""
    n = perm.shape[0]
    if n <= patch:
        return perm
    n_pad = -(-n // patch) * patch
    pad = torch.arange(n_pad, device=perm.device)
    rem = n % patch
    if rem:
        pad[n_pad - patch + rem:] = pad[n_pad - 2 * patch + rem:n_pad - patch].clone()
    return perm[pad].contiguous()


def window_attention(qkv: torch.Tensor, gather: torch.Tensor, heads: int, patch: int = PATCH,
                     scale: float | None = None) -> torch.Tensor:
    """Attention within each serialized window (vae.py:249-266): ``qkv [N, 3 C]`` (layout
    ``[3, heads, D]`` per row), ``gather`` from :func:`window_index`; returns ``[N, C]`` in
    point order."""
    _lib.require_cuda(qkv, gather)
    n, c3 = qkv.shape
    c = c3 // 3
    d = c // heads
    scale = d ** -0.5 if scale is None else scale
    out = torch.empty((n, c), dtype=qkv.dtype, device=qkv.device)
    rc = _lib.load().hi3d_window_attention(qkv.contiguous().data_ptr(), gather.contiguous().data_ptr(), n,
                                           gather.shape[0], patch, heads, d, float(scale), out.data_ptr(),
                                           _lib.dtype_code(qkv), _lib.stream(qkv))
    _lib.check(rc, "window_attention")
    return out
