"""``spconv.pytorch`` subset backed by the B200 sparse kernels.

The API subset the upstream ``sparc3d.ops.sparse_backend`` imports (src/sparc3d/ops/sparse_backend.py:20-148)
and the reference's CPU shim provides (src/hi3d_mac/torch_backend/sparse_conv.py): ``SubMConv3d``,
``SparseConvTensor``, ``ConvAlgo``, ``ops.get_indice_pairs`` and ``core.IndiceData``.  Convolution
semantics are spconv's (the shim's docstring, :4-13): an input voxel at ``p`` feeds the output at
``p + center - r`` for kernel offset ``r``, i.e. ``out[o] = bias + sum_r W[:, r, :] @ in[o + r - center]``.

Indices are ``[N, 4]`` int32 ``(batch, x, y, z)``; batches are separated by offsetting ``x`` so no
voxel neighbours another batch's.  The neighbour table is built on the GPU and cached per
``indice_key`` like spconv's indice dict.  Features run in the weight dtype (fp16/bf16 on the
tensor cores); fp32 weights raise ``NotImplementedError``.
"""

from __future__ import annotations

import enum
import itertools
import math
from typing import Any, Sequence

import torch
from torch import nn

from .. import sparse as _sparse


class ConvAlgo(enum.Enum):
    """spconv algorithm selector; every value runs the same gather-GEMM kernel."""

    Native = 0
    MaskImplicitGemm = 1
    MaskSplitImplicitGemm = 2


class IndiceData:
    """Cached submanifold neighbourhood, mirroring ``spconv.pytorch.core.IndiceData``."""

    def __init__(self, out_indices: torch.Tensor, indices: torch.Tensor, indice_pairs: Any,
                 indice_pair_num: torch.Tensor, spatial_shape: Sequence[int], out_spatial_shape: Sequence[int],
                 is_subm: bool = True, algo: ConvAlgo = ConvAlgo.Native, table: torch.Tensor | None = None,
                 tap_mask: torch.Tensor | None = None, **_: Any):
        self.out_indices = out_indices
        self.indices = indices
        self.indice_pairs = indice_pairs
        self.indice_pair_num = indice_pair_num
        self.spatial_shape = list(spatial_shape)
        self.out_spatial_shape = list(out_spatial_shape)
        self.is_subm = is_subm
        self.algo = algo
        self.table = table
        self.tap_mask = tap_mask


class SparseConvTensor:
    """Features, ``[N, 4]`` int32 ``(batch, x, y, z)`` indices and a shared pair cache."""

    def __init__(self, features: torch.Tensor, indices: torch.Tensor, spatial_shape: Sequence[int],
                 batch_size: int, indice_dict: dict | None = None):
        self._features = features
        self.indices = indices
        self.spatial_shape = [int(v) for v in spatial_shape]
        self.batch_size = int(batch_size)
        self.indice_dict = {} if indice_dict is None else indice_dict

    @property
    def features(self) -> torch.Tensor:
        return self._features

    def replace_feature(self, feature: torch.Tensor) -> "SparseConvTensor":
        return SparseConvTensor(feature, self.indices, self.spatial_shape, self.batch_size, self.indice_dict)

    def find_indice_pair(self, key: str | None) -> IndiceData | None:
        return None if key is None else self.indice_dict.get(key)


def _folded_coords(indices: torch.Tensor, spatial_shape: Sequence[int]) -> torch.Tensor:
    """``(x + batch * (sx + 2), y, z)``: batches never neighbour each other."""
    idx = indices.to(torch.int32)
    stride = int(spatial_shape[0]) + 2
    return torch.stack([idx[:, 1] + idx[:, 0] * stride, idx[:, 2], idx[:, 3]], 1).contiguous()


class _PairTable:
    """``[2, 27, N]``-indexable view over per-offset pair lists (spconv Native layout, unpadded)."""

    def __init__(self, table: torch.Tensor):
        self._table = table
        self._cache: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def _pairs(self, k: int):
        if k not in self._cache:
            col = self._table[:, k].long()
            n = self._table.shape[0]
            dst = torch.nonzero(col < n, as_tuple=False).flatten()
            self._cache[k] = (col[dst], dst)
        return self._cache[k]

    def __getitem__(self, index):
        side, offset, rows = index
        return self._pairs(int(offset))[side][rows]


def _indice_data(indices: torch.Tensor, spatial_shape: Sequence[int], kernel_size: int) -> IndiceData:
    if kernel_size != 3:
        raise NotImplementedError("only 3x3x3 submanifold convolutions are implemented")
    coords = _folded_coords(indices, spatial_shape)
    table = _sparse.neighbour_table(coords)
    n = table.shape[0]
    counts = (table < n).sum(0).to(torch.int32).cpu()
    return IndiceData(indices, indices, _PairTable(table), counts, spatial_shape, spatial_shape, True,
                      ConvAlgo.Native, table=table, tap_mask=_sparse.conv_tap_mask(table, n))


class SubMConv3d(nn.Module):
    """Submanifold 3D convolution with spconv's parameter names and ``(out, k, k, k, in)`` layout."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int | Sequence[int] = 3,
                 stride: int | Sequence[int] = 1, padding: int | Sequence[int] = 0,
                 dilation: int | Sequence[int] = 1, groups: int = 1, bias: bool = True,
                 indice_key: str | None = None, algo: ConvAlgo | None = None, **_: Any):
        super().__init__()
        ks = (kernel_size,) * 3 if isinstance(kernel_size, int) else tuple(kernel_size)
        if len(set(ks)) != 1 or ks[0] % 2 == 0:
            raise ValueError(f"only cubic odd kernels are supported, got {ks}")
        if groups != 1:
            raise ValueError("grouped sparse convolution is not supported")
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = ks
        self.stride = (1, 1, 1)
        self.padding = tuple(k // 2 for k in ks)
        self.dilation = (1, 1, 1)
        self.output_padding = (0, 0, 0)
        self.indice_key = indice_key
        self.algo = algo or ConvAlgo.MaskImplicitGemm
        self.weight = nn.Parameter(torch.empty(out_channels, *ks, in_channels))
        self.bias = nn.Parameter(torch.empty(out_channels)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def _pairs(self, input: SparseConvTensor) -> IndiceData:
        data = input.find_indice_pair(self.indice_key)
        if data is None or data.table is None:
            data = _indice_data(input.indices, input.spatial_shape, self.kernel_size[0])
            if self.indice_key is not None:
                input.indice_dict[self.indice_key] = data
        return data

    def forward(self, input: SparseConvTensor) -> SparseConvTensor:
        if self.weight.dtype not in (torch.float16, torch.bfloat16):
            raise NotImplementedError("the B200 sparse convolution runs in float16 or bfloat16")
        data = self._pairs(input)
        x = input.features.to(self.weight.dtype)
        out = _sparse.conv(x, data.table, self.weight, self.bias, n_in=x.shape[0], tap_mask=data.tap_mask)
        return input.replace_feature(out)


def get_indice_pairs(indices: torch.Tensor, batch_size: int, spatial_shape: Sequence[int], algo: ConvAlgo,
                     ksize: Sequence[int], stride: Sequence[int], padding: Sequence[int], dilation: Sequence[int],
                     out_padding: Sequence[int], subm: bool = False, transpose: bool = False):
    """``spconv.pytorch.ops.get_indice_pairs`` for the submanifold case (as the reference's shim,
    src/hi3d_mac/torch_backend/sparse_conv.py:264-283)."""
    if not subm or transpose:
        raise NotImplementedError("only submanifold index pairs are implemented")
    if tuple(stride) != (1, 1, 1) or tuple(dilation) != (1, 1, 1):
        raise NotImplementedError("only stride 1 / dilation 1 are implemented")
    data = _indice_data(indices, spatial_shape, int(ksize[0]))
    return indices, data.indice_pairs, data.indice_pair_num


KERNEL_OFFSETS = list(itertools.product(range(3), repeat=3))
