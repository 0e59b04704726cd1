"""Sparse voxel structure and convolution on B200.

Mirrors ``hi3d_mac.mlx_backend.sparse`` (src/hi3d_mac/mlx_backend/sparse.py): ``OFFSETS`` (:20),
``neighbour_table`` (:29-43), ``Level`` (:98-115), ``conv_weight`` (:185-188), ``sparse_conv``
(:191-214) and ``downsample_structure`` (:217-233), with the index structures built on the GPU
(hash table + 27 probes per voxel; radix sort for the downsample) instead of numpy, and the
convolution as one tcgen05 gather-GEMM kernel.

Convolution convention (the reference's, verified there against spconv):
``out[o] = b + sum_k W[:, k, :] @ in[o + r_k - 1]`` with ``r_k`` the row-major ``(x, y, z)``
kernel position of flat offset ``k``.
"""

from __future__ import annotations

import ctypes
import itertools

import numpy as np
import torch

from . import _lib

OFFSETS = np.array(list(itertools.product(range(3), repeat=3)), dtype=np.int64) - 1
"""``[27, 3]`` neighbour displacement ``r_k - 1`` for each flat kernel offset."""

CENTER = 13


def _coords_dev(coords, device=None) -> torch.Tensor:
    if isinstance(coords, torch.Tensor):
        t = coords.to(torch.int32)
        if not t.is_cuda:
            t = t.to(device or "cuda")
    else:
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(coords, dtype=np.int32))).to(device or "cuda")
    t = t.reshape(-1, 3).contiguous()
    return t


def _workspace(fn, n: int, device) -> torch.Tensor:
    nbytes = ctypes.c_int64()
    _lib.check(fn(n, ctypes.byref(nbytes)), "workspace size", launched=False)
    return torch.empty(nbytes.value, dtype=torch.uint8, device=device)


def neighbour_table(coords, query=None, stride: int = 1) -> torch.Tensor:
    """``[N, 27]`` int32 neighbour rows (``N`` where absent), on the GPU.

    ``query``/``stride`` give the strided form: row of ``query[o] * stride + d_k``."""
    c = _coords_dev(coords)
    n = c.shape[0]
    q = None if query is None else _coords_dev(query, c.device)
    nq = n if q is None else q.shape[0]
    table = torch.empty((nq, 27), dtype=torch.int32, device=c.device)
    lib = _lib.load()
    ws = _workspace(lib.hi3d_neighbour_map_workspace_size, n, c.device)
    rc = lib.hi3d_neighbour_map_build(c.data_ptr(), n, _lib.ptr(q), nq, stride, table.data_ptr(), ws.data_ptr(),
                                      ws.numel(), _lib.stream(c))
    _lib.check(rc, "neighbour_table")
    return table


def downsample_structure(coords):
    """``(low, inverse, counts)``: unique ``coords // 2`` in lexicographic ``(x, y, z)`` order,
    each row's parent, and children per parent (int32 device tensors).  Synchronises once."""
    c = _coords_dev(coords)
    n = c.shape[0]
    low = torch.empty((max(n, 1), 3), dtype=torch.int32, device=c.device)
    inverse = torch.empty(n, dtype=torch.int32, device=c.device)
    counts = torch.empty(max(n, 1), dtype=torch.int32, device=c.device)
    num = torch.zeros(1, dtype=torch.int32, device=c.device)
    lib = _lib.load()
    ws = _workspace(lib.hi3d_downsample_workspace_size, n, c.device)
    rc = lib.hi3d_downsample_structure(c.data_ptr(), n, low.data_ptr(), inverse.data_ptr(), counts.data_ptr(),
                                       num.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream(c))
    _lib.check(rc, "downsample_structure")
    m = int(num.item())
    return low[:m], inverse, counts[:m]


def downsample_groups(coords):
    """``(low, inverse, counts, children, offsets)``: :func:`downsample_structure` plus the fine
    rows of each low voxel, ``children[offsets[g]:offsets[g + 1]]`` in ascending row order (the
    rows Geometry.downsample averages, transformer.py:261-263).  Synchronises once."""
    c = _coords_dev(coords)
    n = c.shape[0]
    low = torch.empty((max(n, 1), 3), dtype=torch.int32, device=c.device)
    inverse = torch.empty(n, dtype=torch.int32, device=c.device)
    counts = torch.empty(max(n, 1), dtype=torch.int32, device=c.device)
    children = torch.empty(max(n, 1), dtype=torch.int32, device=c.device)
    offsets = torch.empty(n + 1, dtype=torch.int32, device=c.device)
    num = torch.zeros(1, dtype=torch.int32, device=c.device)
    lib = _lib.load()
    ws = _workspace(lib.hi3d_downsample_workspace_size, n, c.device)
    rc = lib.hi3d_downsample_structure_children(c.data_ptr(), n, low.data_ptr(), inverse.data_ptr(),
                                                counts.data_ptr(), children.data_ptr(), offsets.data_ptr(),
                                                num.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream(c))
    _lib.check(rc, "downsample_structure_children")
    m = int(num.item())
    return low[:m], inverse, counts[:m], children[:n], offsets[:m + 1]


def downsample_mean(x: torch.Tensor, children: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """Mean of each low voxel's children with the reference's ``children + 1`` divisor
    (Geometry.downsample, transformer.py:261-263), fp32 sums in ascending row order."""
    _lib.require_cuda(x, children, offsets)
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("downsample_mean takes float16/bfloat16 features")
    x = x.contiguous()
    m = offsets.shape[0] - 1
    out = torch.empty((m, x.shape[1]), dtype=x.dtype, device=x.device)
    rc = _lib.load().hi3d_downsample_mean(x.data_ptr(), children.data_ptr(), offsets.data_ptr(), m, x.shape[1],
                                          out.data_ptr(), _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "downsample_mean")
    return out


def upsample(x: torch.Tensor, inverse: torch.Tensor) -> torch.Tensor:
    """Rows of the low level copied to their fine children (Geometry.upsample,
    transformer.py:265-266)."""
    _lib.require_cuda(x, inverse)
    x = x.contiguous()
    out = torch.empty((inverse.shape[0], x.shape[1]), dtype=x.dtype, device=x.device)
    rc = _lib.load().hi3d_gather_rows(x.data_ptr(), inverse.data_ptr(), inverse.shape[0], x.shape[1], out.data_ptr(),
                                      _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "upsample")
    return out


def up_conv(h_low: torch.Tensor, fine_table: torch.Tensor, inverse: torch.Tensor, weight: torch.Tensor,
            bias: torch.Tensor | None = None) -> torch.Tensor:
    """3x3x3 convolution at the fine level of the upsampled ``h_low`` without materialising the
    upsampled rows (Sparc3DTransformerMLX._up_conv, transformer.py:449-475): every low voxel is
    projected through the 27 taps by one GEMM, ``proj [N_low * 27, Cout]``, then each fine voxel
    sums the projections of its neighbours' parents.  ``weight`` in spconv layout
    ``[Cout, 3, 3, 3, Cin]``."""
    from . import linear as _linear

    _lib.require_cuda(h_low, fine_table, inverse, weight, bias)
    cout = weight.shape[0]
    # [Cout, 27, Cin] -> [27 * Cout, Cin]: GEMM row k * Cout + o is tap k of output channel o
    w_taps = weight.reshape(cout, 27, -1).to(h_low.dtype).permute(1, 0, 2).reshape(27 * cout, -1).contiguous()
    proj = _linear.linear(h_low.contiguous(), w_taps)
    n_fine = fine_table.shape[0]
    out = torch.empty((n_fine, cout), dtype=h_low.dtype, device=h_low.device)
    b = None if bias is None else bias.to(h_low.dtype).contiguous()
    rc = _lib.load().hi3d_upconv_gather_sum(proj.data_ptr(), fine_table.data_ptr(), inverse.data_ptr(), n_fine, cout,
                                            _lib.ptr(b), out.data_ptr(), _lib.dtype_code(h_low),
                                            _lib.stream(h_low))
    _lib.check(rc, "up_conv")
    return out


class Level:
    """One coordinate set and its convolution gather table (``N`` marks absent)."""

    def __init__(self, coords, table: torch.Tensor):
        self.coords = coords
        self.n = int(coords.shape[0])
        self.table = table
        self._mask = None

    @property
    def table_np(self) -> np.ndarray:
        return self.table.cpu().numpy()

    @property
    def tap_mask(self) -> torch.Tensor:
        """Taps present per 128-row tile (built once per level)."""
        if self._mask is None:
            self._mask = conv_tap_mask(self.table, self.n)
        return self._mask

    @classmethod
    def from_coords(cls, coords) -> "Level":
        return cls(coords, neighbour_table(coords))


def conv_tap_mask(table: torch.Tensor, n_in: int) -> torch.Tensor:
    n_out = table.shape[0]
    mask = torch.empty(max(1, (n_out + 127) // 128), dtype=torch.int32, device=table.device)
    rc = _lib.load().hi3d_conv_tap_mask(table.data_ptr(), n_out, n_in, mask.data_ptr(), _lib.stream(table))
    _lib.check(rc, "conv_tap_mask")
    return mask


def conv_weight(weight: torch.Tensor) -> torch.Tensor:
    """spconv ``(out, 3, 3, 3, in)`` -> GEMM layout ``[27 * in, out]`` (sparse.py:185-188)."""
    return weight.reshape(weight.shape[0], -1).t()


def _kernel_weight_from_gemm(weight_t: torch.Tensor) -> torch.Tensor:
    """``[27 * in, out]`` -> the kernel's ``[out, 27, in]`` (spconv order)."""
    k27cin, cout = weight_t.shape
    return weight_t.reshape(27, k27cin // 27, cout).permute(2, 0, 1).contiguous()


def conv(x: torch.Tensor, table: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
         n_in: int | None = None, tap_mask: torch.Tensor | None = None, act: str | None = None) -> torch.Tensor:
    """Gathered 3x3x3 convolution with the spconv weight layout ``weight [out, 3, 3, 3, in]``
    (or ``[out, 27, in]``): ``out[o] = bias + sum_k x[table[o, k]] W_k^T``; ``act="silu"``
    applies SiLU to the rounded output (the conv2 -> SiLU of a res block)."""
    if act not in (None, "silu"):
        raise ValueError(f"unknown activation {act!r}")
    _lib.require_cuda(x, table, weight, bias)
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("sparse conv takes float16/bfloat16 features")
    n_in = x.shape[0] if n_in is None else n_in
    cout = weight.shape[0]
    w = weight.reshape(cout, 27, -1).to(x.dtype).contiguous()
    cin = w.shape[2]
    if x.shape[1] != cin or table.shape[1] != 27:
        raise ValueError(f"incompatible shapes x {tuple(x.shape)} weight {tuple(weight.shape)} table {tuple(table.shape)}")
    x = x.contiguous()
    n_out = table.shape[0]
    if tap_mask is None:
        tap_mask = conv_tap_mask(table, n_in)
    out = torch.empty((n_out, cout), dtype=x.dtype, device=x.device)
    b = None if bias is None else bias.to(x.dtype).contiguous()
    rc = _lib.load().hi3d_sparse_conv_act(x.data_ptr(), table.data_ptr(), tap_mask.data_ptr(), w.data_ptr(),
                                          _lib.ptr(b), out.data_ptr(), n_in, n_out, cin, cout,
                                          1 if act == "silu" else 0, _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "sparse_conv")
    return out


def sparse_conv(x: torch.Tensor, level: Level, weight_t: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """Submanifold 3x3x3 convolution (sparse.py:191-214): ``weight_t [27 * Cin, Cout]`` from
    :func:`conv_weight`; runs in ``weight_t.dtype``."""
    x = x.to(weight_t.dtype)
    return conv(x, level.table, _kernel_weight_from_gemm(weight_t), bias, n_in=level.n, tap_mask=level.tap_mask)


def downsample_conv(x: torch.Tensor, coords, weight: torch.Tensor, bias: torch.Tensor | None = None):
    """Stride-2 3x3x3 sparse convolution (pad 1) onto ``downsample_structure(coords).low``: tap ``k``
    of output ``o`` reads the input at ``2 o + r_k - 1``.  Returns ``(out, low_coords)``."""
    low, _, _ = downsample_structure(coords)
    table = neighbour_table(coords, query=low, stride=2)
    return conv(x, table, weight, bias, n_in=x.shape[0]), low
