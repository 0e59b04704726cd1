"""W8A8 projections: int8 activations and weights on the tcgen05 int8 tensor cores.

Mirrors ``hi3d_mac.mlx_backend.w8a8`` (src/hi3d_mac/mlx_backend/w8a8.py): ``signs`` (:16-18),
``quantize_activation`` (:95-102, kernel :25-58) and ``linear`` (:105-119, GEMM :61-80).
Activations are quantised per row after the signed 64-point Hadamard rotation; weights are
stored int8 per output row in the same rotated domain (the ``hi3d-w8a8-h64`` format), so
``(x S H)(W S H)^T = x W^T``.  The GEMM accumulates exact int32 products and dequantises in its
epilogue, ``half(float(acc) * sa * sw + bias)``.
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np
import torch

from . import _lib
from .linear import _EPI, _gate_args


@lru_cache(None)
def signs(width: int) -> np.ndarray:
    """The per-column sign vector of the rotation (w8a8.py:16-18)."""
    return np.random.default_rng(314159 + width).choice([-1.0, 1.0], width).astype(np.float32)


_SIGN_CACHE: dict = {}


def _signs_on(width: int, device: torch.device) -> torch.Tensor:
    key = (width, str(device))
    if key not in _SIGN_CACHE:
        _SIGN_CACHE[key] = torch.from_numpy(signs(width)).to(device)
    return _SIGN_CACHE[key]


def quantize_activation(x: torch.Tensor, multiplier: torch.Tensor | None = None, rotate: bool = True):
    """Per-row dynamic symmetric int8: returns ``(q [M, K] int8, scale [M] fp32)``.

    With ``rotate`` (the reference behaviour) every 64-block is rotated by the signed
    Walsh-Hadamard transform first; ``multiplier`` replaces the default sign vector.
    ``rotate=False`` is plain per-token quantisation."""
    _lib.require_cuda(x, multiplier)
    k = x.shape[-1]
    if k % 64:
        raise ValueError("signed H64 requires width divisible by 64")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("quantize_activation takes float16/bfloat16 input")
    a = x.reshape(-1, k).contiguous()
    m = a.shape[0]
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty(m, dtype=torch.float32, device=x.device)
    mult = None
    if rotate:
        mult = _signs_on(k, x.device) if multiplier is None else multiplier.float().contiguous()
    rc = _lib.load().hi3d_quantize_act_i8(a.data_ptr(), _lib.ptr(mult), q.data_ptr(), s.data_ptr(), m, k, int(rotate),
                                          _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "quantize_activation")
    return q, s


def quantize_weight(w: torch.Tensor, rotate: bool = True):
    """Symmetric per-output-row int8 weights in the activations' rotated domain
    (``hi3d-w8a8-h64``, models/w8a8/manifest.json:11-16): ``(int8 [N, K], scale [N] fp32)``."""
    return quantize_activation(w.to(torch.float16) if w.dtype not in (torch.float16, torch.bfloat16) else w,
                               rotate=rotate)


def gemm_accumulators(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Exact int32 ``a @ w^T`` for int8 ``a [M, K]``, ``w [N, K]`` (raw tensor-core accumulators)."""
    _lib.require_cuda(a, w)
    if a.dtype != torch.int8 or w.dtype != torch.int8 or a.shape[1] != w.shape[1]:
        raise ValueError("gemm_accumulators takes int8 [M, K] and [N, K]")
    a, w = a.contiguous(), w.contiguous()
    m, k = a.shape
    n = w.shape[0]
    ldo = (n + 3) // 4 * 4
    out = torch.empty((m, ldo), dtype=torch.int32, device=a.device)
    rc = _lib.load().hi3d_gemm_w8a8(a.data_ptr(), w.data_ptr(), None, None, None, out.data_ptr(), m, n, k, ldo,
                                    _lib.EPI_STORE, None, 0, 0, _lib.I32, _lib.stream(a))
    _lib.check(rc, "gemm_accumulators")
    return out[:, :n]


class Quantized:
    """Activations already quantised per row (``q [R, K]`` int8, ``scale [R]`` fp32) standing in
    for the 16-bit ``x [..., K]`` they came from (``shape``, ``dtype``): :func:`linear` and
    :func:`linear_qkv_rope` take them in place of ``x`` and skip their own quantisation.
    ``[b]`` selects batch element ``b`` of a ``[B, N, K]`` input."""

    def __init__(self, q: torch.Tensor, scale: torch.Tensor, shape: tuple, dtype: torch.dtype):
        self.q, self.scale, self.shape, self.dtype = q, scale, tuple(shape), dtype
        self.device = q.device

    def view(self, *shape) -> "Quantized":
        return Quantized(self.q, self.scale, (self.q.shape[0], self.shape[-1]), self.dtype)

    def __getitem__(self, b: int) -> "Quantized":
        if len(self.shape) != 3:
            raise ValueError("batch indexing needs a [B, N, K] input")
        n = self.shape[1]
        return Quantized(self.q[b * n:(b + 1) * n], self.scale[b * n:(b + 1) * n], self.shape[1:], self.dtype)


def layer_norm_quantize(x: torch.Tensor, eps: float, weight: torch.Tensor | None = None,
                        bias: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                        shift: torch.Tensor | None = None) -> Quantized:
    """``quantize_activation(layer_norm_modulate(x, ...))`` in one pass (the 16-bit normalised
    rows are never written); arguments as :func:`hi3d_b200.kernels.layer_norm_modulate`."""
    _lib.require_cuda(x, weight, bias, scale, shift)
    c = x.shape[-1]
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("layer_norm_quantize takes float16/bfloat16 rows")
    if (weight is None) != (bias is None) or (scale is None) != (shift is None):
        raise ValueError("weight/bias and scale/shift come in pairs")
    xc = x.contiguous()
    rows = xc.numel() // c
    rows_per_batch, mod_stride = rows, 0
    if scale is not None:
        scale = scale.to(x.dtype).reshape(-1, c).contiguous()
        shift = shift.to(x.dtype).reshape(-1, c).contiguous()
        nb = scale.shape[0]
        if nb > 1:
            if x.dim() < 3 or x.shape[0] != nb:
                raise ValueError(f"per-batch modulation [{nb}, C] needs x [{nb}, N, C]")
            rows_per_batch, mod_stride = rows // nb, c
    if weight is not None:
        weight = weight.float().contiguous()
        bias = bias.float().contiguous()
    q = torch.empty((rows, c), dtype=torch.int8, device=x.device)
    s = torch.empty(rows, dtype=torch.float32, device=x.device)
    rc = _lib.load().hi3d_layer_norm_quantize(xc.data_ptr(), q.data_ptr(), s.data_ptr(), rows, c, float(eps),
                                              _lib.ptr(weight), _lib.ptr(bias), _lib.ptr(scale), _lib.ptr(shift),
                                              rows_per_batch, mod_stride, _signs_on(c, x.device).data_ptr(),
                                              _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "layer_norm_quantize")
    return Quantized(q, s, x.shape, x.dtype)


def _quantized(x, multiplier, rotate):
    """``(q, scale, out_dtype)`` of ``x`` (or of an already quantised :class:`Quantized`)."""
    if isinstance(x, Quantized):
        return x.q, x.scale, x.dtype
    out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
    q, s = quantize_activation(x.to(out_dtype), multiplier, rotate)
    return q, s, out_dtype


def linear(x: torch.Tensor, w: torch.Tensor, sw: torch.Tensor, bias: torch.Tensor, tile=(64, 128),
           multiplier: torch.Tensor | None = None, epilogue: str = "store", residual: torch.Tensor | None = None,
           gate: torch.Tensor | None = None, rotate: bool = True) -> torch.Tensor:
    """``x @ W^T + bias`` through int8: quantise ``x`` per row, int8 GEMM with exact int32
    accumulation, dequantise ``half(float(acc) * sa * sw + bias)`` (w8a8.py:105-119).
    ``tile`` is accepted for signature compatibility (the B200 kernel uses 128 x 256 tiles).
    ``epilogue``/``residual``/``gate`` as in :func:`hi3d_b200.linear.linear`."""
    _lib.require_cuda(x if isinstance(x, torch.Tensor) else x.q, w, sw, bias, residual, gate)
    if w.dtype != torch.int8 or sw.dtype != torch.float32:
        raise ValueError("W8A8 requires int8 weights and float32 scales")
    if w.dim() != 2 or x.shape[-1] != w.shape[1] or sw.shape != (w.shape[0],) or bias.shape != (w.shape[0],):
        raise ValueError("incompatible W8A8 projection shapes")
    a, sa, out_dtype = _quantized(x, multiplier, rotate)
    m, k = a.shape
    n = w.shape[0]
    epi = _EPI[epilogue]
    if epilogue == "residual":
        if residual is None or residual.numel() != m * n or not residual.is_contiguous():
            raise ValueError("residual epilogue needs a contiguous residual [..., N] with the rows of x")
        out = residual
    else:
        out = torch.empty((*x.shape[:-1], n), dtype=out_dtype, device=x.device)
    g, rpb, gs = _gate_args(gate, m, n, out_dtype)
    b = bias.to(out_dtype).contiguous()
    rc = _lib.load().hi3d_gemm_w8a8(a.data_ptr(), w.contiguous().data_ptr(), sa.data_ptr(), sw.contiguous().data_ptr(),
                                    b.data_ptr(), out.data_ptr(), m, n, k, n, epi, _lib.ptr(g), rpb, gs,
                                    _lib.dtype_code(out), _lib.stream(x))
    _lib.check(rc, "w8a8.linear")
    return out


def linear_qkv_rope(x: torch.Tensor, w: torch.Tensor, sw: torch.Tensor, bias: torch.Tensor, cos: torch.Tensor,
                    sin: torch.Tensor, gamma_q: torch.Tensor, gamma_k: torch.Tensor, batch: int, heads: int,
                    head_dim: int, token_major: bool = False, multiplier: torch.Tensor | None = None,
                    rotate: bool = True, out: tuple | None = None, peer_offsets: tuple[int, ...] = (),
                    multicast_offset: int = 0):
    """The attention input projection through int8 (as :func:`linear`, w8a8.py:105-119) with
    RoPE + QK RMS norm + head split in the GEMM epilogue (as ``hi3d_b200.linear.linear_qkv_rope``)."""
    from .linear import _qkv_rope_args, peer_offset_array

    _lib.require_cuda(x if isinstance(x, torch.Tensor) else x.q, w, sw, bias, cos, sin, gamma_q, gamma_k)
    if w.dtype != torch.int8 or sw.dtype != torch.float32:
        raise ValueError("W8A8 requires int8 weights and float32 scales")
    if w.shape != (3 * heads * head_dim, x.shape[-1]) or sw.shape != (w.shape[0],) or bias.shape != (w.shape[0],):
        raise ValueError("incompatible W8A8 projection shapes")
    aq, sa, out_dtype = _quantized(x, multiplier, rotate)
    _, m, n, cos, sin, gq, gk, q, k, v = _qkv_rope_args(aq, cos, sin, gamma_q, gamma_k, batch, heads, head_dim,
                                                        token_major, out_dtype, out)
    b = bias.to(out_dtype).contiguous()
    rc = _lib.load().hi3d_gemm_w8a8_qkv_rope_peers(aq.data_ptr(), w.contiguous().data_ptr(), sa.data_ptr(),
                                                   sw.contiguous().data_ptr(), b.data_ptr(), cos.data_ptr(),
                                                   sin.data_ptr(), gq.data_ptr(), gk.data_ptr(), q.data_ptr(),
                                                   k.data_ptr(), v.data_ptr(), m, n, heads, head_dim, aq.shape[1],
                                                   int(token_major), _lib.dtype_code(q),
                                                   peer_offset_array(peer_offsets), len(peer_offsets),
                                                   int(multicast_offset), _lib.stream(x))
    _lib.check(rc, "w8a8.linear_qkv_rope")
    return q, k, v
