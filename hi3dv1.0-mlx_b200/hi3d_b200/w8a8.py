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


def linear(x: torch.Tensor, w: torch.Tensor, sw: torch.Tensor, bias: torch.Tensor, tile=(64, 128),
           multiplier: torch.Tensor | None = None, epilogue: str = "store", residual: torch.Tensor | None = None,
           gate: torch.Tensor | None = None, rotate: bool = True) -> torch.Tensor:
    """``x @ W^T + bias`` through int8: quantise ``x`` per row, int8 GEMM with exact int32
    accumulation, dequantise ``half(float(acc) * sa * sw + bias)`` (w8a8.py:105-119).
    ``tile`` is accepted for signature compatibility (the B200 kernel uses 128 x 256 tiles).
    ``epilogue``/``residual``/``gate`` as in :func:`hi3d_b200.linear.linear`."""
    _lib.require_cuda(x, w, sw, bias, residual, gate)
    if w.dtype != torch.int8 or sw.dtype != torch.float32:
        raise ValueError("W8A8 requires int8 weights and float32 scales")
    if w.dim() != 2 or x.shape[-1] != w.shape[1] or sw.shape != (w.shape[0],) or bias.shape != (w.shape[0],):
        raise ValueError("incompatible W8A8 projection shapes")
    out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
    a, sa = quantize_activation(x.to(out_dtype), multiplier, rotate)
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
                    rotate: bool = True):
    """The attention input projection through int8 (as :func:`linear`, w8a8.py:105-119) with
    RoPE + QK RMS norm + head split in the GEMM epilogue (as ``hi3d_b200.linear.linear_qkv_rope``)."""
    from .linear import _qkv_rope_args

    _lib.require_cuda(x, w, sw, bias, cos, sin, gamma_q, gamma_k)
    if w.dtype != torch.int8 or sw.dtype != torch.float32:
        raise ValueError("W8A8 requires int8 weights and float32 scales")
    if w.shape != (3 * heads * head_dim, x.shape[-1]) or sw.shape != (w.shape[0],) or bias.shape != (w.shape[0],):
        raise ValueError("incompatible W8A8 projection shapes")
    out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
    aq, sa = quantize_activation(x.to(out_dtype), multiplier, rotate)
    _, m, n, cos, sin, gq, gk, q, k, v = _qkv_rope_args(x, cos, sin, gamma_q, gamma_k, batch, heads, head_dim,
                                                        token_major, out_dtype)
    b = bias.to(out_dtype).contiguous()
    rc = _lib.load().hi3d_gemm_w8a8_qkv_rope(aq.data_ptr(), w.contiguous().data_ptr(), sa.data_ptr(),
                                             sw.contiguous().data_ptr(), b.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                             gq.data_ptr(), gk.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), m,
                                             n, heads, head_dim, aq.shape[1], int(token_major),
                                             _lib.dtype_code(q), _lib.stream(x))
    _lib.check(rc, "w8a8.linear_qkv_rope")
    return q, k, v
