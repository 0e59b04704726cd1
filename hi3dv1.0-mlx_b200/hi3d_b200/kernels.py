"""Fused row kernels: LayerNorm + adaLN modulation, RoPE + QK RMS norm + head split.

Same names, arguments and output layouts as ``hi3d_mac.mlx_backend.kernels``
(src/hi3d_mac/mlx_backend/kernels.py:62-90, :137-157, :206-237) with torch CUDA
tensors in place of MLX arrays.  Each call enqueues one sm_100a kernel on the
current stream and returns new tensors (inputs are never mutated).
"""

from __future__ import annotations

import torch

from . import _lib


def layer_norm_modulate(x: torch.Tensor, eps: float, weight: torch.Tensor | None = None,
                        bias: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                        shift: torch.Tensor | None = None, act: str | None = None) -> torch.Tensor:
    """``LayerNorm32`` of fp16/bf16 rows (fp32 statistics), then optionally the adaLN
    modulation ``h * scale + shift`` with two roundings, in one pass over ``x``.

    ``weight``/``bias`` are fp32 ``[C]`` (affine, as ``norm2``); ``scale``/``shift`` are
    ``[C]``, ``[1, C]`` or ``[B, C]`` in the dtype of ``x`` (``[B, C]`` modulates batch
    element ``b`` of ``x [B, N, C]`` with row ``b``).  Reference: kernels.py:162-237.
    ``act="silu"`` appends the SiLU of the transformer's res-block norms
    (src/hi3d_mac/mlx_backend/transformer.py:418-437); it follows either the affine or the
    modulation.
    """
    _lib.require_cuda(x, weight, bias, scale, shift)
    c = x.shape[-1]
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("layer_norm_modulate takes float16/bfloat16 rows")
    if (weight is None) != (bias is None) or (scale is None) != (shift is None):
        raise ValueError("weight/bias and scale/shift come in pairs")
    x = x.contiguous()
    rows = x.numel() // c
    out = torch.empty_like(x)
    rows_per_batch, mod_stride = rows, 0
    if scale is not None:
        scale = scale.to(x.dtype).reshape(-1, c).contiguous()
        shift = shift.to(x.dtype).reshape(-1, c).contiguous()
        if scale.shape != shift.shape:
            raise ValueError("scale and shift shapes differ")
        nb = scale.shape[0]
        if nb > 1:
            if x.dim() < 3 or x.shape[0] != nb:
                raise ValueError(f"per-batch modulation [{nb}, C] needs x [{nb}, N, C]")
            rows_per_batch, mod_stride = rows // nb, c
    if weight is not None:
        weight = weight.float().contiguous()
        bias = bias.float().contiguous()
    lib = _lib.load()
    if act is None:
        rc = lib.hi3d_layer_norm_modulate(x.data_ptr(), out.data_ptr(), rows, c, float(eps), _lib.ptr(weight),
                                          _lib.ptr(bias), _lib.ptr(scale), _lib.ptr(shift), rows_per_batch,
                                          mod_stride, _lib.dtype_code(x), _lib.stream(x))
    elif act == "silu":
        rc = lib.hi3d_layer_norm_act(x.data_ptr(), out.data_ptr(), rows, c, float(eps), _lib.ptr(weight),
                                     _lib.ptr(bias), _lib.ptr(scale), _lib.ptr(shift), rows_per_batch, mod_stride, 1,
                                     _lib.dtype_code(x), _lib.stream(x))
    else:
        raise ValueError(f"unknown activation {act!r}")
    _lib.check(rc, "layer_norm_modulate")
    return out


def qkv_rope_rms(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, gamma_q: torch.Tensor,
                 gamma_k: torch.Tensor, batch: int, heads: int, head_dim: int, token_major: bool = False,
                 out: tuple | None = None):
    """Split a fused ``[B * N, 3 * H * D]`` projection into ``q, k, v [B, H, N, D]``.

    RoPE on adjacent channel pairs (``cos``/``sin`` ``[N, D/2]`` fp32), then
    ``x / max(|x|, 1e-12) * gamma * sqrt(D)`` on queries and keys in fp32; values are
    copied bit-exactly.  Reference: kernels.py:22-90.  ``token_major=True`` returns
    ``[B, N, H, D]`` instead (rows contiguous per token, for a cross-rank gather).  ``out``:
    optional ``(q, k, v)`` tensors to write (None entries are allocated).
    """
    _lib.require_cuda(qkv, cos, sin, gamma_q, gamma_k)
    rows = qkv.shape[0]
    if qkv.dim() != 2 or qkv.shape[1] != 3 * heads * head_dim or rows % batch:
        raise ValueError(f"qkv must be [B*N, 3*H*D], got {tuple(qkv.shape)}")
    if head_dim % 2:
        raise ValueError("an even head dimension is required")
    n = rows // batch
    qkv = qkv.contiguous()
    cos = cos.float().contiguous()
    sin = sin.float().contiguous()
    if cos.shape != (n, head_dim // 2) or sin.shape != (n, head_dim // 2):
        raise ValueError(f"cos/sin must be [N, D/2] = [{n}, {head_dim // 2}]")
    gq = gamma_q.float().reshape(heads, head_dim).contiguous()
    gk = gamma_k.float().reshape(heads, head_dim).contiguous()
    shape = (batch, n, heads, head_dim) if token_major else (batch, heads, n, head_dim)
    from .linear import qkv_outputs

    q, k, v = qkv_outputs(shape, qkv.dtype, qkv.device, out)
    rc = _lib.load().hi3d_qkv_rope_rms(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), gq.data_ptr(), gk.data_ptr(),
                                       q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, n, heads, head_dim,
                                       int(token_major), _lib.dtype_code(qkv), _lib.stream(qkv))
    _lib.check(rc, "qkv_rope_rms")
    return q, k, v


def qkv_rope_rms_simd(qkv, cos, sin, gamma_q, gamma_k, batch, heads, head_dim, group=16):
    """Subgroup-cooperative variant of :func:`qkv_rope_rms` (kernels.py:137-157).

    On B200 both names run the same warp-cooperative kernel (a lane group per
    head, shuffle-reduced norm); ``group`` is validated as the reference does.
    """
    if group not in (8, 16, 32) or head_dim % 2:
        raise ValueError("an even head dimension and subgroup width 8, 16 or 32 are required")
    return qkv_rope_rms(qkv, cos, sin, gamma_q, gamma_k, batch, heads, head_dim)


def gate_residual(x: torch.Tensor, y: torch.Tensor, gate: torch.Tensor | None) -> torch.Tensor:
    """``x + y * gate`` with two roundings in ``x``'s dtype, written into ``x`` (in place).

    ``x``/``y`` ``[B, N, C]`` or ``[R, C]``; ``gate`` ``[C]``, ``[1, C]`` or ``[B, C]``.
    Reference: transformer.py:570, :588.
    """
    _lib.require_cuda(x, y, gate)
    c = x.shape[-1]
    rows = x.numel() // c
    if not x.is_contiguous():
        raise ValueError("gate_residual updates x in place; x must be contiguous")
    y = y.contiguous()
    rows_per_batch, stride = rows, 0
    if gate is not None:
        gate = gate.to(x.dtype).reshape(-1, c).contiguous()
        if gate.shape[0] > 1:
            rows_per_batch, stride = rows // gate.shape[0], c
    rc = _lib.load().hi3d_gate_residual(x.data_ptr(), y.data_ptr(), _lib.ptr(gate), rows, c, rows_per_batch, stride,
                                        _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "gate_residual")
    return x


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """tanh-approximated GELU in fp32, rounded once (transformer.py:176-179)."""
    _lib.require_cuda(x)
    x = x.contiguous()
    out = torch.empty_like(x)
    rc = _lib.load().hi3d_gelu_tanh(x.data_ptr(), out.data_ptr(), x.numel(), _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "gelu_tanh")
    return out
