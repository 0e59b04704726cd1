"""Projections on the tcgen05 GEMM with fused epilogues (``hi3d_gemm`` of the C ABI).

``linear(x, weight, bias)`` is ``x @ weight^T + bias`` in the weight dtype with fp32
accumulation, as ``mx.addmm`` in the reference block (src/hi3d_mac/mlx_backend/transformer.py:111-119,
501-516).  The epilogue can also apply the block's tanh-GELU (transformer.py:587) or update the
residual stream in place, ``x = x + y * gate`` (transformer.py:570, :588), saving a pass over HBM.
"""

from __future__ import annotations

import torch

from . import _lib

_EPI = {"store": _lib.EPI_STORE, "gelu": _lib.EPI_GELU, "residual": _lib.EPI_RESIDUAL}


def _gate_args(gate: torch.Tensor | None, rows: int, n: int, dtype: torch.dtype):
    if gate is None:
        return None, rows, 0
    gate = gate.to(dtype).reshape(-1, n).contiguous()
    nb = gate.shape[0]
    if rows % nb:
        raise ValueError("gate batch does not divide the rows")
    return gate, rows // nb, (n if nb > 1 else 0)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, epilogue: str = "store",
           residual: torch.Tensor | None = None, gate: torch.Tensor | None = None) -> torch.Tensor:
    """``y = x @ weight^T + bias`` (x ``[..., K]``, weight ``[N, K]``), then the epilogue:
    ``"store"`` returns y, ``"gelu"`` returns gelu_tanh(y), ``"residual"`` adds ``y * gate`` into
    ``residual`` (``[..., N]``, contiguous, updated in place and returned); ``gate`` is ``[N]`` or
    ``[B, N]`` for ``residual [B, rows, N]``."""
    _lib.require_cuda(x, weight, bias, residual, gate)
    if x.dtype not in (torch.float16, torch.bfloat16) or weight.dtype != x.dtype:
        raise ValueError("linear takes float16/bfloat16 activations and weights of one dtype")
    k = x.shape[-1]
    n, kw = weight.shape
    if kw != k:
        raise ValueError(f"incompatible shapes x {tuple(x.shape)} weight {tuple(weight.shape)}")
    a = x.reshape(-1, k)
    if not a.is_contiguous():
        a = a.contiguous()
    w = weight.contiguous()
    m = a.shape[0]
    if bias is not None:
        bias = bias.to(x.dtype).contiguous()
    epi = _EPI[epilogue]
    if epilogue == "residual":
        if residual is None or residual.shape[-1] != n or residual.numel() != m * n or not residual.is_contiguous():
            raise ValueError("residual epilogue needs a contiguous residual [..., N] with the rows of x")
        out = residual
    else:
        out = torch.empty((*x.shape[:-1], n), dtype=x.dtype, device=x.device)
    g, rpb, gs = _gate_args(gate, m, n, x.dtype)
    rc = _lib.load().hi3d_gemm(a.data_ptr(), w.data_ptr(), _lib.ptr(bias), out.data_ptr(), m, n, k, n, epi,
                               _lib.ptr(g), rpb, gs, _lib.dtype_code(x), _lib.stream(x))
    _lib.check(rc, "linear")
    return out
