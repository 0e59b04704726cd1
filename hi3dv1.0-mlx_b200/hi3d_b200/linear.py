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


def qkv_rope_supported(heads: int, head_dim: int) -> bool:
    """Whether :func:`linear_qkv_rope` handles this head layout (head dim 64, ``heads * 64``
    a multiple of the 256-column GEMM tile)."""
    return head_dim == 64 and (heads * 64) % 256 == 0


def qkv_outputs(shape: tuple, dtype: torch.dtype, device, out: tuple | None):
    """``q, k, v`` output tensors of ``shape``: new ones, or the caller's (``out``), which must be
    contiguous tensors of that shape and dtype on the device (e.g. this rank's slot of a K/V
    gather buffer, so the projection writes there directly)."""
    if out is None:
        q = torch.empty(shape, dtype=dtype, device=device)
        return q, torch.empty_like(q), torch.empty_like(q)
    for t in out:
        if t is not None and (tuple(t.shape) != tuple(shape) or t.dtype != dtype or not t.is_contiguous()
                              or t.device != torch.device(device)):
            raise ValueError(f"q/k/v outputs must be contiguous {tuple(shape)} {dtype} tensors on {device}")
    return tuple(torch.empty(shape, dtype=dtype, device=device) if t is None else t for t in out)


def _qkv_rope_args(x, cos, sin, gamma_q, gamma_k, batch, heads, head_dim, token_major, dtype, out=None):
    k = x.shape[-1]
    a = x.reshape(-1, k)
    if not a.is_contiguous():
        a = a.contiguous()
    m = a.shape[0]
    if m % batch:
        raise ValueError("rows must be batch * n")
    n = m // batch
    cos = cos.float().contiguous()
    sin = sin.float().contiguous()
    if cos.shape != (n, head_dim // 2) or sin.shape != (n, head_dim // 2):
        raise ValueError(f"cos/sin must be [N, D/2] = [{n}, {head_dim // 2}]")
    gq = gamma_q.float().reshape(heads, head_dim).contiguous()
    gk = gamma_k.float().reshape(heads, head_dim).contiguous()
    shape = (batch, n, heads, head_dim) if token_major else (batch, heads, n, head_dim)
    q, k, v = qkv_outputs(shape, dtype, x.device, out)
    return a, m, n, cos, sin, gq, gk, q, k, v


def linear_qkv_rope(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, cos: torch.Tensor,
                    sin: torch.Tensor, gamma_q: torch.Tensor, gamma_k: torch.Tensor, batch: int, heads: int,
                    head_dim: int, token_major: bool = False, out: tuple | None = None,
                    peer_offsets: tuple[int, ...] = (), multicast_offset: int = 0):
    """The attention input projection ``x @ W^T + bias`` (``W [3 H D, K]``) split into
    ``q, k, v [B, H, N, D]`` with RoPE + QK RMS norm applied in the GEMM epilogue: the same
    result as :func:`linear` followed by :func:`hi3d_b200.kernels.qkv_rope_rms`
    (transformer.py:501-516, kernels.py:22-90) without writing the projection to memory.
    ``token_major=True`` returns ``[B, N, H, D]``.  ``out``: optional ``(q, k, v)`` tensors to write
    (None entries are allocated).  ``peer_offsets``: byte offsets from ``k``/``v`` to the same rows of
    the peers' gather buffers, which the epilogue also stores (``hi3d_gemm_qkv_rope_peers``; see
    :class:`hi3d_b200.peer.PeerKV`); or ``multicast_offset``: byte offset from ``k``/``v`` to their
    NVLink multicast mapping, stored once for every GPU.  Raises ``NotImplementedError`` unless
    :func:`qkv_rope_supported`."""
    _lib.require_cuda(x, weight, bias, cos, sin, gamma_q, gamma_k)
    if x.dtype not in (torch.float16, torch.bfloat16) or weight.dtype != x.dtype:
        raise ValueError("linear_qkv_rope takes float16/bfloat16 activations and weights of one dtype")
    if weight.shape != (3 * heads * head_dim, x.shape[-1]):
        raise ValueError(f"weight must be [3*H*D, K], got {tuple(weight.shape)}")
    a, m, n, cos, sin, gq, gk, q, k, v = _qkv_rope_args(x, cos, sin, gamma_q, gamma_k, batch, heads, head_dim,
                                                        token_major, x.dtype, out)
    b = None if bias is None else bias.to(x.dtype).contiguous()
    offs = peer_offset_array(peer_offsets)
    rc = _lib.load().hi3d_gemm_qkv_rope_peers(a.data_ptr(), weight.contiguous().data_ptr(), _lib.ptr(b),
                                              cos.data_ptr(), sin.data_ptr(), gq.data_ptr(), gk.data_ptr(),
                                              q.data_ptr(), k.data_ptr(), v.data_ptr(), m, n, heads, head_dim,
                                              a.shape[1], int(token_major), _lib.dtype_code(x), offs,
                                              len(peer_offsets), int(multicast_offset), _lib.stream(x))
    _lib.check(rc, "linear_qkv_rope")
    return q, k, v


def peer_offset_array(peer_offsets: tuple[int, ...]):
    """The host ``int64`` array of peer byte offsets for the ``*_qkv_rope_peers`` entries (None
    when empty)."""
    import ctypes

    if not peer_offsets:
        return None
    return (ctypes.c_int64 * len(peer_offsets))(*[int(o) for o in peer_offsets])
