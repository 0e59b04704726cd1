"""``flash_attn`` varlen functions backed by the B200 tcgen05 attention kernel.

Same signatures as the functions the upstream code calls
(src/sparc3d/nn/sparse/attention/full_attn.py:56-76) and as the reference's CPU shim
(src/hi3d_mac/torch_backend/attention.py:77-109), including its errors for causal or
dropout attention.  Inputs are fp16/bf16 CUDA tensors, as for flash-attn itself.
"""

from __future__ import annotations

import torch

from .. import attention as _attn


def flash_attn_varlen_qkvpacked_func(qkv: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int,
                                     dropout_p: float = 0.0, softmax_scale: float | None = None,
                                     causal: bool = False, **_: object) -> torch.Tensor:
    """Self-attention over packed ``[T, 3, H, D]`` sequences; returns ``[T, H, D]``."""
    if causal or dropout_p:
        raise NotImplementedError("causal or dropout attention is not used by Hi3D")
    q, k, v = qkv.unbind(1)
    scale = q.shape[-1] ** -0.5 if softmax_scale is None else softmax_scale
    return _attn.flash_attn_varlen(q, k, v, cu_seqlens, cu_seqlens, int(max_seqlen), scale)


def flash_attn_varlen_kvpacked_func(q: torch.Tensor, kv: torch.Tensor, cu_seqlens_q: torch.Tensor,
                                    cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int,
                                    dropout_p: float = 0.0, softmax_scale: float | None = None,
                                    causal: bool = False, **_: object) -> torch.Tensor:
    """Cross-attention of packed queries ``[T, H, D]`` over packed ``[S, 2, H, D]``."""
    if causal or dropout_p:
        raise NotImplementedError("causal or dropout attention is not used by Hi3D")
    k, v = kv.unbind(1)
    scale = q.shape[-1] ** -0.5 if softmax_scale is None else softmax_scale
    return _attn.flash_attn_varlen(q, k, v, cu_seqlens_q.to(q.device), cu_seqlens_k.to(q.device),
                                   int(max_seqlen_q), scale)
