"""The sparse-DiT refinement block and its 24-block stack on B200.

Mirrors ``Sparc3DTransformerMLX._block_fn.block`` (src/hi3d_mac/mlx_backend/transformer.py:543-588)
operation by operation, which in turn mirrors the upstream
``ModulatedSparseTransformerCrossBlock.forward`` (src/sparc3d/nn/sparse/transformer/modulated.py:45-65):

1. ``parts = modulation(fp32) + mod``; shift/gate cast to the torso dtype; ``scale = (1 + parts)`` cast
2. ``h = LN(x) * scale_msa + shift_msa``                       (fused LN-modulate kernel)
3. ``qkv = h @ Wqkv^T + b``                                    (GEMM)
4. RoPE + QK RMS norm + split ``[B, H, N, D]``                (fused kernel)
5. self-attention                                             (tcgen05 flash attention)
6. ``x = x + (a @ Wout^T + b) * gate_msa``                      (GEMM + gate/residual kernel)
7. ``h = LN(x; norm2)``; cross-attention to the cached condition K/V; ``x = x + cross``
8. ``h = LN(x) * scale_mlp + shift_mlp``; ``x = x + mlp(h) * gate_mlp`` (GELU-tanh in fp32)

``x`` is ``[B, N, C]`` with ``n_pos`` conditioned branches first and optionally one zero-condition
branch last, whose cross-attention is the constant ``negative = to_out(v_bias)``
(transformer.py:396-409).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import attention, kernels
from . import linear as _linear
from . import w8a8 as _w8a8

# fp16 GEMMs accumulate in fp32, as mx.addmm does (transformer.py:119).
torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False


@dataclass(frozen=True)
class Precision:
    """Torso precision (transformer.py:50-67): ``dtype`` of activations/GEMMs and the GEMM mode."""

    dtype: torch.dtype = torch.float16
    gemm: str = "fp16"  # "fp16" (GEMM in ``dtype``) or "w8a8" (int8 activations and weights)


def rope_tables(coords: np.ndarray, head_dim: int = 96) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin ``[N, head_dim/2]`` fp32 of ``RotaryPositionEmbedder`` for ``coords``
    (transformer.py:189-210; upstream src/sparc3d/nn/rope.py:38-58, 82-90): ``head_dim//3//2``
    frequencies per axis, NTK rescale when the largest coordinate is >= 64, phases ordered
    ``[x f, y f, z f]``, remaining pairs padded with cos 1 / sin 0."""
    freq_dim = head_dim // 3 // 2
    freqs = (1.0 / (10000.0 ** (np.arange(freq_dim, dtype=np.float32) / np.float32(freq_dim)))).astype(np.float32)
    max_length = int(coords.max())
    if max_length >= 64:
        train, infer = 64, (64 + max_length) // 2
        wavelengths = freqs * train / (2 * math.pi)
        ratio = (wavelengths - 1) / (24 - 1)
        ratio = ratio + (1 - ratio) * train / infer
        ratio = np.where(wavelengths > 24, 1.0, ratio)
        ratio = np.where(wavelengths < 1, train / infer, ratio)
        freqs = (freqs * ratio).astype(np.float32)
    phases = (coords.astype(np.float32).reshape(-1)[:, None] * freqs[None, :]).reshape(coords.shape[0], -1)
    pad = head_dim // 2 - phases.shape[1]
    cos, sin = np.cos(phases), np.sin(phases)
    if pad > 0:
        cos = np.concatenate([cos, np.ones((cos.shape[0], pad), np.float32)], 1)
        sin = np.concatenate([sin, np.zeros((sin.shape[0], pad), np.float32)], 1)
    return cos.astype(np.float32), sin.astype(np.float32)


def to_device(w: dict, device, dtype: torch.dtype = torch.float16) -> dict:
    """Block parameters on the device: fp16 tensors in the torso dtype, fp32 kept fp32."""
    out = {}
    for k, v in w.items():
        t = torch.as_tensor(np.ascontiguousarray(v))
        out[k] = t.to(device=device, dtype=dtype if t.dtype == torch.float16 else t.dtype)
    return out


def linear(x: torch.Tensor, w: dict, name: str, epilogue: str = "store", residual: torch.Tensor | None = None,
           gate: torch.Tensor | None = None) -> torch.Tensor:
    """Projection ``name`` of a block: ``x @ W^T + b`` on the tcgen05 GEMM, in the weight dtype
    with fp32 accumulation (transformer.py:111-119), or through int8 when the block holds W8A8
    weights (``<name>.w8_scale`` present, the hook at transformer.py:504-507).  ``epilogue``
    fuses GELU or the gated residual update into the GEMM."""
    if f"{name}.w8_scale" in w:
        return _w8a8.linear(x, w[f"{name}.weight"], w[f"{name}.w8_scale"], w[f"{name}.bias"], epilogue=epilogue,
                            residual=residual, gate=gate)
    return _linear.linear(x, w[f"{name}.weight"], w[f"{name}.bias"], epilogue=epilogue, residual=residual, gate=gate)


def qkv_rope(h: torch.Tensor, w: dict, cos: torch.Tensor, sin: torch.Tensor, batch: int, heads: int, d: int,
             token_major: bool = False, out: tuple | None = None, peer_offsets: tuple[int, ...] = (),
             multicast_offset: int = 0):
    """``q, k, v`` of the self-attention: the ``self_attn.to_qkv`` projection with RoPE + QK RMS
    norm (transformer.py:501-516 then kernels.py:22-90).  Fused into the GEMM epilogue when the
    head layout allows it (head dim 64), else the projection followed by the row kernel.
    ``out``: optional ``(q, k, v)`` tensors written in place of new ones.  ``peer_offsets`` /
    ``multicast_offset``: the fused projection also stores K/V into the peers' gather buffers
    (only the fused form can; ``NotImplementedError`` otherwise)."""
    name = "self_attn.to_qkv"
    gq, gk = w["self_attn.q_rms_norm.gamma"], w["self_attn.k_rms_norm.gamma"]
    if _linear.qkv_rope_supported(heads, d):
        if f"{name}.w8_scale" in w:
            return _w8a8.linear_qkv_rope(h, w[f"{name}.weight"], w[f"{name}.w8_scale"], w[f"{name}.bias"], cos, sin,
                                         gq, gk, batch, heads, d, token_major, out=out, peer_offsets=peer_offsets,
                                         multicast_offset=multicast_offset)
        return _linear.linear_qkv_rope(h, w[f"{name}.weight"], w[f"{name}.bias"], cos, sin, gq, gk, batch, heads, d,
                                       token_major, out=out, peer_offsets=peer_offsets,
                                       multicast_offset=multicast_offset)
    if peer_offsets or multicast_offset:
        raise NotImplementedError("peer stores need the fused QKV projection (head_dim 64, heads * 64 % 256 == 0)")
    qkv = linear(h, w, name)
    return kernels.qkv_rope_rms(qkv, cos, sin, gq, gk, batch, heads, d, token_major=token_major, out=out)


BLOCK_PROJECTIONS = ("self_attn.to_qkv", "self_attn.to_out", "cross_attn.to_q", "cross_attn.to_out", "mlp.mlp.0",
                     "mlp.mlp.2")


def to_w8a8(w: dict, rotate: bool = True) -> dict:
    """Block weights in the ``hi3d-w8a8-h64`` form: the six block projections as int8 rows in
    the rotated domain plus ``<name>.w8_scale`` (models/w8a8/manifest.json:9-16); the condition
    K/V projection, norms and modulation stay as they are."""
    out = dict(w)
    for name in BLOCK_PROJECTIONS:
        q, s = _w8a8.quantize_weight(w[f"{name}.weight"], rotate=rotate)
        out[f"{name}.weight"] = q
        out[f"{name}.w8_scale"] = s
    return out


def context_kv(w: dict, cond: torch.Tensor, heads: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Cross-attention ``k, v`` views ``[1, H, L, D]`` of the projected condition ``[L, Cc]``
    (transformer.py:382-394), computed once per pass."""
    kv = linear(cond, w, "cross_attn.to_kv")
    L, c2 = kv.shape
    d = c2 // 2 // heads
    kv = kv.view(L, 2, heads, d)
    return kv[:, 0].permute(1, 0, 2).unsqueeze(0), kv[:, 1].permute(1, 0, 2).unsqueeze(0)


def negative_cross(w: dict) -> torch.Tensor:
    """``to_out(v_bias)``: cross-attention output for the all-zero condition (transformer.py:396-409)."""
    c = w["cross_attn.to_out.weight"].shape[0]
    v_bias = w["cross_attn.to_kv.bias"][c:].unsqueeze(0)
    return linear(v_bias, w, "cross_attn.to_out")


def _norm_for(w: dict, name: str):
    """The norm feeding projection ``name``: LayerNorm-modulate into 16-bit rows, or, when the
    projection is W8A8, fused with the activation quantiser (the int8 rows and scales the
    projection would compute itself; the 16-bit rows are never written)."""
    if f"{name}.w8_scale" in w:
        return _w8a8.layer_norm_quantize
    return kernels.layer_norm_modulate


def _modulation(w: dict, mod: torch.Tensor, c: int, dt: torch.dtype):
    """shift/gate in the torso dtype and ``(1 + scale)`` rounded to it (transformer.py:545-548)."""
    parts = (w["modulation"] + mod.float()).view(6, c)
    shift_msa, gate_msa, shift_mlp, gate_mlp = (parts[j].to(dt) for j in (0, 2, 3, 5))
    scale_msa, scale_mlp = ((1 + parts[j]).to(dt) for j in (1, 4))
    return shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp


def modulation_all(mod_w: torch.Tensor, mod: torch.Tensor, c: int, dt: torch.dtype) -> list[tuple]:
    """:func:`_modulation` of every block at once: ``mod_w [blocks, 6C]`` stacked block
    parameters; same element-wise operations, so the values are identical."""
    parts = (mod_w + mod.float().reshape(1, -1)).view(mod_w.shape[0], 6, c)
    sg = parts[:, [0, 2, 3, 5]].to(dt)
    sc = (1 + parts[:, [1, 4]]).to(dt)
    return [(sg[i, 0], sc[i, 0], sg[i, 1], sg[i, 2], sc[i, 1], sg[i, 3]) for i in range(mod_w.shape[0])]


def block_forward(w: dict, x: torch.Tensor, mod: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  ck: torch.Tensor | None, cv: torch.Tensor | None, negative: torch.Tensor | None, heads: int,
                  n_pos: int = 1, inplace: bool = False, shared_self: bool = False,
                  mods: tuple | None = None) -> torch.Tensor:
    """One block on ``x [B, N, C]`` (the MLX form, transformer.py:543-588): ``B`` branches of one
    object, ``n_pos`` conditioned by the cached condition K/V ``(ck, cv) [1, H, L, D]`` and the
    rest by the zero condition (constant ``negative [1, C]``).

    ``inplace=True`` updates ``x`` (the stack does this to avoid a copy per block).
    ``shared_self=True`` states that every branch holds the same ``x`` (the first block of a
    guided evaluation): the self-attention sub-layer then runs once and its result is copied to
    the other branches, which is bit-identical because rows of every kernel are independent
    (the reference's shared first-block attention, transformer.py:550-569, 656-664).
    ``mods``: this block's modulation vectors precomputed by :func:`modulation_all`.
    """
    batch, n, c = x.shape
    dt = x.dtype
    d = c // heads
    scale = d ** -0.5
    if not inplace:
        x = x.clone()
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = mods if mods is not None else \
        _modulation(w, mod, c, dt)

    # self-attention
    xs = x[:1] if shared_self and batch > 1 else x
    h = _norm_for(w, "self_attn.to_qkv")(xs, 1e-6, scale=scale_msa, shift=shift_msa)
    q, k, v = qkv_rope(h.view(-1, c), w, cos, sin, xs.shape[0], heads, d)
    a = attention.flash_attention(q, k, v, scale)
    linear(a, w, "self_attn.to_out", epilogue="residual", residual=xs, gate=gate_msa)
    if xs.shape[0] != batch:
        x[1:].copy_(xs.expand(batch - 1, n, c))

    # cross-attention (positive branches), constant for the zero-condition branch
    h = _norm_for(w, "cross_attn.to_q")(x, 1e-6, weight=w["norm2.weight"], bias=w["norm2.bias"])
    for b in range(n_pos):
        qc = linear(h[b], w, "cross_attn.to_q").view(1, n, heads, d)
        o = attention.flash_attention(qc, ck, cv, scale, q_layout="bnhd")[0]
        linear(o, w, "cross_attn.to_out", epilogue="residual", residual=x[b])
    if negative is not None:
        for b in range(n_pos, batch):
            kernels.gate_residual(x[b], negative.to(dt).expand(n, c).contiguous(), None)

    # MLP
    h = _norm_for(w, "mlp.mlp.0")(x, 1e-6, scale=scale_mlp, shift=shift_mlp)
    h = linear(h, w, "mlp.mlp.0", epilogue="gelu")
    linear(h, w, "mlp.mlp.2", epilogue="residual", residual=x, gate=gate_mlp)
    return x


def block_forward_packed(w: dict, x: torch.Tensor, mod: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         ck: torch.Tensor, cv: torch.Tensor, heads: int, cu_seqlens: torch.Tensor,
                         max_seqlen: int, inplace: bool = False) -> torch.Tensor:
    """One block on packed objects ``x [T, C]`` (the upstream ``SparseTensor`` form,
    modulated.py:45-65): self-attention within each object (``cu_seqlens`` int32 on the
    device), cross-attention of every object to the shared condition K/V ``[1, H, L, D]``.
    ``cos``/``sin`` are ``[T, D/2]`` for the packed rows."""
    t, c = x.shape
    dt = x.dtype
    d = c // heads
    scale = d ** -0.5
    if not inplace:
        x = x.clone()
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = _modulation(w, mod, c, dt)

    h = _norm_for(w, "self_attn.to_qkv")(x, 1e-6, scale=scale_msa, shift=shift_msa)
    q, k, v = qkv_rope(h, w, cos, sin, 1, heads, d)
    tr = lambda z: z[0].permute(1, 0, 2)  # [1, H, T, D] -> [T, H, D] view
    a = attention.flash_attn_varlen(tr(q), tr(k), tr(v), cu_seqlens, cu_seqlens, max_seqlen, scale)
    linear(a.view(t, c), w, "self_attn.to_out", epilogue="residual", residual=x, gate=gate_msa)

    h = _norm_for(w, "cross_attn.to_q")(x, 1e-6, weight=w["norm2.weight"], bias=w["norm2.bias"])
    qc = linear(h, w, "cross_attn.to_q").view(t, heads, d)
    o = attention.flash_attn_varlen(qc, ck[0].permute(1, 0, 2), cv[0].permute(1, 0, 2), cu_seqlens, None,
                                    max_seqlen, scale)
    linear(o.view(t, c), w, "cross_attn.to_out", epilogue="residual", residual=x)

    h = _norm_for(w, "mlp.mlp.0")(x, 1e-6, scale=scale_mlp, shift=shift_mlp)
    h = linear(h, w, "mlp.mlp.0", epilogue="gelu")
    linear(h, w, "mlp.mlp.2", epilogue="residual", residual=x, gate=gate_mlp)
    return x


class BlockStack:
    """``num_blocks`` blocks of one architecture (transformer.py:656-667): the refinement torso."""

    def __init__(self, weights: list[dict], heads: int):
        self.weights = weights
        self.heads = heads
        self._mod_w = None  # [blocks, 6C] stacked modulation parameters (built on first use)

    def prepare(self, cond: torch.Tensor) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """Per-block condition K/V for a ``[L, Cc]`` condition (once per sampling pass)."""
        return [context_kv(w, cond, self.heads) for w in self.weights]

    def __call__(self, x: torch.Tensor, mod: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 kvs: list[tuple[torch.Tensor, torch.Tensor]], negatives: list[torch.Tensor] | None = None,
                 n_pos: int = 1, shared_input: bool = False) -> torch.Tensor:
        """``shared_input=True``: every branch of ``x`` holds the same rows (a guided evaluation),
        so the first block's self-attention runs once."""
        x = x.clone()
        if self._mod_w is None:
            self._mod_w = torch.stack([w["modulation"].reshape(-1).float() for w in self.weights])
        mods = modulation_all(self._mod_w, mod, x.shape[-1], x.dtype)
        for i, w in enumerate(self.weights):
            ck, cv = kvs[i] if kvs is not None else (None, None)
            neg = None if negatives is None else negatives[i]
            block_forward(w, x, mod, cos, sin, ck, cv, neg, self.heads, n_pos=n_pos, inplace=True,
                          shared_self=shared_input and i == 0, mods=mods[i])
        return x
