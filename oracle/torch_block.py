"""The reference's own CPU path of one sparse-DiT block, restated in torch fp32.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module: ``tests/`` use it as
the checker for the full-size parity tests (cfg1 / cfg2 blocks on sampled rows, the 24-block
stack), and ``bench.py``'s reference arm times it as the CPU baseline.

What it restates.  The reference runs the upstream PyTorch block on CPU with its torch shims
registered in place of CUDA-only ``flash_attn`` (src/hi3d_mac/torch_backend/__init__.py:34-64):

* ``ModulatedSparseTransformerCrossBlock.forward``
  (src/sparc3d/nn/sparse/transformer/modulated.py:45-65): adaLN chunks of
  ``modulation + mod``, LayerNorm32 without/with affine (src/sparc3d/nn/norm.py:12-17),
  gated residuals, GELU(tanh) MLP (src/sparc3d/nn/sparse/transformer/blocks.py);
* ``SparseMultiHeadAttention.forward`` (src/sparc3d/nn/sparse/attention/modules.py:97-123):
  fused QKV, rotary embedding as a complex product in fp32 (src/sparc3d/nn/rope.py:66-93), then
  ``F.normalize(x) * gamma * sqrt(D)`` per head (modules.py:17-32), cross K/V from the context;
* the ``flash_attn`` varlen shim (src/hi3d_mac/torch_backend/attention.py:20-72): fp32
  ``F.scaled_dot_product_attention`` per sequence, queries split into blocks whose score matrix
  ``heads x block x keys`` stays within 768 MiB.

The cos/sin tables are the reference's ``rope_tables`` values (cos/sin of the same phases the
upstream embedder builds with ``torch.polar``).  ``tests/test_oracle_golden.py`` pins this
function to the upstream module's output (``tests/golden/block.npz``).
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

SCORE_BYTES = 768 * 1024 * 1024  # torch_backend/attention.py:16


def _t(a) -> torch.Tensor:
    return a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))


def weights_f32(w: dict) -> dict:
    """The block's parameters as fp32 CPU tensors (the reference holds them in fp32 on CPU)."""
    return {k: _t(v).float() for k, v in w.items()}


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """One sequence ``q [Lq, H, D]`` over ``k, v [Lk, H, D]`` -> ``[Lq, H, D]`` fp32, queries in
    blocks of at most SCORE_BYTES of scores (torch_backend/attention.py:20-38)."""
    heads, lk = q.shape[1], k.shape[0]
    qf, kf, vf = (t.float().transpose(0, 1)[None] for t in (q, k, v))
    block = max(1, min(q.shape[0], SCORE_BYTES // max(1, heads * lk * 4)))
    outs = [F.scaled_dot_product_attention(qf[:, :, s:s + block], kf, vf, scale=scale)
            for s in range(0, q.shape[0], block)]
    return torch.cat(outs, 2)[0].transpose(0, 1)


def _rope_norm(z: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """Rotate adjacent pairs by the token's phases, then per-head L2 normalisation * gamma * sqrt(D)."""
    t, heads, d = z.shape
    zz = z.reshape(t, heads, d // 2, 2)
    c, s = cos[:, None, :], sin[:, None, :]
    re = zz[..., 0] * c - zz[..., 1] * s
    im = zz[..., 0] * s + zz[..., 1] * c
    y = torch.stack([re, im], -1).reshape(t, heads, d)
    return F.normalize(y, dim=-1) * gamma * math.sqrt(d)


def _ln(x: torch.Tensor, weight=None, bias=None) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps=1e-6)


def block_forward(w: dict, x, mod, cos, sin, ctx, heads: int, seqlens: list[int] | None = None,
                  rows=None) -> torch.Tensor:
    """The block's fp32 output ``[T, C]`` for packed tokens ``x [T, C]`` (objects of ``seqlens``
    tokens), or only its rows ``rows`` (sorted indices): keys and values of self-attention then
    still come from every token, every per-query step runs on the selected rows alone.

    ``w`` as :func:`weights_f32` returns (or raw arrays), ``mod [1, 6C]``, ``cos/sin [T, D/2]``,
    ``ctx [L, Cc]`` shared by every object.
    """
    if not isinstance(w.get("modulation"), torch.Tensor) or w["modulation"].dtype != torch.float32:
        w = weights_f32(w)
    x = _t(x).float()
    cos, sin, ctx, mod = (_t(a).float() for a in (cos, sin, ctx, mod))
    t, c = x.shape
    d = c // heads
    seqlens = list(seqlens or [t])
    bounds = np.concatenate([[0], np.cumsum(seqlens)]).astype(np.int64)
    sel = None if rows is None else torch.as_tensor(np.asarray(rows, np.int64))
    parts = (w["modulation"] + mod).reshape(6, c)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = parts

    def lin(h, name, lo=None, hi=None):
        wt, b = w[f"{name}.weight"], w[f"{name}.bias"]
        if lo is not None:
            wt, b = wt[lo:hi], b[lo:hi]
        return F.linear(h, wt, b)

    # self-attention: keys/values of every token, queries of the selected rows
    h = _ln(x) * (1 + scale_msa) + shift_msa
    k = _rope_norm(lin(h, "self_attn.to_qkv", c, 2 * c).reshape(t, heads, d), cos, sin,
                   w["self_attn.k_rms_norm.gamma"])
    v = lin(h, "self_attn.to_qkv", 2 * c, 3 * c).reshape(t, heads, d)
    hq, cq, sq, xq = (h, cos, sin, x) if sel is None else (h[sel], cos[sel], sin[sel], x[sel])
    q = _rope_norm(lin(hq, "self_attn.to_qkv", 0, c).reshape(-1, heads, d), cq, sq, w["self_attn.q_rms_norm.gamma"])
    qrows = np.arange(t) if sel is None else sel.numpy()
    a = torch.empty_like(q)
    for i in range(len(seqlens)):
        lo, hi = int(bounds[i]), int(bounds[i + 1])
        qi = np.nonzero((qrows >= lo) & (qrows < hi))[0]
        if len(qi) == 0:
            continue
        a[qi] = attend(q[qi], k[lo:hi], v[lo:hi], d ** -0.5)
    xq = xq + lin(a.reshape(-1, c), "self_attn.to_out") * gate_msa
    # cross-attention to the shared condition
    h = _ln(xq, w["norm2.weight"], w["norm2.bias"])
    qc = lin(h, "cross_attn.to_q").reshape(-1, heads, d)
    kv = lin(ctx, "cross_attn.to_kv").reshape(-1, 2, heads, d)
    o = attend(qc, kv[:, 0], kv[:, 1], d ** -0.5)
    xq = xq + lin(o.reshape(-1, c), "cross_attn.to_out")
    # MLP
    h = _ln(xq) * (1 + scale_mlp) + shift_mlp
    h = F.gelu(lin(h, "mlp.mlp.0"), approximate="tanh")
    return xq + lin(h, "mlp.mlp.2") * gate_mlp
