"""Query-sharded execution of the block stack across the GPUs of one node.

Rank ``r`` of ``P`` owns a contiguous slice of the object's tokens (query rows).
Everything in the block is row-local except self-attention, which needs the
keys/values of every token: each block all-gathers K and V (token-major
``[T/P, H, D]`` shards -> ``[T, H, D]``) with NCCL over NVLink, then runs the
local queries against all keys.  Cross-attention K/V (the condition) are
replicated.  This is a plain context-parallel split; softmax rows never cross
ranks, so the result equals the single-GPU block up to GEMM shape effects.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import attention, kernels
from .transformer import _modulation, linear, qkv_rope


def shard_slice(total: int, rank: int, world: int) -> slice:
    """Contiguous query-row slice of ``rank``: the rows ``[rank * total / world, ...)``."""
    if total % world:
        raise ValueError(f"{total} rows do not split evenly over {world} ranks")
    per = total // world
    return slice(rank * per, (rank + 1) * per)


def gather_rows(local: torch.Tensor, group=None, out: torch.Tensor | None = None, async_op: bool = False):
    """All-gather equal row shards ``[rows, ...]`` of every rank into ``[world * rows, ...]`` in rank
    order (NCCL over NVLink for CUDA tensors, gloo for CPU tensors)."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
    work = dist.all_gather_into_tensor(out, local.contiguous(), group=group, async_op=async_op)
    return (out, work) if async_op else out


def block_forward_sharded(w: dict, x: torch.Tensor, mod: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                          ck: torch.Tensor, cv: torch.Tensor, heads: int, group=None,
                          kv_buffers: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """One block on this rank's rows ``x [T/P, C]`` (updated in place) of a single object."""
    t_local, c = x.shape
    world = dist.get_world_size(group)
    d = c // heads
    scale = d ** -0.5
    dt = x.dtype
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = _modulation(w, mod, c, dt)

    h = kernels.layer_norm_modulate(x, 1e-6, scale=scale_msa, shift=shift_msa)
    q, k, v = qkv_rope(h, w, cos, sin, 1, heads, d, token_major=True)
    if kv_buffers is None:
        kv_buffers = tuple(torch.empty((world * t_local, heads, d), dtype=dt, device=x.device) for _ in range(2))
    k_all, v_all = kv_buffers
    _, hk = gather_rows(k[0], group, out=k_all, async_op=True)
    _, hv = gather_rows(v[0], group, out=v_all, async_op=True)
    # Attend to this rank's own keys while the others are being gathered, then to the keys
    # before and after the local shard; the partials are merged by their log-sum-exp weights.
    rank = dist.get_rank(group)
    bhnd = lambda t: t.permute(1, 0, 2)[None]  # [rows, H, D] token-major -> [1, H, rows, D] view
    key_sets = [(0, rank * t_local), ((rank + 1) * t_local, world * t_local)]
    splits = [attention.auto_key_splits(t_local, t_local, heads, d, device=x.device)]
    splits += [attention.auto_key_splits(t_local, hi - lo, heads, d, device=x.device) for lo, hi in key_sets if hi > lo]
    parts = attention.AttentionParts(q, scale, sum(splits), q_layout="bnhd")
    parts.add(bhnd(k[0]), bhnd(v[0]), splits[0])
    hk.wait()
    hv.wait()
    i = 1
    for lo, hi in key_sets:
        if hi > lo:
            parts.add(bhnd(k_all[lo:hi]), bhnd(v_all[lo:hi]), splits[i])
            i += 1
    a = parts.merge()
    linear(a[0], w, "self_attn.to_out", epilogue="residual", residual=x, gate=gate_msa)

    h = kernels.layer_norm_modulate(x, 1e-6, weight=w["norm2.weight"], bias=w["norm2.bias"])
    qc = linear(h, w, "cross_attn.to_q").view(1, t_local, heads, d)
    o = attention.flash_attention(qc, ck, cv, scale, q_layout="bnhd")[0]
    linear(o, w, "cross_attn.to_out", epilogue="residual", residual=x)

    h = kernels.layer_norm_modulate(x, 1e-6, scale=scale_mlp, shift=shift_mlp)
    h = linear(h, w, "mlp.mlp.0", epilogue="gelu")
    linear(h, w, "mlp.mlp.2", epilogue="residual", residual=x, gate=gate_mlp)
    return x


class ShardedBlockStack:
    """The block stack over ``P`` ranks, token-sharded; weights replicated on every rank."""

    def __init__(self, weights: list[dict], heads: int, group=None):
        self.weights = weights
        self.heads = heads
        self.group = group
        self._kv = None

    def __call__(self, x_local: torch.Tensor, mod: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 kvs: list[tuple[torch.Tensor, torch.Tensor]]) -> torch.Tensor:
        x = x_local.clone()
        t_local, c = x.shape
        world = dist.get_world_size(self.group)
        shape = (world * t_local, self.heads, c // self.heads)
        if self._kv is None or self._kv[0].shape != shape or self._kv[0].device != x.device:
            self._kv = tuple(torch.empty(shape, dtype=x.dtype, device=x.device) for _ in range(2))
        for i, w in enumerate(self.weights):
            block_forward_sharded(w, x, mod, cos, sin, kvs[i][0], kvs[i][1], self.heads, self.group, self._kv)
        return x
