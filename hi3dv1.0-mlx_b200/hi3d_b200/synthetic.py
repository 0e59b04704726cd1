"""Seeded synthetic inputs with the shapes and distributions of the BASELINE configs.

No checkpoints or datasets exist on the box, so every workload is generated:
voxel coordinates on a noisy spherical shell in a ``G^3`` grid, N(0, 1)
features and condition tokens, N(0, 0.02) weights, and the adaLN modulation
computed from a random timestep embedder (the upstream ``TimestepEmbedder`` /
``adaLN_modulation`` chain, src/sparc3d/models/transformers/sparc3d_transformer.py:29-76).
Everything is numpy on the host so the CPU oracle and the GPU path see
bit-identical inputs.
"""

from __future__ import annotations

import math

import numpy as np


def shell_coords(n: int, grid: int, radius: float, thickness: float, seed: int) -> np.ndarray:
    """``n`` distinct int32 ``(x, y, z)`` voxels on a seeded shell, lexicographically sorted.

    Directions are normalised N(0, 1) vectors, radii U(radius - thickness, radius + thickness);
    ``round(v * r + grid / 2)`` clipped to the grid.  Points are drawn until at least ``n``
    distinct sites exist, then a seeded subset of ``n`` is kept.
    """
    rng = np.random.default_rng(seed)
    seen = np.zeros((0, 3), np.int64)
    draw = max(4 * n, 1024)
    for _ in range(64):
        v = rng.standard_normal((draw, 3))
        v /= np.linalg.norm(v, axis=1, keepdims=True)
        r = rng.uniform(radius - thickness, radius + thickness, (draw, 1))
        p = np.clip(np.rint(v * r + grid / 2), 0, grid - 1).astype(np.int64)
        seen = np.unique(np.concatenate([seen, p]), axis=0)
        if seen.shape[0] >= n:
            break
    if seen.shape[0] < n:
        raise ValueError(f"shell of radius {radius}±{thickness} in {grid}^3 holds fewer than {n} voxels")
    keep = np.sort(rng.choice(seen.shape[0], n, replace=False))
    return seen[keep].astype(np.int32)


def timestep_embedding(t: np.ndarray, dim: int = 256, max_period: int = 10000) -> np.ndarray:
    """Sinusoidal embedding (transformer.py:182-186)."""
    half = dim // 2
    freqs = np.exp(-math.log(max_period) * np.arange(half, dtype=np.float32) / half).astype(np.float32)
    args = t[:, None].astype(np.float32) * freqs[None]
    return np.concatenate([np.cos(args), np.sin(args)], axis=-1).astype(np.float32)


def _silu(x):
    return x / (1.0 + np.exp(-x))


def modulation(channels: int, t: float, seed: int) -> np.ndarray:
    """adaLN ``mod [1, 6C]`` from a random timestep embedder at time ``t`` (model sees 1000 t)."""
    rng = np.random.default_rng(seed)
    w = lambda o, i: rng.normal(0, 0.02, (o, i)).astype(np.float32)
    temb = timestep_embedding(np.array([np.float32(1000.0) * np.float32(t)], np.float32))
    emb = temb @ w(channels, 256).T + rng.normal(0, 0.02, channels).astype(np.float32)
    emb = _silu(emb) @ w(channels, channels).T + rng.normal(0, 0.02, channels).astype(np.float32)
    mod = _silu(emb) @ w(6 * channels, channels).T + rng.normal(0, 0.02, 6 * channels).astype(np.float32)
    return mod.astype(np.float32)


BLOCK_LINEARS = (
    ("self_attn.to_qkv", 1, 3),
    ("self_attn.to_out", 1, 1),
    ("cross_attn.to_q", 1, 1),
    ("cross_attn.to_out", 1, 1),
    ("mlp.mlp.0", 1, 4),
    ("mlp.mlp.2", 4, 1),
)


def block_weights(channels: int, ctx_channels: int, heads: int, seed: int, gamma_random: bool = False) -> dict:
    """Random block parameters named as the reference checkpoint names them.

    Linear weights/biases N(0, 0.02) rounded to fp16 (the released torso dtype);
    ``modulation`` N(0, 1)/sqrt(C) fp32 (modulated.py:43); norm2 affine and the QK
    gains fp32 (ones, or U(0.5, 1.5) with ``gamma_random``).
    """
    rng = np.random.default_rng(seed)
    c, d = channels, channels // heads
    w: dict[str, np.ndarray] = {}
    for name, i_mult, o_mult in BLOCK_LINEARS:
        w[f"{name}.weight"] = rng.normal(0, 0.02, (o_mult * c, i_mult * c)).astype(np.float16)
        w[f"{name}.bias"] = rng.normal(0, 0.02, o_mult * c).astype(np.float16)
    w["cross_attn.to_kv.weight"] = rng.normal(0, 0.02, (2 * c, ctx_channels)).astype(np.float16)
    w["cross_attn.to_kv.bias"] = rng.normal(0, 0.02, 2 * c).astype(np.float16)
    w["modulation"] = (rng.standard_normal((1, 6 * c)) / math.sqrt(c)).astype(np.float32)
    if gamma_random:
        w["norm2.weight"] = rng.uniform(0.5, 1.5, c).astype(np.float32)
        w["norm2.bias"] = rng.normal(0, 0.1, c).astype(np.float32)
        w["self_attn.q_rms_norm.gamma"] = rng.uniform(0.5, 1.5, (heads, d)).astype(np.float32)
        w["self_attn.k_rms_norm.gamma"] = rng.uniform(0.5, 1.5, (heads, d)).astype(np.float32)
    else:
        w["norm2.weight"] = np.ones(c, np.float32)
        w["norm2.bias"] = np.zeros(c, np.float32)
        w["self_attn.q_rms_norm.gamma"] = np.ones((heads, d), np.float32)
        w["self_attn.k_rms_norm.gamma"] = np.ones((heads, d), np.float32)
    return w


def features(rows: int, channels: int, seed: int, dtype=np.float16) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((rows, channels)).astype(np.float32).astype(dtype)


def resblock_shapes(channels: int, out_channels: int, emb_channels: int) -> dict:
    """Parameter shapes of one sparse res block (``SparseResBlock3d``,
    src/sparc3d/models/transformers/sparc3d_transformer.py:80-130): hidden = out // 2."""
    hid = out_channels // 2
    shapes = {
        "norm1.weight": (channels,), "norm1.bias": (channels,),
        "conv1.conv.weight": (hid, 3, 3, 3, channels), "conv1.conv.bias": (hid,),
        "conv2.conv.weight": (hid, 3, 3, 3, hid), "conv2.conv.bias": (hid,),
        "linear.weight": (out_channels, hid), "linear.bias": (out_channels,),
        "emb_layers.1.weight": (2 * hid, emb_channels), "emb_layers.1.bias": (2 * hid,),
    }
    if channels != out_channels:
        shapes.update({"skip_connection.weight": (out_channels, channels), "skip_connection.bias": (out_channels,)})
    return shapes


def model_weights(channels: int, ctx_channels: int, heads: int, num_blocks: int, io_channels: int = 256,
                  in_channels: int = 32, out_channels: int = 32, seed: int = 0, std: float | None = 0.02) -> dict:
    """Random parameters of the whole refinement transformer, named as the upstream state dict
    (``Sparc3DTransformer``, sparc3d_transformer.py:149-230) for one I/O stage of two res blocks.

    Linear and convolution parameters of the fp16 torso (I/O res blocks and blocks) are rounded
    to fp16, as ``convert_to_fp16`` stores them; the timestep embedder, adaLN, input/output
    layers and the norms stay fp32.  ``std`` is the weight standard deviation (BASELINE: 0.02);
    ``None`` scales each weight by 1/sqrt(fan-in) and randomises the norm affines, which keeps
    activations O(1) through the stack for parity tests.
    """
    rng = np.random.default_rng(seed)

    def weight(shape, fan_in):
        s = std if std is not None else 1.0 / math.sqrt(fan_in)
        return rng.normal(0, s, shape).astype(np.float32)

    w: dict[str, np.ndarray] = {}
    c = channels
    for name, (o, i) in (("t_embedder.mlp.0", (c, 256)), ("t_embedder.mlp.2", (c, c)),
                         ("adaLN_modulation.1", (6 * c, c)), ("input_layer", (io_channels, in_channels))):
        w[f"{name}.weight"] = weight((o, i), i)
        w[f"{name}.bias"] = rng.normal(0, 0.02, o).astype(np.float32)
    stages = (("input_blocks.0", io_channels, io_channels), ("input_blocks.1", io_channels, c),
              ("out_blocks.0", 2 * c, io_channels), ("out_blocks.1", 2 * io_channels, io_channels))
    for name, cin, cout in stages:
        for key, shape in resblock_shapes(cin, cout, c).items():
            full = f"{name}.{key}"
            if key == "norm1.weight":
                w[full] = (np.ones(shape, np.float32) if std is not None else
                           rng.uniform(0.5, 1.5, shape).astype(np.float32))
            elif key == "norm1.bias":
                w[full] = (np.zeros(shape, np.float32) if std is not None else
                           rng.normal(0, 0.1, shape).astype(np.float32))
            elif key.endswith("bias"):
                w[full] = rng.normal(0, 0.02, shape).astype(np.float16)
            else:
                w[full] = weight(shape, int(np.prod(shape[1:]))).astype(np.float16)
    for i in range(num_blocks):
        for k, v in block_weights(c, ctx_channels, heads, seed=seed * 1000 + i + 1, gamma_random=std is None).items():
            w[f"blocks.{i}.{k}"] = v
    w["out_layer.weight"] = weight((out_channels, io_channels), io_channels)
    w["out_layer.bias"] = rng.normal(0, 0.02, out_channels).astype(np.float32)
    return w
