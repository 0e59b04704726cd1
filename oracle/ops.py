"""CPU oracle of the Hi3D sparse-DiT block path: numpy restatements of the reference.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use it, and only as the checker (or as the timed CPU baseline), never as the
thing measured on the GPU.

Each function restates the reference algorithm it cites (paths inside the
devin-lai/Hi3Dv1.0-mlx tree).  Where the reference is a Metal kernel that cannot
run here, the restatement follows the kernel source line by line, including
its fp32/fp16 rounding points.  Pinning: ``tests/golden/make_golden.py``
records outputs of the reference's own runnable code (the upstream PyTorch
modules with the reference's torch shims, and the pure-numpy helpers of the
MLX path) into ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks
every function here against those fixtures.  The W8A8 quantizer's rounding
(Metal fast-math division) has no runnable reference: it is pinned only by the
structure tests (Hadamard identity, sign table) and the reference's own
numpy int64 GEMM contract (tests/test_w8a8_inference.py:8-20).
"""

from __future__ import annotations

import itertools
import math

import numpy as np

F16, F32 = np.float16, np.float32

# ----------------------------------------------------------------------------- geometry


# sparse.py:20 -- neighbour displacement r_k - 1 of flat kernel offset k = r0*9 + r1*3 + r2
OFFSETS = np.array(list(itertools.product(range(3), repeat=3)), dtype=np.int64) - 1


def neighbour_table(coords: np.ndarray) -> np.ndarray:
    """``[N, 27]`` int32 neighbour rows, ``N`` where absent (sparse.py:29-43)."""
    coords = np.asarray(coords, dtype=np.int64)
    n = coords.shape[0]
    if n == 0:
        return np.zeros((0, 27), np.int32)
    extent = coords.max(axis=0) + 3
    grid = np.full(tuple(extent), n, dtype=np.int32)
    grid[tuple((coords + 1).T)] = np.arange(n, dtype=np.int32)
    table = np.empty((n, 27), dtype=np.int32)
    for k, d in enumerate(OFFSETS):
        table[:, k] = grid[tuple((coords + 1 + d).T)]
    return table


def downsample_structure(coords: np.ndarray):
    """Unique ``coords // 2`` (lexicographic), inverse, counts (sparse.py:217-233)."""
    half = np.asarray(coords, dtype=np.int64) // 2
    extent = half.max(axis=0) + 1
    codes = (half[:, 0] * extent[1] + half[:, 1]) * extent[2] + half[:, 2]
    unique, inverse, counts = np.unique(codes, return_inverse=True, return_counts=True)
    low = np.stack([unique // (extent[1] * extent[2]), (unique // extent[2]) % extent[1], unique % extent[2]],
                   axis=1).astype(np.int32)
    return low, inverse.astype(np.int32), counts.astype(np.int32)


def subm_conv(x: np.ndarray, table: np.ndarray, weight_t: np.ndarray, bias: np.ndarray | None,
              dtype=np.float64) -> np.ndarray:
    """Submanifold 3x3x3 conv as gathered GEMM (sparse.py:191-214):
    ``out[o] = b + sum_k in[table[o, k]] @ W_k`` with ``weight_t [27*Cin, Cout]``."""
    n, cin = x.shape
    padded = np.concatenate([x.astype(dtype), np.zeros((1, cin), dtype)], 0)
    out = np.zeros((n, weight_t.shape[1]), dtype)
    w = weight_t.astype(dtype).reshape(27, cin, -1)
    for k in range(27):
        out += padded[table[:, k]] @ w[k]
    if bias is not None:
        out += bias.astype(dtype)
    return out


def conv_weight(weight: np.ndarray) -> np.ndarray:
    """spconv ``(out, 3, 3, 3, in)`` -> GEMM layout ``[27 * in, out]`` (sparse.py:185-188)."""
    return weight.reshape(weight.shape[0], -1).T


# ----------------------------------------------------------------------------- VAE decoder


def group_stats_f64(x: np.ndarray, eps: float = 1e-6):
    """PointGroupNorm statistics (vae.py:142-164): groups of ``c / groups`` channels, 32 groups
    (``c // 4`` below 128 channels); mean = S1 / (count + eps), var = S2 / (count + eps) - mean^2,
    inv = 1 / sqrt(var + eps), count = n * width; repeated per channel."""
    n, c = x.shape
    groups = 32 if 4 * 32 <= c else c // 4
    width = c // groups
    xf = x.astype(np.float64)
    s1 = xf.sum(0).reshape(groups, width).sum(1)
    s2 = (xf * xf).sum(0).reshape(groups, width).sum(1)
    count = n * width + eps
    mean = s1 / count
    inv = 1.0 / np.sqrt(s2 / count - mean * mean + eps)
    return np.repeat(mean, width), np.repeat(inv, width)


def group_norm_swish(x: np.ndarray, mean, inv, w, b) -> np.ndarray:
    """``u * sigmoid(u)``, ``u = (x - mean) * inv * w + b`` in float64 (kernels.py:242-260)."""
    u = (x.astype(np.float64) - mean) * inv * w + b
    return u / (1.0 + np.exp(-u))


def child_offset_tables():
    """Parent-neighbourhood offset and child slot of every (slot, offset) (sparse.py:46-58)."""
    pk = np.zeros((8, 27), np.int32)
    ss = np.zeros((8, 27), np.int32)
    for s in range(8):
        bits = np.array([(s >> 2) & 1, (s >> 1) & 1, s & 1])
        for k, d in enumerate(OFFSETS):
            t = bits + d
            pd, cb = t >> 1, t & 1
            pk[s, k] = (pd[0] + 1) * 9 + (pd[1] + 1) * 3 + (pd[2] + 1)
            ss[s, k] = cb[0] * 4 + cb[1] * 2 + cb[2]
    return pk, ss


def child_neighbour_table(parent_table: np.ndarray, child_mask: np.ndarray):
    """Children of an octree upsampling and their neighbour table (sparse.py:64-95)."""
    pk, ss = child_offset_tables()
    p = child_mask.shape[0]
    ids = np.flatnonzero(child_mask.reshape(-1))
    nc = ids.size
    lookup = np.full(p * 8 + 8, nc, np.int64)
    lookup[ids] = np.arange(nc)
    parent, slot = ids // 8, ids % 8
    rows = parent_table[parent]
    nbp = np.take_along_axis(rows, pk[slot], axis=1).astype(np.int64)
    table = lookup[nbp * 8 + ss[slot]]
    return table.astype(np.int32), parent.astype(np.int32), slot.astype(np.int32)


def morton(coords: np.ndarray, depth: int) -> np.ndarray:
    """Interleaved keys, x highest (vae.py:49-55)."""
    x, y, z = (coords[:, i].astype(np.int64) for i in range(3))
    key = np.zeros_like(x)
    for i in range(depth):
        key |= ((x >> i) & 1) << (3 * i + 2) | ((y >> i) & 1) << (3 * i + 1) | ((z >> i) & 1) << (3 * i)
    return key


def serialization(coords: np.ndarray):
    """``[(perm, inverse)]`` for the orders z and z-trans (vae.py:58-69)."""
    depth = int(coords.max()).bit_length()
    out = []
    for order in ("z", "z-trans"):
        c = coords if order == "z" else coords[:, [1, 0, 2]]
        perm = np.argsort(morton(c, depth), kind="stable")
        inverse = np.empty_like(perm)
        inverse[perm] = np.arange(perm.shape[0])
        out.append((perm.astype(np.int32), inverse.astype(np.int32)))
    return out


def window_index(perm: np.ndarray, patch: int = 48) -> np.ndarray:
    """Rows in padded window order (vae.py:72-88)."""
    n = perm.shape[0]
    if n <= patch:
        return perm
    n_pad = -(-n // patch) * patch
    pad = np.arange(n_pad)
    rem = n % patch
    if rem:
        pad[n_pad - patch + rem:] = pad[n_pad - 2 * patch + rem:n_pad - patch]
    return perm[pad]


def window_attention_f64(qkv: np.ndarray, gather: np.ndarray, inverse: np.ndarray, heads: int,
                         patch: int = 48) -> np.ndarray:
    """Attention within windows of ``patch`` rows of ``qkv [n, 3, heads, D]`` taken in ``gather``
    order, scattered back by ``inverse`` (vae.py:249-266), float64."""
    n = qkv.shape[0]
    length = patch if gather.shape[0] >= patch else gather.shape[0]
    d = qkv.shape[1] // 3 // heads
    g = qkv.astype(np.float64)[gather].reshape(-1, length, 3, heads, d)
    q, k, v = (g[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    s = q @ k.transpose(0, 1, 3, 2) * d ** -0.5
    p = np.exp(s - s.max(-1, keepdims=True))
    o = (p / p.sum(-1, keepdims=True)) @ v
    o = o.transpose(0, 2, 1, 3).reshape(-1, heads * d)
    return o[inverse]


# ----------------------------------------------------------------------------- rope


def rope_tables(coords: np.ndarray, head_dim: int = 96):
    """cos/sin ``[N, head_dim/2]`` fp32 (transformer.py:189-210; upstream rope.py:38-58,82-90)."""
    freq_dim = head_dim // 3 // 2
    freqs = 1.0 / (10000.0 ** (np.arange(freq_dim, dtype=np.float32) / np.float32(freq_dim)))
    freqs = freqs.astype(np.float32)
    max_length = int(coords.max())
    if max_length >= 64:
        train, infer = 64, (64 + max_length) // 2
        wavelengths = freqs * train / (2 * math.pi)
        ratio = (wavelengths - 1) / (24 - 1)
        ratio = ratio + (1 - ratio) * train / infer
        ratio = np.where(wavelengths > 24, 1.0, ratio)
        ratio = np.where(wavelengths < 1, train / infer, ratio)
        freqs = (freqs * ratio).astype(np.float32)
    phases = coords.astype(np.float32).reshape(-1)[:, None] * freqs[None, :]
    phases = phases.reshape(coords.shape[0], 3 * freq_dim)
    pad = head_dim // 2 - phases.shape[1]
    cos, sin = np.cos(phases), np.sin(phases)
    if pad > 0:
        cos = np.concatenate([cos, np.ones((cos.shape[0], pad), np.float32)], 1)
        sin = np.concatenate([sin, np.zeros((sin.shape[0], pad), np.float32)], 1)
    return cos.astype(np.float32), sin.astype(np.float32)


def qkv_rope_rms(qkv: np.ndarray, cos: np.ndarray, sin: np.ndarray, gq: np.ndarray, gk: np.ndarray, batch: int,
                 heads: int, head_dim: int):
    """RoPE + QK RMS norm + split to ``[B, H, N, D]`` in fp32 math (kernels.py:22-57).

    Returns q, k, v in ``qkv``'s dtype; v is the bit-exact copy."""
    m = qkv.shape[0]
    n = m // batch
    d2 = head_dim // 2
    x = qkv.reshape(batch, n, 3, heads, d2, 2).astype(np.float32)
    c = cos.astype(np.float32)[None, :, None, :]
    s = sin.astype(np.float32)[None, :, None, :]
    outs = []
    for part, g in ((0, gq), (1, gk)):
        x0, x1 = x[:, :, part, ..., 0], x[:, :, part, ..., 1]
        re = x0 * c - x1 * s
        im = x0 * s + x1 * c
        ss = (re * re + im * im).sum(-1, keepdims=True, dtype=np.float32)
        nrm = np.maximum(np.sqrt(ss), np.float32(1e-12))
        scale = np.float32(math.sqrt(head_dim))
        gg = g.astype(np.float32).reshape(heads, d2, 2)
        y = np.stack([re / nrm * gg[..., 0] * scale, im / nrm * gg[..., 1] * scale], -1)
        outs.append(y.reshape(batch, n, heads, head_dim).transpose(0, 2, 1, 3).astype(qkv.dtype))
    v = qkv.reshape(batch, n, 3, heads, head_dim)[:, :, 2].transpose(0, 2, 1, 3).copy()
    return outs[0], outs[1], v


def qkv_rope_rms_f64(qkv: np.ndarray, cos, sin, gq, gk, batch, heads, head_dim):
    """Float64 complex-rotation oracle of the same op (tests/test_fast.py:25-31)."""
    b, n = batch, qkv.shape[0] // batch
    x = qkv.astype(np.float64).reshape(b, n, 3, heads, head_dim // 2, 2)
    c, s = cos.astype(np.float64), sin.astype(np.float64)
    outs = []
    for part, g in ((0, gq), (1, gk)):
        z = (x[:, :, part, ..., 0] + 1j * x[:, :, part, ..., 1]) * (c + 1j * s)[None, :, None, :]
        y = np.stack((z.real, z.imag), -1).reshape(b, n, heads, head_dim)
        y = y / np.linalg.norm(y, axis=-1, keepdims=True) * g.astype(np.float64) * np.sqrt(head_dim)
        outs.append(y.transpose(0, 2, 1, 3))
    return outs[0], outs[1]


# ----------------------------------------------------------------------------- norms / elementwise


def layer_norm_modulate(x: np.ndarray, eps: float, weight=None, bias=None, scale=None, shift=None) -> np.ndarray:
    """LayerNorm32 (+fp32 affine) (+adaLN modulation, two fp16 roundings) of fp16 rows.

    kernels.py:162-201: mean = sum/C; var = sum((x-mean)^2)/C (two pass, fp32);
    inv = 1/sqrt(var + eps); y = (x-mean)*inv; y = y*w + b; h = half(y);
    h = half(float(h)*float(scale)); h = half(float(h)+float(shift))."""
    dt = x.dtype
    xf = x.astype(np.float32)
    c = np.float32(x.shape[-1])
    mean = xf.sum(-1, keepdims=True, dtype=np.float32) / c
    d = xf - mean
    var = (d * d).sum(-1, keepdims=True, dtype=np.float32) / c
    inv = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    y = d * inv
    if weight is not None:
        y = y * weight.astype(np.float32) + bias.astype(np.float32)
    h = y.astype(dt)
    if scale is not None:
        h = (h.astype(np.float32) * scale.astype(np.float32)).astype(dt)
        h = (h.astype(np.float32) + shift.astype(np.float32)).astype(dt)
    return h


def layer_norm32_f32(x: np.ndarray, weight=None, bias=None, eps: float = 1e-6) -> np.ndarray:
    """Upstream LayerNorm32 in fp32 (norm.py:12-17)."""
    xf = x.astype(np.float32)
    mean = xf.mean(-1, keepdims=True)
    var = ((xf - mean) ** 2).mean(-1, keepdims=True)
    y = (xf - mean) / np.sqrt(var + np.float32(eps))
    if weight is not None:
        y = y * weight + bias
    return y.astype(np.float32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """tanh GELU in fp32, rounded to x's dtype (transformer.py:176-179)."""
    xf = x.astype(np.float32)
    y = 0.5 * xf * (1.0 + np.tanh(np.float32(math.sqrt(2.0 / math.pi)) * (xf + np.float32(0.044715) * xf * xf * xf)))
    return y.astype(x.dtype)


def gate_residual(x: np.ndarray, y: np.ndarray, gate: np.ndarray | None) -> np.ndarray:
    """``x + y * gate`` in x's dtype with two roundings (transformer.py:570,588)."""
    dt = x.dtype
    yy = y.astype(np.float32)
    if gate is not None:
        yy = (yy * gate.astype(np.float32)).astype(dt).astype(np.float32)
    return (x.astype(np.float32) + yy).astype(dt)


# ----------------------------------------------------------------------------- attention


def attention_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """Exact attention in float64, ``[B, H, Nq, D]`` x ``[B|1, H, Nk, D]`` -> ``[B, Nq, H*D]``
    (tests/test_mlx_kernels.py:153-160)."""
    qf, kf, vf = (np.asarray(t, np.float64) for t in (q, k, v))
    kf = np.broadcast_to(kf, (qf.shape[0],) + kf.shape[1:])
    vf = np.broadcast_to(vf, (qf.shape[0],) + vf.shape[1:])
    out = np.empty((qf.shape[0], qf.shape[1], qf.shape[2], qf.shape[3]))
    for b in range(qf.shape[0]):
        for h in range(qf.shape[1]):
            s = qf[b, h] @ kf[b, h].T * scale
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            out[b, h] = p @ vf[b, h]
    return out.transpose(0, 2, 1, 3).reshape(qf.shape[0], qf.shape[2], -1)


def attention_varlen(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_q, cu_k, scale: float,
                     dtype=np.float64) -> np.ndarray:
    """Packed varlen attention ``q [Tq, H, D]``, ``k, v [Tk, H, D]`` per sequence
    (torch_backend/attention.py:174-206); ``cu_k=None`` shares all keys."""
    out = np.zeros(q.shape, dtype)
    for i in range(len(cu_q) - 1):
        qs = slice(int(cu_q[i]), int(cu_q[i + 1]))
        ks = slice(0, k.shape[0]) if cu_k is None else slice(int(cu_k[i]), int(cu_k[i + 1]))
        if qs.stop <= qs.start:
            continue
        qq, kk, vv = (np.asarray(t[sl], dtype) for t, sl in ((q, qs), (k, ks), (v, ks)))
        for h in range(q.shape[1]):
            s = qq[:, h] @ kk[:, h].T * scale
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            out[qs, h] = p @ vv[:, h]
    return out


# ----------------------------------------------------------------------------- W8A8


def signs(width: int) -> np.ndarray:
    """Per-column sign vector of the signed H64 rotation (w8a8.py:16-18)."""
    return np.random.default_rng(314159 + width).choice([-1.0, 1.0], width).astype(np.float32)


def _h64_butterfly(x: np.ndarray, sign: np.ndarray) -> np.ndarray:
    """Signed 64-point Walsh-Hadamard / 8 per 64-block, in the fp32 operation order of the
    reference quantizer (w8a8.py:25-45): five xor-butterflies over the lane pair (c, c+32),
    then lo = (u+v)/8 at c, hi = (u-v)/8 at c+32."""
    rows, k = x.shape
    xb = (x.astype(np.float32) * sign.astype(np.float32)).reshape(rows, k // 64, 2, 32)
    u, v = xb[:, :, 0, :], xb[:, :, 1, :]
    lane = np.arange(32)
    for d in (1, 2, 4, 8, 16):
        au, av = u[..., lane ^ d], v[..., lane ^ d]
        bit = (lane & d) != 0
        u = np.where(bit, au - u, u + au).astype(np.float32)
        v = np.where(bit, av - v, v + av).astype(np.float32)
    lo = (u + v) * np.float32(0.125)
    hi = (u - v) * np.float32(0.125)
    return np.stack([lo, hi], 2).reshape(rows, k).astype(np.float32)


def quantize_activation(x: np.ndarray, multiplier: np.ndarray | None = None):
    """Per-row dynamic int8 with signed H64 rotation (w8a8.py:25-58, :95-102).

    s = max(max|y|, 1e-8) / 127 (fp32); q = clamp(rint(y / s), -127, 127), round half even."""
    k = x.shape[-1]
    if k % 64:
        raise ValueError("signed H64 requires width divisible by 64")
    x = x.reshape(-1, k)
    y = _h64_butterfly(x, signs(k) if multiplier is None else multiplier)
    s = (np.maximum(np.abs(y).max(-1), np.float32(1e-8)) / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(y / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def quantize_weight(w: np.ndarray, rotate: bool = True):
    """Symmetric per-output-row int8 weights (models/w8a8/manifest.json:14-15):
    optionally in the signed-H64 domain of the activations, sw = max|w_row| / 127,
    q = rint(w / sw) (round half even)."""
    wf = w.astype(np.float32)
    if rotate:
        wf = _h64_butterfly(wf, signs(w.shape[1]))
    sw = (np.maximum(np.abs(wf).max(-1), np.float32(1e-8)) / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(wf / sw[:, None]), -127, 127).astype(np.int8)
    return q, sw


def w8a8_accumulate(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators ``a @ w.T`` (tests/test_w8a8_inference.py:15)."""
    return (a.astype(np.int64) @ w.astype(np.int64).T).astype(np.int32)


def w8a8_linear_expected(a, sa, w, sw, bias) -> np.ndarray:
    """``acc * sa * sw + bias`` in fp32 (tests/test_w8a8_inference.py:15-16; epilogue w8a8.py:77)."""
    acc = w8a8_accumulate(a, w)
    return acc.astype(np.float32) * sa[:, None] * sw[None, :] + bias.astype(np.float32)


# ----------------------------------------------------------------------------- block (fp32)


def block_forward_f32(w: dict, x: np.ndarray, mod: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                      ctx: np.ndarray, heads: int, seqlens: list[int] | None = None) -> np.ndarray:
    """``ModulatedSparseTransformerCrossBlock.forward`` in fp32
    (src/sparc3d/nn/sparse/transformer/modulated.py:45-65; MLX form transformer.py:543-588).

    x ``[T, C]`` (objects packed by ``seqlens``), mod ``[1, 6C]``, cos/sin ``[T, D/2]``,
    ctx ``[L, Cc]`` (one condition shared by all objects), weights as the reference names them.
    """
    f = np.float32
    x = x.astype(f)
    t, c = x.shape
    d = c // heads
    seqlens = seqlens or [t]
    cu = np.concatenate([[0], np.cumsum(seqlens)])
    parts = (w["modulation"].astype(f) + mod.astype(f)).reshape(6, c)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = parts

    def lin(h, name):
        return h @ w[f"{name}.weight"].astype(f).T + w[f"{name}.bias"].astype(f)

    h = layer_norm32_f32(x) * (1 + scale_msa) + shift_msa
    qkv = lin(h, "self_attn.to_qkv").reshape(t, 3, heads, d // 2, 2)
    cc, ss = cos[:, None, :], sin[:, None, :]
    qk = []
    for part, g in ((0, "self_attn.q_rms_norm.gamma"), (1, "self_attn.k_rms_norm.gamma")):
        re = qkv[:, part, ..., 0] * cc - qkv[:, part, ..., 1] * ss
        im = qkv[:, part, ..., 0] * ss + qkv[:, part, ..., 1] * cc
        y = np.stack([re, im], -1).reshape(t, heads, d)
        y = y / np.maximum(np.linalg.norm(y, axis=-1, keepdims=True), 1e-12) * w[g].astype(f) * f(math.sqrt(d))
        qk.append(y.astype(f))
    v = qkv[:, 2].reshape(t, heads, d)
    a = attention_varlen(qk[0], qk[1], v, cu, cu, d ** -0.5, dtype=np.float32).reshape(t, c)
    x = x + lin(a, "self_attn.to_out") * gate_msa
    h = layer_norm32_f32(x, w["norm2.weight"].astype(f), w["norm2.bias"].astype(f))
    q = lin(h, "cross_attn.to_q").reshape(t, heads, d)
    kv = lin(ctx.astype(f), "cross_attn.to_kv").reshape(-1, 2, heads, d)
    o = attention_varlen(q, kv[:, 0], kv[:, 1], cu, None, d ** -0.5, dtype=np.float32).reshape(t, c)
    x = x + lin(o, "cross_attn.to_out")
    h = layer_norm32_f32(x) * (1 + scale_mlp) + shift_mlp
    h = lin(h, "mlp.mlp.0")
    h = 0.5 * h * (1.0 + np.tanh(f(math.sqrt(2.0 / math.pi)) * (h + f(0.044715) * h * h * h)))
    return (x + lin(h, "mlp.mlp.2") * gate_mlp).astype(f)


# ----------------------------------------------------------------------------- full transformer (fp32)


def silu_f32(x: np.ndarray) -> np.ndarray:
    """``x * sigmoid(x)`` (transformer.py:172-173)."""
    x = x.astype(F32)
    return (x / (F32(1) + np.exp(-x))).astype(F32)


def timestep_embedding_f32(t: np.ndarray, dim: int = 256, max_period: int = 10000) -> np.ndarray:
    """Sinusoidal embedding ``[cos, sin]`` (transformer.py:182-186)."""
    half = dim // 2
    freqs = np.exp(-math.log(max_period) * np.arange(half, dtype=F32) / half).astype(F32)
    args = t[:, None].astype(F32) * freqs[None]
    return np.concatenate([np.cos(args), np.sin(args)], axis=-1).astype(F32)


def downsample_mean_f32(x: np.ndarray, inverse: np.ndarray, counts: np.ndarray) -> np.ndarray:
    """Geometry.downsample (transformer.py:261-263): scatter-add of the children from a zero row,
    divided by ``counts + 1`` (transformer.py:249-251)."""
    sums = np.zeros((counts.shape[0], x.shape[1]), F32)
    np.add.at(sums, inverse, x.astype(F32))
    return (sums / (counts.astype(F32) + 1)[:, None]).astype(F32)


def up_conv_f32(h_low: np.ndarray, weight: np.ndarray, bias: np.ndarray, fine_table: np.ndarray,
                inverse: np.ndarray) -> np.ndarray:
    """Sparc3DTransformerMLX._up_conv (transformer.py:449-475) with the gather table of
    Geometry.__post_init__ (transformer.py:253-259): every low voxel projected through the 27
    taps, then each fine voxel sums the projections of its neighbours' parents."""
    n_low, cin = h_low.shape
    cout = weight.shape[0]
    w_taps = weight.astype(F32).reshape(cout, 27, cin).transpose(2, 1, 0).reshape(cin, 27 * cout)
    proj = (h_low.astype(F32) @ w_taps).reshape(-1, cout)
    proj = np.concatenate([proj, np.zeros((1, cout), F32)], 0)
    parent_of = np.append(inverse, n_low).astype(np.int64)
    nb_parent = parent_of[fine_table]
    flat = nb_parent * 27 + np.arange(27)[None, :]
    flat[nb_parent == n_low] = n_low * 27
    return (proj[flat].sum(axis=1) + bias.astype(F32)).astype(F32)


def _lin(w: dict, name: str, x: np.ndarray) -> np.ndarray:
    return (x.astype(F32) @ w[f"{name}.weight"].astype(F32).T + w[f"{name}.bias"].astype(F32)).astype(F32)


def _conv(w: dict, name: str, x: np.ndarray, table: np.ndarray) -> np.ndarray:
    out = subm_conv(x, table, conv_weight(w[f"{name}.conv.weight"]), w[f"{name}.conv.bias"], dtype=np.float64)
    return out.astype(F32)


def _emb_scale_shift(w: dict, name: str, emb: np.ndarray):
    """transformer.py:413-416"""
    y = _lin(w, f"{name}.emb_layers.1", silu_f32(emb))
    return np.split(y, 2, axis=1)


def _resblock_tail(w: dict, name: str, h: np.ndarray, table: np.ndarray, scale, shift) -> np.ndarray:
    """norm2 -> modulate -> SiLU -> conv2 -> SiLU -> linear (transformer.py:418-424)."""
    h = layer_norm32_f32(h) * (1 + scale) + shift
    h = _conv(w, f"{name}.conv2", silu_f32(h), table)
    return _lin(w, f"{name}.linear", silu_f32(h))


def resblock_f32(w: dict, name: str, x: np.ndarray, emb: np.ndarray, table: np.ndarray) -> np.ndarray:
    """A res block without resampling (transformer.py:426-437)."""
    scale, shift = _emb_scale_shift(w, name, emb)
    h = silu_f32(layer_norm32_f32(x, w[f"{name}.norm1.weight"].astype(F32), w[f"{name}.norm1.bias"].astype(F32)))
    h = _resblock_tail(w, name, _conv(w, f"{name}.conv1", h, table), table, scale, shift)
    skip = _lin(w, f"{name}.skip_connection", x) if f"{name}.skip_connection.weight" in w else x.astype(F32)
    return (h + skip).astype(F32)


def forward_f32(w: dict, feats: np.ndarray, coords: np.ndarray, t: float, cond: np.ndarray | None,
                heads: int) -> np.ndarray:
    """Velocity of Sparc3DTransformerMLX.__call__ for one conditioned branch, in fp32
    (transformer.py:606-668; upstream Sparc3DTransformer.forward,
    src/sparc3d/models/transformers/sparc3d_transformer.py:252-290).

    ``w``: parameters named as the upstream state dict; ``feats [N, in]`` on fine ``coords [N, 3]``;
    the network sees ``1000 t``; ``cond [L, Cc]``.  One I/O stage (patch size 2, two res blocks
    per stage), as the reference's ``input_stage``/``output_stage`` hard-code.
    """
    coords = np.asarray(coords, np.int32)
    full_table = neighbour_table(coords)
    low, inverse, counts = downsample_structure(coords)
    low_table = neighbour_table(low)
    # embed (transformer.py:606-617)
    temb = timestep_embedding_f32(np.array([F32(1000.0) * F32(t)], F32))
    emb = _lin(w, "t_embedder.mlp.2", silu_f32(_lin(w, "t_embedder.mlp.0", temb)))
    mod = _lin(w, "adaLN_modulation.1", silu_f32(emb))
    # input stage (transformer.py:619-625, :439-447)
    h = _lin(w, "input_layer", feats)
    h = resblock_f32(w, "input_blocks.0", h, emb, full_table)
    skip0 = h
    name = "input_blocks.1"
    scale, shift = _emb_scale_shift(w, name, emb)
    xd = downsample_mean_f32(h, inverse, counts)
    hd = silu_f32(layer_norm32_f32(xd, w[f"{name}.norm1.weight"].astype(F32), w[f"{name}.norm1.bias"].astype(F32)))
    hd = _resblock_tail(w, name, _conv(w, f"{name}.conv1", hd, low_table), low_table, scale, shift)
    h = hd + _lin(w, f"{name}.skip_connection", xd)
    skip_low = h
    # torso (transformer.py:656-667)
    c = h.shape[1]
    cos, sin = rope_tables(low, c // heads)
    for i in sorted({int(k.split(".")[1]) for k in w if k.startswith("blocks.")}):
        bw = {k[len(f"blocks.{i}."):]: v for k, v in w.items() if k.startswith(f"blocks.{i}.")}
        h = block_forward_f32(bw, h, mod, cos, sin, cond, heads)
    # output stage (transformer.py:627-634, :477-485)
    name = "out_blocks.0"
    xl = np.concatenate([h, skip_low], axis=1)
    scale, shift = _emb_scale_shift(w, name, emb)
    hl = silu_f32(layer_norm32_f32(xl, w[f"{name}.norm1.weight"].astype(F32), w[f"{name}.norm1.bias"].astype(F32)))
    hf = up_conv_f32(hl, w[f"{name}.conv1.conv.weight"], w[f"{name}.conv1.conv.bias"], full_table, inverse)
    hf = _resblock_tail(w, name, hf, full_table, scale, shift)
    h = hf + _lin(w, f"{name}.skip_connection", xl)[inverse]
    h = resblock_f32(w, "out_blocks.1", np.concatenate([h, skip0], axis=1), emb, full_table)
    xf = h.astype(F32)
    mean = xf.mean(-1, keepdims=True)
    var = ((xf - mean) ** 2).mean(-1, keepdims=True)
    h = (xf - mean) / np.sqrt(var + F32(1e-5))
    return _lin(w, "out_layer", h)


def guidance_scale_f32(t) -> float:
    """Zero-condition guidance scale in float32 (pipeline.py:75-82)."""
    t32 = F32(t)
    if t32 >= 1.0:
        return 4.0
    if t32 >= 0.7:
        return float(F32(10.0) * (t32 * t32))
    return 1.0


def sample_f32(w: dict, noise: np.ndarray, coords: np.ndarray, cond: np.ndarray, heads: int,
               sigmas: np.ndarray, sigma_hats: np.ndarray, scheduler: str = "heun") -> np.ndarray:
    """Hi3DPipelineMLX.sample (pipeline.py:156-229) on the fp32 forward: guided velocity
    ``neg + s (pos - neg)`` with the all-zero condition as the negative branch (its cross-attention
    reduces to the value bias, as the reference's negative branch computes directly), then Heun
    (predictor at the next sigma, averaged slopes) or Euler updates."""
    zeros = np.zeros_like(cond)

    def velocity(x, t):
        pos = forward_f32(w, x, coords, float(t), cond, heads)
        if F32(t) < 0.7:
            return pos
        neg = forward_f32(w, x, coords, float(t), zeros, heads)
        return (neg + F32(guidance_scale_f32(t)) * (pos - neg)).astype(F32)

    x = noise.astype(F32)
    for i in range(sigma_hats.shape[0]):
        t, t_next = F32(sigma_hats[i]), F32(sigmas[i + 1])
        dt = F32(t - t_next)
        v1 = velocity(x, t)
        if scheduler == "heun":
            v2 = velocity((x - dt * v1).astype(F32), t_next)
            x = (x - dt * (F32(0.5) * (v1 + v2))).astype(F32)
        else:
            x = (x - dt * v1).astype(F32)
    return x
