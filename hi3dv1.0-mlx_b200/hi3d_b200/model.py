"""The whole refinement transformer on B200: timestep embedding, I/O res blocks, block stack.

Mirrors ``Sparc3DTransformerMLX`` (src/hi3d_mac/mlx_backend/transformer.py:235-266, :413-485,
:606-668), itself the upstream ``Sparc3DTransformer`` (src/sparc3d/models/transformers/
sparc3d_transformer.py:149-290) restructured for inference:

* ``embed(t)``: sinusoidal embedding of ``1000 t`` -> ``t_embedder`` MLP -> ``adaLN_modulation``
  (fp32, once per timestep and cached, as the reference caches it);
* ``input_stage``: ``input_layer`` (fp32) -> res block at the fine level -> downsampling res block
  (mean of each low voxel's children, divisor ``children + 1``);
* the block stack at the low level (:class:`hi3d_b200.transformer.BlockStack`);
* ``output_stage``: concatenation with the low skip -> upsampling res block whose first
  convolution is computed from the low level (one GEMM through all 27 taps, then a gather-sum per
  fine voxel) -> concatenation with the fine skip -> res block -> LayerNorm (eps 1e-5, fp32) ->
  ``out_layer`` (fp32).

The sparse convolutions, norms (with the SiLU fused), fp16 projections, resampling and the whole
stack run on this library's sm_100a kernels.  The fp32 parts the reference keeps in fp32 -- the
timestep MLP and adaLN (one row per timestep), ``input_layer`` (32 input channels) and the output
LayerNorm + ``out_layer`` (32 output channels) -- are plain fp32 GEMMs on cuBLAS through torch.
One I/O stage of two res blocks (patch size 2), the released configuration, which the
reference's ``input_stage``/``output_stage`` hard-code.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from . import kernels, sparse, transformer
from . import linear as _linear


@dataclass(frozen=True)
class ModelConfig:
    """The dimensions of ``Sparc3DTransformerConfig`` (src/sparc3d/models/transformers/config.py:92-125)
    that the inference model needs."""

    model_channels: int = 2112
    cond_channels: int = 2048
    num_heads: int = 22
    num_blocks: int = 24
    io_channels: int = 256
    in_channels: int = 32
    out_channels: int = 32

    @property
    def head_dim(self) -> int:
        return self.model_channels // self.num_heads


class Geometry:
    """Index structures of one sampling pass (transformer.py:235-266): the fine level and its
    neighbour table, the downsampled level (children lists for the mean, parent of each fine row)
    and its neighbour table, and the RoPE tables of the low coordinates.  Built once per pass;
    synchronises once (the downsampling validates the coordinates)."""

    def __init__(self, coords, head_dim: int, device=None):
        c = sparse._coords_dev(coords, device)
        self.device = c.device
        self.full = sparse.Level(c, sparse.neighbour_table(c))
        low, inverse, counts, children, offsets = sparse.downsample_groups(c)
        self.low = sparse.Level(low, sparse.neighbour_table(low))
        self.inverse, self.counts, self.children, self.offsets = inverse, counts, children, offsets
        cos, sin = transformer.rope_tables(low.cpu().numpy(), head_dim)
        self.rope_cos = torch.from_numpy(cos).to(self.device)
        self.rope_sin = torch.from_numpy(sin).to(self.device)

    def downsample(self, x: torch.Tensor) -> torch.Tensor:
        return sparse.downsample_mean(x, self.children, self.offsets)

    def upsample(self, x: torch.Tensor) -> torch.Tensor:
        return sparse.upsample(x, self.inverse)


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: int = 10000) -> torch.Tensor:
    """Sinusoidal embedding ``[cos, sin]`` (transformer.py:182-186), fp32."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t[:, None].float() * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


class Sparc3DTransformer:
    """Inference-only sparse flow transformer on one GPU (transformer.py:272-668).

    ``weights`` maps upstream state-dict names to arrays/tensors (``synthetic.model_weights``
    produces them); fp16 torso parameters are used in ``dtype``, fp32 ones stay fp32.
    """

    def __init__(self, config: ModelConfig, weights: dict, device=None, dtype: torch.dtype = torch.float16):
        self.config = config
        self.dt = dtype
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.p = transformer.to_device({k: v for k, v in weights.items() if not k.startswith("blocks.")}, self.device,
                                       dtype)
        blocks = []
        for i in range(config.num_blocks):
            pre = f"blocks.{i}."
            blocks.append(transformer.to_device({k[len(pre):]: v for k, v in weights.items() if k.startswith(pre)},
                                                self.device, dtype))
        self.stack = transformer.BlockStack(blocks, config.num_heads)
        self._embed_cache: dict[bytes, tuple[torch.Tensor, torch.Tensor]] = {}

    # -- helpers ------------------------------------------------------------------------

    def _f32_linear(self, x: torch.Tensor, name: str) -> torch.Tensor:
        return F.linear(x.float(), self.p[f"{name}.weight"].float(), self.p[f"{name}.bias"].float())

    def _linear(self, x: torch.Tensor, name: str, **kw) -> torch.Tensor:
        return _linear.linear(x, self.p[f"{name}.weight"], self.p[f"{name}.bias"], **kw)

    def _conv(self, x: torch.Tensor, level: sparse.Level, name: str, act: str | None = None) -> torch.Tensor:
        return sparse.conv(x, level.table, self.p[f"{name}.conv.weight"], self.p[f"{name}.conv.bias"], n_in=level.n,
                           tap_mask=level.tap_mask, act=act)

    def _norm1(self, x: torch.Tensor, name: str) -> torch.Tensor:
        """``silu(LayerNorm32(x; norm1))`` (transformer.py:428-429)."""
        return kernels.layer_norm_modulate(x, 1e-6, weight=self.p[f"{name}.norm1.weight"],
                                           bias=self.p[f"{name}.norm1.bias"], act="silu")

    # -- building blocks (transformer.py:413-485) ----------------------------------------

    def _emb_scale_shift(self, emb: torch.Tensor, name: str) -> tuple[torch.Tensor, torch.Tensor]:
        """``emb_layers(silu(emb))`` split into scale, shift (transformer.py:413-416)."""
        y = self._linear(F.silu(emb), f"{name}.emb_layers.1")
        scale, shift = y.chunk(2, dim=1)
        return scale.contiguous(), shift.contiguous()

    def _resblock_tail(self, h: torch.Tensor, name: str, level: sparse.Level, scale, shift,
                       skip: torch.Tensor) -> torch.Tensor:
        """``norm2 -> modulate -> SiLU -> conv2 -> SiLU -> linear`` (transformer.py:418-424), the
        final projection adding into ``skip`` in its epilogue (updated in place and returned)."""
        h = kernels.layer_norm_modulate(h, 1e-6, scale=(1 + scale).to(self.dt), shift=shift, act="silu")
        h = self._conv(h, level, f"{name}.conv2", act="silu")
        return self._linear(h, f"{name}.linear", epilogue="residual", residual=skip)

    def _skip(self, x: torch.Tensor, name: str) -> torch.Tensor:
        if f"{name}.skip_connection.weight" in self.p:
            return self._linear(x, f"{name}.skip_connection")
        return x.clone()

    def _resblock(self, x: torch.Tensor, emb: torch.Tensor, name: str, level: sparse.Level) -> torch.Tensor:
        """A res block without resampling (transformer.py:426-437)."""
        scale, shift = self._emb_scale_shift(emb, name)
        h = self._conv(self._norm1(x, name), level, f"{name}.conv1")
        return self._resblock_tail(h, name, level, scale, shift, self._skip(x, name))

    def _down_block(self, x: torch.Tensor, emb: torch.Tensor, geo: Geometry) -> torch.Tensor:
        """The downsampling res block (transformer.py:439-447)."""
        name = "input_blocks.1"
        scale, shift = self._emb_scale_shift(emb, name)
        x = geo.downsample(x)
        h = self._conv(self._norm1(x, name), geo.low, f"{name}.conv1")
        return self._resblock_tail(h, name, geo.low, scale, shift, self._skip(x, name))

    def _up_block(self, x_low: torch.Tensor, emb: torch.Tensor, geo: Geometry) -> torch.Tensor:
        """The upsampling res block (transformer.py:477-485): norm1 at the low level (row-wise,
        so it commutes with the upsampling), the first convolution from the low level."""
        name = "out_blocks.0"
        scale, shift = self._emb_scale_shift(emb, name)
        h = self._norm1(x_low, name)
        h = sparse.up_conv(h, geo.full.table, geo.inverse, self.p[f"{name}.conv1.conv.weight"],
                           self.p[f"{name}.conv1.conv.bias"])
        skip = geo.upsample(self._linear(x_low, f"{name}.skip_connection"))
        return self._resblock_tail(h, name, geo.full, scale, shift, skip)

    # -- forward (transformer.py:606-668) -------------------------------------------------

    def embed(self, t: float) -> tuple[torch.Tensor, torch.Tensor]:
        """Timestep embedding ``emb [1, C]`` and the shared adaLN ``mod [1, 6C]`` (fp32), cached per
        timestep (transformer.py:606-617)."""
        key = np.float32(t).tobytes()
        if key not in self._embed_cache:
            tt = torch.tensor([np.float32(1000.0) * np.float32(t)], dtype=torch.float32, device=self.device)
            emb = self._f32_linear(timestep_embedding(tt), "t_embedder.mlp.0")
            emb = self._f32_linear(F.silu(emb), "t_embedder.mlp.2")
            mod = self._f32_linear(F.silu(emb), "adaLN_modulation.1")
            self._embed_cache[key] = (emb, mod)
        return self._embed_cache[key]

    def prepare(self, cond: torch.Tensor) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """Per-block condition K/V of a ``[L, Cc]`` condition (once per sampling pass)."""
        return self.stack.prepare(cond.to(self.dt))

    def input_stage(self, feats: torch.Tensor, emb: torch.Tensor, geo: Geometry):
        """``input_layer`` -> res block -> downsampling res block (transformer.py:619-625)."""
        conv_emb = emb.to(self.dt)
        h = self._f32_linear(feats, "input_layer").to(self.dt)
        h = self._resblock(h, conv_emb, "input_blocks.0", geo.full)
        skip0 = h
        return self._down_block(h, conv_emb, geo), skip0

    def output_stage(self, h: torch.Tensor, skip_low: torch.Tensor, skip0: torch.Tensor, emb: torch.Tensor,
                     geo: Geometry) -> torch.Tensor:
        """Upsampling res block -> res block -> LayerNorm (eps 1e-5) -> ``out_layer``, fp32 output
        (transformer.py:627-634)."""
        conv_emb = emb.to(self.dt)
        h = self._up_block(torch.cat([h, skip_low], dim=1), conv_emb, geo)
        h = self._resblock(torch.cat([h, skip0], dim=1), conv_emb, "out_blocks.1", geo.full)
        h = F.layer_norm(h.float(), (h.shape[1],), eps=1e-5)
        return self._f32_linear(h, "out_layer")

    def __call__(self, feats: torch.Tensor, t: float, geo: Geometry, kvs: list | None,
                 negative: bool = False) -> list[torch.Tensor]:
        """Velocities ``[N, out]`` (fp32) for the branches: the condition (``kvs`` from
        :meth:`prepare`, or ``None`` for none) then, with ``negative``, the zero condition
        (transformer.py:636-668)."""
        emb, mod = self.embed(t)
        mod = mod.to(self.dt)
        h, skip0 = self.input_stage(feats.to(self.device), emb, geo)
        skip_low = h
        n_pos = 0 if kvs is None else 1
        batch = n_pos + (1 if negative else 0)
        if batch == 0:
            raise ValueError("branches must be [condition], [condition, None] or [None]")
        negatives = [transformer.negative_cross(w) for w in self.stack.weights] if negative else None
        x = h[None].expand(batch, *h.shape).contiguous()
        x = self.stack(x, mod, geo.rope_cos, geo.rope_sin, kvs, negatives, n_pos=n_pos,
                       shared_input=batch > 1)
        return [self.output_stage(x[b], skip_low, skip0, emb, geo) for b in range(batch)]
