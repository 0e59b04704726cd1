"""Checkpoint formats of the refinement transformer: the official safetensors (fp16 torso, fp32
rest) and the released pre-quantized ``hi3d-w8a8-h64`` files.

Mirrors the loading in ``Sparc3DTransformerMLX.__init__`` (src/hi3d_mac/mlx_backend/
transformer.py:272-301) and the file layout recorded in models/w8a8/manifest.json:

* ``config.json`` of a ``transformer_*`` artifact holds the upstream ``Sparc3DTransformerConfig``
  fields (src/sparc3d/models/transformers/config.py:92-125), including the latent mean/std the
  sampler's output is de-normalised with;
* ``model.safetensors`` holds the upstream state dict;
* a ``hi3d-w8a8-h64`` file (safetensors metadata ``format``) replaces the six projections of every
  block (24 x 6 = 144 tensors) by int8 rows in the signed-H64 rotated domain, ``<name>.weight``,
  with fp32 per-row scales ``<name>.w8_scale`` (symmetric, maxabs / 127, round half to even);
  everything else is as in the official file.

:func:`convert_w8a8` produces such a file from official weights with this library's quantizer
(the same rotation and rounding as the activations).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from .model import ModelConfig, Sparc3DTransformer
from .transformer import BLOCK_PROJECTIONS, Precision

W8A8_FORMAT = "hi3d-w8a8-h64"
W8A8_METADATA = {
    "format": W8A8_FORMAT,
    "rotation": "signed normalized H64",
    "signs": "numpy.default_rng(314159+width).choice([-1.,1.],width)",
    "rounding": "nearest even",
    "weight_scaling": "symmetric per output row, maxabs/127",
}


def load_config(artifact: str | Path) -> tuple[ModelConfig, dict]:
    """``(ModelConfig, raw config dict)`` from an artifact's ``config.json``: one I/O stage
    (``io_block_channels`` of length 1, patch size 2) is required, as the reference's stages are
    written for it."""
    raw = json.loads((Path(artifact) / "config.json").read_text())
    io = list(raw.get("io_block_channels", [256]))
    if len(io) != 1 or int(raw.get("patch_size", 2)) != 2 or int(raw.get("num_io_res_blocks", 2)) != 2:
        raise ValueError("only one I/O stage (patch size 2, two res blocks) is supported, as in the reference")
    cfg = ModelConfig(model_channels=int(raw.get("model_channels", 2112)),
                      cond_channels=int(raw.get("cond_channels", 2048)), num_heads=int(raw.get("num_heads", 22)),
                      num_blocks=int(raw.get("num_blocks", 24)), io_channels=int(io[0]),
                      in_channels=int(raw.get("in_channels", 32)), out_channels=int(raw.get("out_channels", 32)))
    return cfg, raw


def load_weights(path: str | Path) -> tuple[dict[str, np.ndarray], dict[str, str]]:
    """All tensors of a safetensors file as numpy arrays, and its metadata."""
    from safetensors import safe_open

    tensors, meta = {}, {}
    with safe_open(str(path), framework="numpy") as f:
        meta = dict(f.metadata() or {})
        for k in f.keys():
            tensors[k] = f.get_tensor(k)
    return tensors, meta


def save_weights(path: str | Path, weights: dict, metadata: dict[str, str] | None = None) -> None:
    from safetensors.numpy import save_file

    arrays = {k: np.ascontiguousarray(v.detach().cpu().numpy() if isinstance(v, torch.Tensor) else v)
              for k, v in weights.items()}
    save_file(arrays, str(path), metadata=metadata)


def check_precision(tensors: dict, metadata: dict, precision: Precision) -> None:
    """The reference's checks (transformer.py:291-300): a ``hi3d-w8a8-h64`` file needs the W8A8
    GEMM mode and an fp16 torso; the W8A8 mode needs such a file.

    Any other pre-quantized file is the reference's affine group-quantized weight-only format
    (a ``layout`` metadata entry and ``*.scales``/``*.biases`` tensors, transformer.py:296-298,
    consumed by MLX ``quantized_matmul``); it is not supported here and is rejected by name
    instead of being read as dense weights."""
    if metadata.get("format") != W8A8_FORMAT and (
            "layout" in metadata or any(k.endswith((".scales", ".biases")) for k in tensors)):
        raise NotImplementedError(
            "affine group-quantized (weight-only INT8/INT4 'layout') checkpoints are not supported; "
            "use the original fp16/fp32 safetensors or a hi3d-w8a8-h64 file")
    if metadata.get("format") == W8A8_FORMAT:
        if precision.gemm != "w8a8" or precision.dtype != torch.float16:
            raise ValueError("W8A8 weights require the w8a8 GEMM mode and fp16 torso")
    if precision.gemm == "w8a8" and "blocks.0.self_attn.to_qkv.w8_scale" not in tensors:
        raise ValueError("W8A8 requires the released Hi3Dv1.0-mlx-w8a8 checkpoints")


def from_checkpoint(artifact: str | Path, weights_file: str | Path | None = None,
                    precision: Precision = Precision(), device=None) -> tuple[Sparc3DTransformer, dict]:
    """A model from an artifact directory (``config.json`` + ``model.safetensors``) or from a
    released pre-quantized file; returns ``(model, raw config)`` (the config carries
    ``latent_mean``/``latent_std`` for :func:`hi3d_b200.sampler.sample`)."""
    cfg, raw = load_config(artifact)
    tensors, meta = load_weights(weights_file if weights_file is not None else Path(artifact) / "model.safetensors")
    check_precision(tensors, meta, precision)
    return Sparc3DTransformer(cfg, tensors, device=device, dtype=precision.dtype), raw


def convert_w8a8(weights: dict, num_blocks: int, device=None) -> dict[str, np.ndarray]:
    """Official weights -> the ``hi3d-w8a8-h64`` tensor set: the six projections of every block
    quantized on the GPU (signed-H64 rotation, per-row maxabs / 127, round half to even)."""
    from . import w8a8

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = {k: (v.detach().cpu().numpy() if isinstance(v, torch.Tensor) else v) for k, v in weights.items()}
    for i in range(num_blocks):
        for name in BLOCK_PROJECTIONS:
            key = f"blocks.{i}.{name}"
            w = torch.as_tensor(np.ascontiguousarray(out[f"{key}.weight"])).to(dev, torch.float16)
            q, s = w8a8.quantize_weight(w, rotate=True)
            out[f"{key}.weight"] = q.cpu().numpy()
            out[f"{key}.w8_scale"] = s.cpu().numpy().astype(np.float32)
    return out


def save_w8a8(path: str | Path, weights: dict, num_blocks: int, device=None) -> dict[str, np.ndarray]:
    """Write the ``hi3d-w8a8-h64`` file of ``weights``; returns the tensors written."""
    q = convert_w8a8(weights, num_blocks, device)
    save_weights(path, q, dict(W8A8_METADATA))
    return q
