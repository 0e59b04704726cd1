"""Checkpoint formats: config parsing, safetensors round trips, the reference's precision checks
(CPU); official and hi3d-w8a8-h64 files driving the B200 model (GPU)."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch
from conftest import rel_l2

from hi3d_b200 import checkpoint, synthetic
from hi3d_b200.transformer import Precision

SMALL = dict(model_channels=128, cond_channels=96, num_heads=2, num_blocks=2, io_block_channels=[64],
             in_channels=32, out_channels=32, patch_size=2, num_io_res_blocks=2)


def _artifact(tmp_path, weights):
    (tmp_path / "config.json").write_text(json.dumps(SMALL))
    checkpoint.save_weights(tmp_path / "model.safetensors", weights)
    return tmp_path


def test_config_and_round_trip(tmp_path):
    w = synthetic.model_weights(128, 96, 2, 2, io_channels=64, seed=3, std=None)
    art = _artifact(tmp_path, w)
    cfg, raw = checkpoint.load_config(art)
    assert (cfg.model_channels, cfg.num_heads, cfg.num_blocks, cfg.io_channels, cfg.head_dim) == (128, 2, 2, 64, 64)
    back, meta = checkpoint.load_weights(art / "model.safetensors")
    assert meta == {} or "format" not in meta
    assert set(back) == set(w)
    for k, v in w.items():
        assert back[k].dtype == v.dtype and np.array_equal(back[k], v), k


def test_config_rejects_other_io_stages(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps(dict(SMALL, io_block_channels=[64, 128], patch_size=4)))
    with pytest.raises(ValueError):
        checkpoint.load_config(tmp_path)


def test_precision_checks_follow_the_reference():
    w8 = {"blocks.0.self_attn.to_qkv.w8_scale": np.ones(3, np.float32)}
    meta = {"format": checkpoint.W8A8_FORMAT}
    checkpoint.check_precision(w8, meta, Precision(gemm="w8a8"))
    with pytest.raises(ValueError, match="w8a8 GEMM mode"):
        checkpoint.check_precision(w8, meta, Precision())
    with pytest.raises(ValueError, match="fp16 torso"):
        checkpoint.check_precision(w8, meta, Precision(dtype=torch.bfloat16, gemm="w8a8"))
    with pytest.raises(ValueError, match="released"):
        checkpoint.check_precision({}, {}, Precision(gemm="w8a8"))
    checkpoint.check_precision({}, {}, Precision())


def test_group_quantized_weight_only_files_are_rejected_by_name():
    # the reference's affine group-quantized format: 'layout' metadata + .scales/.biases
    layout = {"layout": json.dumps({"blocks.0.mlp.mlp.0": [64, 8]})}
    with pytest.raises(NotImplementedError, match="group-quantized"):
        checkpoint.check_precision({"blocks.0.mlp.mlp.0.weight": np.zeros(2, np.uint32)}, layout, Precision())
    with pytest.raises(NotImplementedError, match="group-quantized"):
        checkpoint.check_precision({"blocks.0.mlp.mlp.0.scales": np.ones(2, np.float16)}, {}, Precision())


@pytest.mark.gpu
def test_checkpoints_drive_the_model(tmp_path):
    from test_oracle_golden import forward_case

    from hi3d_b200 import model

    g, w, heads = forward_case()
    art = _artifact(tmp_path, w)
    m0 = model.Sparc3DTransformer(model.ModelConfig(128, 96, 2, 2, 64), w, device="cuda")
    m1, _ = checkpoint.from_checkpoint(art, device="cuda")
    geo = model.Geometry(g["coords"], 64)
    cond = torch.from_numpy(g["cond"]).cuda()
    feats = torch.from_numpy(g["feats"])
    v0 = m0(feats, float(g["t"]), geo, m0.prepare(cond))[0]
    v1 = m1(feats, float(g["t"]), geo, m1.prepare(cond))[0]
    assert torch.equal(v0, v1)

    q = checkpoint.save_w8a8(tmp_path / "w8a8.safetensors", w, num_blocks=2)
    loaded, meta = checkpoint.load_weights(tmp_path / "w8a8.safetensors")
    assert meta["format"] == checkpoint.W8A8_FORMAT
    assert sum(k.endswith(".w8_scale") for k in loaded) == 2 * 6
    assert loaded["blocks.1.mlp.mlp.2.weight"].dtype == np.int8
    assert np.array_equal(loaded["blocks.1.mlp.mlp.2.weight"], q["blocks.1.mlp.mlp.2.weight"])
    with pytest.raises(ValueError):
        checkpoint.from_checkpoint(art, tmp_path / "w8a8.safetensors", device="cuda")
    m2, _ = checkpoint.from_checkpoint(art, tmp_path / "w8a8.safetensors", Precision(gemm="w8a8"), device="cuda")
    v2 = m2(feats, float(g["t"]), geo, m2.prepare(cond))[0]
    assert torch.isfinite(v2).all()
    assert rel_l2(v2.cpu().numpy(), v0.cpu().numpy()) < 5e-2
