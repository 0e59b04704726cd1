"""Pins the CPU oracle (oracle/ops.py) to outputs of the reference's own code.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py from the
reference's upstream PyTorch modules + torch shims and its pure-numpy MLX helpers.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import GOLDEN, rel_l2

from oracle import ops


def _load(name):
    return np.load(GOLDEN / f"{name}.npz")


@pytest.mark.parametrize("tag", ["a", "b"])
@pytest.mark.parametrize("d", [64, 96])
def test_rope_tables_bit_exact(tag, d):
    g = _load("rope")
    cos, sin = ops.rope_tables(g[f"coords_{tag}"], d)
    assert np.array_equal(cos, g[f"cos_{tag}{d}"]) and np.array_equal(sin, g[f"sin_{tag}{d}"])


def test_qkv_rope_rms_matches_upstream_modules():
    g = _load("rope")
    cos, sin = ops.rope_tables(g["coords_b"], 64)
    q, k, v = ops.qkv_rope_rms(g["qkv"], cos, sin, g["gq"], g["gk"], 1, 3, 64)
    # oracle is [B, H, N, D]; upstream gives [N, H, D]
    assert np.allclose(q[0].transpose(1, 0, 2), g["q_ref"], atol=2e-5, rtol=1e-5)
    assert np.allclose(k[0].transpose(1, 0, 2), g["k_ref"], atol=2e-5, rtol=1e-5)
    assert np.array_equal(v[0].transpose(1, 0, 2), g["qkv"].reshape(50, 3, 3, 64)[:, 2])


def test_layer_norm_modulate_matches_upstream_fp16_path():
    g = _load("layernorm")
    x = g["x"]
    scale16 = (1 + g["scale"]).astype(np.float16)  # sparse_batch_broadcast rounds (1 + scale) to fp16
    shift16 = g["shift"].astype(np.float16)
    for got, ref in ((ops.layer_norm_modulate(x, 1e-6), g["plain"]),
                     (ops.layer_norm_modulate(x, 1e-6, g["w"], g["b"]), g["affine"]),
                     (ops.layer_norm_modulate(x, 1e-6, scale=scale16, shift=shift16), g["modulated"])):
        assert got.dtype == np.float16 and ref.dtype == np.float16
        assert (got == ref).mean() > 0.999
        assert np.allclose(got.astype(np.float32), ref.astype(np.float32), atol=1e-2, rtol=1e-3)


def test_attention_matches_reference_shim():
    g = _load("attention")
    qkv, cu = g["qkv"], g["cu"]
    got = ops.attention_varlen(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, cu, 64 ** -0.5)
    assert np.allclose(got, g["self_out"], atol=1e-5)
    kv = g["kv"]
    got = ops.attention_varlen(g["q"], kv[:, 0], kv[:, 1], [0, 70], [0, 30], 64 ** -0.5)
    assert np.allclose(got, g["cross_out"], atol=1e-5)


def test_sparse_structure_bit_exact():
    g = _load("sparse")
    assert np.array_equal(ops.neighbour_table(g["coords"]), g["table"])
    low, inv, cnt = ops.downsample_structure(g["coords"])
    assert np.array_equal(low, g["low"]) and np.array_equal(inv, g["inverse"]) and np.array_equal(cnt, g["counts"])


def test_subm_conv_matches_spconv_shim():
    g = _load("sparse")
    table = ops.neighbour_table(g["coords"])
    out = ops.subm_conv(g["feats"], table, ops.conv_weight(g["weight"]), g["bias"])
    assert np.allclose(out, g["conv_out"], atol=1e-10, rtol=1e-10)


def test_block_forward_matches_upstream_module():
    g = _load("block")
    w = {k[2:]: g[k] for k in g.files if k.startswith("w:")}
    coords = g["coords"][:, 1:]
    lens = [int(n) for n in g["lens"]]
    cos, sin = ops.rope_tables(coords, 64)
    y = ops.block_forward_f32(w, g["x"], g["mod"], cos, sin, g["ctx"], heads=2, seqlens=lens)
    assert rel_l2(y, g["y"]) < 1e-5


def test_torch_block_port_matches_upstream_module():
    """The torch restatement of the reference's CPU path (timed as the CPU baseline, and the
    checker of the full-size parity tests) against the upstream module, in full and on a row
    subset (keys and values still from every token)."""
    from oracle import torch_block

    g = _load("block")
    w = {k[2:]: g[k] for k in g.files if k.startswith("w:")}
    lens = [int(n) for n in g["lens"]]
    cos, sin = ops.rope_tables(g["coords"][:, 1:], 64)
    y = torch_block.block_forward(w, g["x"], g["mod"], cos, sin, g["ctx"], 2, seqlens=lens).numpy()
    assert rel_l2(y, g["y"]) < 1e-5
    rows = np.array([0, 3, 59, 60, 61, 119])
    yr = torch_block.block_forward(w, g["x"], g["mod"], cos, sin, g["ctx"], 2, seqlens=lens, rows=rows).numpy()
    assert rel_l2(yr, g["y"][rows]) < 1e-5


def forward_case():
    """Inputs, weights and the upstream velocity of the whole-transformer fixture."""
    from hi3d_b200 import synthetic

    g = _load("forward")
    c, cc, heads, nblk, io, seed = (int(v) for v in g["config"])
    w = synthetic.model_weights(c, cc, heads, nblk, io_channels=io, seed=seed, std=None)
    checksum = sum(float(np.abs(v.astype(np.float64)).sum()) for v in w.values())
    assert checksum == float(g["weight_checksum"]), "the seeded weight generator changed"
    return g, w, heads


def test_forward_matches_upstream_transformer():
    """The whole refinement transformer (fp32): oracle vs the upstream Sparc3DTransformer."""
    g, w, heads = forward_case()
    vel = ops.forward_f32(w, g["feats"], g["coords"], float(g["t"]), g["cond"], heads)
    assert vel.shape == g["velocity"].shape
    assert rel_l2(vel, g["velocity"]) < 1e-5


def test_resampling_oracle_identities():
    """The restructured up-convolution equals upsample-then-conv, and the mean divides by
    children + 1 (transformer.py:249-251, :449-475)."""
    rng = np.random.default_rng(5)
    coords = np.unique(rng.integers(0, 12, (300, 3)), axis=0).astype(np.int32)
    low, inverse, counts = ops.downsample_structure(coords)
    x = rng.standard_normal((coords.shape[0], 8)).astype(np.float32)
    mean = ops.downsample_mean_f32(x, inverse, counts)
    j = int(inverse[0])
    assert np.allclose(mean[j], x[inverse == j].sum(0) / (counts[j] + 1), rtol=1e-6)
    h = rng.standard_normal((low.shape[0], 16)).astype(np.float32)
    wt = rng.standard_normal((8, 3, 3, 3, 16)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    table = ops.neighbour_table(coords)
    direct = ops.subm_conv(h[inverse], table, ops.conv_weight(wt), b)
    assert rel_l2(ops.up_conv_f32(h, wt, b, table, inverse), direct) < 1e-6


def test_vae_index_structures_bit_exact():
    """Octree child table, serialization and window index vs the reference's MLX helpers."""
    g = _load("vae")
    table, parent, slot = ops.child_neighbour_table(g["parent_table"], g["child_mask"])
    assert np.array_equal(table, g["child_table"])
    assert np.array_equal(parent, g["child_parent"]) and np.array_equal(slot, g["child_slot"])
    for i, (perm, inverse) in enumerate(ops.serialization(g["serial_coords"])):
        assert np.array_equal(perm, g[f"perm{i}"]) and np.array_equal(inverse, g[f"inverse{i}"])
        assert np.array_equal(ops.window_index(perm), g[f"gather{i}"])
        assert np.array_equal(inverse, g[f"scatter{i}"])


def test_child_table_geometry():
    """A child's neighbour rows are the children at its coordinate + offset."""
    g = _load("vae")
    table, parent, slot = ops.child_neighbour_table(g["parent_table"], g["child_mask"])
    bits = np.stack([(slot >> 2) & 1, (slot >> 1) & 1, slot & 1], 1)
    coords = g["parent_coords"][parent] * 2 + bits
    assert np.array_equal(table, ops.neighbour_table(coords))


@pytest.mark.parametrize("k", [64, 1024, 2112, 4096])
def test_w8a8_signs_bit_exact(k):
    assert np.array_equal(ops.signs(k), _load("w8a8")[f"signs{k}"])


def test_h64_is_the_natural_order_hadamard():
    from scipy.linalg import hadamard

    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 128)).astype(np.float32)
    y = ops._h64_butterfly(x, np.ones(128, np.float32))
    h = hadamard(64).astype(np.float64) / 8
    ref = np.concatenate([x[:, :64] @ h.T, x[:, 64:] @ h.T], 1)
    assert np.allclose(y, ref, atol=1e-5)


def test_w8a8_reference_contract_on_oracle():
    """tests/test_w8a8_inference.py:8-20 of the reference, with the oracle quantizer."""
    rng = np.random.default_rng(7)
    for rows, cols, width in ((3, 17, 64), (65, 131, 2112), (7, 33, 8448)):
        x = rng.normal(size=(rows, width)).astype(np.float16)
        w = rng.integers(-127, 128, size=(cols, width), dtype=np.int8)
        sw = rng.uniform(.0001, .001, cols).astype(np.float32)
        bias = rng.normal(0, .01, cols).astype(np.float16)
        a, sa = ops.quantize_activation(x)
        assert a.dtype == np.int8 and np.abs(a).max() <= 127 and sa.shape == (rows,)
        y = ops.w8a8_linear_expected(a, sa, w, sw, bias)
        assert np.isfinite(y).all()
