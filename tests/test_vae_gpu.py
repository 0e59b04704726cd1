"""Sparse VAE decoder kernels on the GPU vs the CPU oracle: GroupNorm statistics and swish,
conv(swish(GN(x))), the octree child table, serialization and window attention
(src/hi3d_mac/mlx_backend/vae.py, kernels.py:242-296, sparse.py:46-95)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN, rel_l2

from hi3d_b200 import sparse, synthetic, vae
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


# 512/128/64/256: row-blocked swish kernel (256 % (c / 8) == 0); 24: 8-channel vector kernel;
# 12: scalar kernels
@pytest.mark.parametrize("c,dtype", [(512, np.float16), (128, np.float32), (64, np.float16), (256, np.float32),
                                     (24, np.float16), (12, np.float32)])
def test_group_stats_and_swish(c, dtype):
    rng = np.random.default_rng(c)
    x = (rng.standard_normal((20000, c)) * rng.uniform(0.5, 3, c) + rng.normal(0, 1, c)).astype(dtype)
    mean, inv = vae.group_stats(_t(x))
    rm, ri = ops.group_stats_f64(x)
    assert np.allclose(mean.cpu().numpy(), rm, rtol=1e-5, atol=1e-6)
    assert np.allclose(inv.cpu().numpy(), ri, rtol=1e-5)
    w = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = rng.normal(0, 0.2, c).astype(np.float32)
    want = ops.group_norm_swish(x, rm, ri, w, b)
    out32 = vae.group_norm_swish(_t(x), mean, inv, _t(w), _t(b), out_dtype=torch.float32).cpu().numpy()
    assert np.allclose(out32, want, rtol=2e-5, atol=2e-6)
    out16 = vae.group_norm_swish(_t(x), mean, inv, _t(w), _t(b), out_dtype=torch.float16).cpu().numpy()
    assert np.allclose(out16.astype(np.float64), want, rtol=1e-3, atol=1e-4)


def test_conv_gn_swish_matches_oracle():
    rng = np.random.default_rng(4)
    coords = synthetic.shell_coords(6000, 48, 16, 3, seed=5)
    level = sparse.Level.from_coords(coords)
    cin, cout = 256, 128
    x = (rng.standard_normal((coords.shape[0], cin)) * 2).astype(np.float16)
    nw, nb = rng.uniform(0.5, 1.5, cin).astype(np.float32), rng.normal(0, 0.1, cin).astype(np.float32)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) / np.sqrt(27 * cin)).astype(np.float16)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float16)
    got = vae.conv_gn_swish(_t(x), level, _t(nw), _t(nb), _t(w), _t(b)).cpu().numpy()
    m, i = ops.group_stats_f64(x)
    act = ops.group_norm_swish(x, m, i, nw, nb)
    want = ops.subm_conv(act, level.table_np, ops.conv_weight(w.astype(np.float64)), b.astype(np.float64))
    assert rel_l2(got, want) < 2e-3


def test_child_table_matches_reference_helper():
    g = np.load(GOLDEN / "vae.npz")
    table, parent, slot = vae.child_neighbour_table(_t(g["parent_table"]), _t(g["child_mask"]))
    t = table.cpu().numpy()
    assert t.shape == g["child_table"].shape, (t.shape, g["child_table"].shape)
    bad = np.argwhere(t != g["child_table"])
    assert bad.size == 0, (bad[:5], t[tuple(bad[:5].T)], g["child_table"][tuple(bad[:5].T)])
    assert np.array_equal(parent.cpu().numpy(), g["child_parent"])
    assert np.array_equal(slot.cpu().numpy(), g["child_slot"])


@pytest.mark.parametrize("density", [0.0, 0.05, 0.5, 1.0])
def test_child_table_large_and_edge_masks(density):
    rng = np.random.default_rng(int(density * 100))
    coords = synthetic.shell_coords(50000, 96, 30, 3, seed=7)
    ptable = sparse.neighbour_table(coords)
    mask = rng.random((coords.shape[0], 8)) < density
    table, parent, slot = (t.cpu().numpy() for t in vae.child_neighbour_table(ptable, _t(mask)))
    rt, rp, rs = ops.child_neighbour_table(ptable.cpu().numpy(), mask)
    assert table.shape == rt.shape
    assert np.array_equal(table, rt) and np.array_equal(parent, rp) and np.array_equal(slot, rs)


def test_serialization_bit_exact():
    g = np.load(GOLDEN / "vae.npz")
    for coords in (g["serial_coords"], synthetic.shell_coords(100000, 128, 48, 4, seed=9)):
        ours = vae.serialization(coords)
        for (perm, inverse), (rp, ri) in zip(ours, ops.serialization(coords)):
            assert np.array_equal(perm.cpu().numpy(), rp) and np.array_equal(inverse.cpu().numpy(), ri)
            assert np.array_equal(vae.window_index(perm).cpu().numpy(), ops.window_index(rp))


# misaligned: qkv starts one element past a 16-byte boundary (the scalar kernel); otherwise
# the vectorised kernel
@pytest.mark.parametrize("n,heads,d,dtype,misaligned",
                         [(1000, 32, 16, torch.float32, False), (1000, 32, 16, torch.float16, False),
                          (960, 8, 32, torch.float16, False), (30, 4, 64, torch.float32, False),
                          (5000, 32, 16, torch.float16, False), (1000, 32, 16, torch.float16, True),
                          (700, 4, 64, torch.float32, True), (700, 4, 64, torch.float16, False)])
def test_window_attention_matches_oracle(n, heads, d, dtype, misaligned):
    rng = np.random.default_rng(n + d)
    coords = synthetic.shell_coords(n, 48, 14, 3, seed=n)
    perm, inverse = vae.serialization(coords)[n % 2]
    gather = vae.window_index(perm)
    qkv = rng.standard_normal((n, 3 * heads * d)).astype(np.float32)
    q_dev = _t(qkv).to(dtype)
    if misaligned:
        buf = torch.empty(q_dev.numel() + 1, dtype=dtype, device=DEV)
        buf[1:].copy_(q_dev.reshape(-1))
        q_dev = buf[1:].view(q_dev.shape)
        assert q_dev.is_contiguous() and q_dev.data_ptr() % 16 != 0
    got = vae.window_attention(q_dev, gather, heads).float().cpu().numpy()
    want = ops.window_attention_f64(qkv, gather.cpu().numpy(), inverse.cpu().numpy(), heads)
    assert rel_l2(got, want) < (2e-6 if dtype == torch.float32 else 2e-3)
