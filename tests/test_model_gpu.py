"""The whole refinement transformer and its I/O kernels on the GPU, against the CPU oracle.

Kernels: LayerNorm + SiLU, sparse conv + SiLU, children lists of the downsampling, the mean
downsample, the up-convolution gather-sum and the row gather (src/hi3d_mac/mlx_backend/
transformer.py:235-266, :413-485).  Model: the fp16 forward vs the fp32 oracle, which
tests/test_oracle_golden.py pins to the upstream Sparc3DTransformer.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import rel_l2
from test_oracle_golden import forward_case

from hi3d_b200 import kernels, model, sparse, synthetic
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


def _silu16(h: np.ndarray) -> np.ndarray:
    return ops.silu_f32(h.astype(np.float32)).astype(np.float16)


def _ulps_close(a: np.ndarray, b: np.ndarray, min_equal: float) -> None:
    """Within a few fp16 ulps of the expected value everywhere (relative 4e-3) and bit-identical
    on ``min_equal`` of the elements.  SiLU is evaluated with the fast exponential, and the
    LayerNorm statistics may differ from the oracle's summation order in the last bit; near zero
    SiLU halves its input, so one ulp of its input is two of its output."""
    af, bf = a.astype(np.float32), b.astype(np.float32)
    bad = np.abs(af - bf) > 4e-3 * np.abs(bf) + 1e-7
    assert not bad.any(), (int(bad.sum()), af[bad][:5], bf[bad][:5])
    equal = (a.astype(np.float16).view(np.int16) == b.astype(np.float16).view(np.int16)).mean()
    assert equal >= min_equal, equal


@pytest.mark.parametrize("c", [64, 256, 1056, 4224])
def test_layer_norm_silu(c):
    rng = np.random.default_rng(c)
    x = (rng.standard_normal((300, c)) * 2 + 0.3).astype(np.float16)
    w = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = rng.normal(0, 0.1, c).astype(np.float32)
    sc = (1 + 0.2 * rng.standard_normal(c)).astype(np.float16)
    sh = (0.1 * rng.standard_normal(c)).astype(np.float16)
    for kw in (dict(weight=w, bias=b), dict(scale=sc, shift=sh)):
        dkw = {k: _t(v) for k, v in kw.items()}
        plain = kernels.layer_norm_modulate(_t(x), 1e-6, **dkw).cpu().numpy()
        got = kernels.layer_norm_modulate(_t(x), 1e-6, act="silu", **dkw).cpu().numpy()
        # the fused SiLU vs SiLU of the kernel's own LayerNorm output
        _ulps_close(got, _silu16(plain), 0.99)
        # and the LayerNorm part vs the oracle (one ulp where the fp32 summation order differs)
        assert (plain == ops.layer_norm_modulate(x, 1e-6, **kw)).mean() > 0.999


def test_layer_norm_silu_rejects_affine_and_modulation_together():
    x = torch.zeros(8, 64, dtype=torch.float16, device=DEV)
    one = torch.ones(64, device=DEV)
    with pytest.raises(NotImplementedError):
        kernels.layer_norm_modulate(x, 1e-6, weight=one, bias=one, scale=one.half(), shift=one.half(), act="silu")


def test_conv_silu_equals_conv_then_silu():
    rng = np.random.default_rng(3)
    coords = synthetic.shell_coords(3000, 32, 10, 2, seed=4)
    table = sparse.neighbour_table(coords)
    x = _t(rng.standard_normal((coords.shape[0], 64)).astype(np.float16))
    w = _t((rng.standard_normal((32, 3, 3, 3, 64)) * 0.03).astype(np.float16))
    b = _t((rng.standard_normal(32) * 0.1).astype(np.float16))
    plain = sparse.conv(x, table, w, b).cpu().numpy()
    fused = sparse.conv(x, table, w, b, act="silu").cpu().numpy()
    _ulps_close(fused, _silu16(plain), 0.99)


def test_downsample_children_and_structure():
    rng = np.random.default_rng(8)
    coords = synthetic.shell_coords(5000, 64, 24, 3, seed=9)
    coords = coords[rng.permutation(coords.shape[0])]
    low, inverse, counts, children, offsets = (t.cpu().numpy() for t in sparse.downsample_groups(coords))
    rl, ri, rc = ops.downsample_structure(coords)
    assert np.array_equal(low, rl) and np.array_equal(inverse, ri) and np.array_equal(counts, rc)
    assert np.array_equal(children, np.argsort(ri, kind="stable"))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(rc)]))


def _mean_in_row_order(x: np.ndarray, children: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    """fp32 sums over the children in ascending row order, / (count + 1), rounded once."""
    m = offsets.shape[0] - 1
    acc = np.zeros((m, x.shape[1]), np.float32)
    cnt = np.diff(offsets)
    xf = x.astype(np.float32)
    for j in range(int(cnt.max())):
        has = cnt > j
        acc[has] = acc[has] + xf[children[offsets[:-1][has] + j]]
    return (acc / (cnt.astype(np.float32) + 1)[:, None]).astype(x.dtype)


@pytest.mark.parametrize("c", [64, 1024])
def test_downsample_mean_bit_exact(c):
    rng = np.random.default_rng(c)
    coords = synthetic.shell_coords(4000, 48, 16, 3, seed=c)
    x = (rng.standard_normal((coords.shape[0], c)) * 3).astype(np.float16)
    _, inverse, counts, children, offsets = sparse.downsample_groups(coords)
    got = sparse.downsample_mean(_t(x), children, offsets).cpu().numpy()
    want = _mean_in_row_order(x, children.cpu().numpy(), offsets.cpu().numpy())
    assert np.array_equal(got.view(np.int16), want.view(np.int16))
    ref = ops.downsample_mean_f32(x, inverse.cpu().numpy(), counts.cpu().numpy())
    assert rel_l2(got, ref) < 1e-3


def test_upconv_gather_sum_bit_exact_and_equals_upsampled_conv():
    rng = np.random.default_rng(11)
    coords = synthetic.shell_coords(3000, 40, 12, 3, seed=12)
    geo = model.Geometry(coords, head_dim=64)
    cin, cout = 128, 32
    h = (rng.standard_normal((geo.low.n, cin))).astype(np.float16)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) / np.sqrt(27 * cin)).astype(np.float16)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float16)
    got = sparse.up_conv(_t(h), geo.full.table, geo.inverse, _t(w), _t(b)).cpu().numpy()
    # the kernel's sums, restated: the GEMM's projections (taken from the GPU, rounded to fp16),
    # then fp32 in tap order and + bias
    w_taps = torch.from_numpy(w.reshape(cout, 27, cin).transpose(1, 0, 2).reshape(27 * cout, cin).copy())
    from hi3d_b200 import linear

    proj = linear.linear(_t(h), w_taps.to(DEV)).cpu().numpy().reshape(-1, cout).astype(np.float32)
    table = geo.full.table.cpu().numpy()
    inv = geo.inverse.cpu().numpy()
    n = coords.shape[0]
    acc = np.zeros((n, cout), np.float32)
    for k in range(27):
        j = table[:, k]
        has = j < n
        acc[has] = acc[has] + proj[inv[j[has]].astype(np.int64) * 27 + k]
    want = (acc + b.astype(np.float32)).astype(np.float16)
    assert np.array_equal(got.view(np.int16), want.view(np.int16))
    ref = ops.subm_conv(h[inv], table, ops.conv_weight(w.astype(np.float32)), b.astype(np.float32))
    assert rel_l2(got, ref) < 2e-3


def test_gather_rows_exact():
    rng = np.random.default_rng(2)
    src = rng.standard_normal((100, 48)).astype(np.float16)
    idx = rng.integers(0, 100, 777).astype(np.int32)
    got = sparse.upsample(_t(src), _t(idx)).cpu().numpy()
    assert np.array_equal(got, src[idx])


def _forward_setup():
    g, w, heads = forward_case()
    c, cc, _, nblk, io, _ = (int(v) for v in g["config"])
    cfg = model.ModelConfig(model_channels=c, cond_channels=cc, num_heads=heads, num_blocks=nblk, io_channels=io)
    m = model.Sparc3DTransformer(cfg, w, device=DEV)
    geo = model.Geometry(g["coords"], cfg.head_dim)
    return g, w, heads, m, geo


def test_forward_matches_oracle_and_upstream():
    """fp16 forward on the B200 kernels vs the fp32 oracle and the upstream fp32 velocity."""
    g, w, heads, m, geo = _forward_setup()
    kvs = m.prepare(_t(g["cond"]))
    vel = m(_t(g["feats"]), float(g["t"]), geo, kvs)[0].cpu().numpy()
    ref = ops.forward_f32(w, g["feats"], g["coords"], float(g["t"]), g["cond"], heads)
    assert vel.dtype == np.float32 and vel.shape == ref.shape
    assert rel_l2(vel, ref) < 5e-3
    assert rel_l2(vel, g["velocity"]) < 5e-3


def test_forward_branches_share_the_conditioned_result():
    """The [condition, zero condition] batch gives the single-branch velocity for its first
    branch (rows of the batched GEMMs and attention are independent)."""
    g, w, heads, m, geo = _forward_setup()
    kvs = m.prepare(_t(g["cond"]))
    single = m(_t(g["feats"]), float(g["t"]), geo, kvs)[0]
    both = m(_t(g["feats"]), float(g["t"]), geo, kvs, negative=True)
    assert len(both) == 2
    assert torch.equal(both[0], single)
    assert torch.isfinite(both[1]).all() and not torch.equal(both[1], single)
