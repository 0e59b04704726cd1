"""GPU sparse structure (bit-exact) and gather-GEMM convolution vs the CPU oracle.

Pair/structure exactness follows the reference's own checks (tests/test_backends.py:21-67,
tests/test_mlx_kernels.py:79-89): neighbour tables and downsample structures bit-exact; the
convolution against float64 gathers and a dense ``conv3d``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN, rel_l2

from hi3d_b200 import sparse, synthetic
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


def test_neighbour_table_and_downsample_golden():
    g = np.load(GOLDEN / "sparse.npz")
    table = sparse.neighbour_table(g["coords"]).cpu().numpy()
    assert np.array_equal(table, g["table"])
    low, inv, cnt = (t.cpu().numpy() for t in sparse.downsample_structure(g["coords"]))
    assert np.array_equal(low, g["low"]) and np.array_equal(inv, g["inverse"]) and np.array_equal(cnt, g["counts"])


def test_structures_bit_exact_at_config5_size():
    coords = synthetic.shell_coords(200_000, 128, 48, 4, seed=5)
    coords = coords[np.random.default_rng(0).permutation(coords.shape[0])]  # arbitrary row order
    assert np.array_equal(sparse.neighbour_table(coords).cpu().numpy(), ops.neighbour_table(coords))
    got = [t.cpu().numpy() for t in sparse.downsample_structure(coords)]
    for a, b in zip(got, ops.downsample_structure(coords)):
        assert np.array_equal(a, b)


def test_strided_query_table():
    rng = np.random.default_rng(1)
    coords = np.argwhere(rng.random((20, 20, 20)) < 0.2).astype(np.int32)
    low, _, _ = ops.downsample_structure(coords)
    got = sparse.neighbour_table(coords, query=low, stride=2).cpu().numpy()
    n = coords.shape[0]
    lut = {tuple(c): i for i, c in enumerate(coords)}
    want = np.full((low.shape[0], 27), n, np.int32)
    for o, q in enumerate(low):
        for k, d in enumerate(ops.OFFSETS):
            want[o, k] = lut.get(tuple(2 * q + d), n)
    assert np.array_equal(got, want)


def test_empty_and_single_voxel():
    t = sparse.neighbour_table(np.array([[3, 4, 5]], np.int32)).cpu().numpy()
    assert t.shape == (1, 27) and t[0, 13] == 0 and (np.delete(t[0], 13) == 1).all()
    assert sparse.neighbour_table(np.zeros((0, 3), np.int32)).shape == (0, 27)


def test_subm_conv_matches_spconv_shim_golden():
    g = np.load(GOLDEN / "sparse.npz")
    # the golden uses 5 -> 7 channels; the kernel needs multiples of 8: zero-pad both
    w = np.zeros((8, 3, 3, 3, 8))
    w[:7, ..., :5] = g["weight"]
    feats = np.zeros((g["feats"].shape[0], 8))
    feats[:, :5] = g["feats"]
    bias = np.zeros(8)
    bias[:7] = g["bias"]
    level = sparse.Level.from_coords(g["coords"])
    out = sparse.conv(_t(feats, torch.float16), level.table, _t(w, torch.float16), _t(bias, torch.float16))
    got = out.float().cpu().numpy()[:, :7]
    assert rel_l2(got, g["conv_out"]) < 3e-3  # fp16 inputs/weights vs the fp64 reference


@pytest.mark.parametrize("cin,cout,dtype", [(64, 64, torch.float16), (256, 256, torch.float16), (96, 320, torch.float16),
                                            (128, 128, torch.bfloat16)])
def test_subm_conv_matches_float64_gather(cin, cout, dtype):
    rng = np.random.default_rng(cin + cout)
    coords = synthetic.shell_coords(5000, 48, 16, 3, seed=cin)
    coords = coords[rng.permutation(coords.shape[0])]
    x = _t(rng.standard_normal((coords.shape[0], cin)).astype(np.float32), dtype)
    w = _t((rng.standard_normal((cout, 3, 3, 3, cin)) * 0.05).astype(np.float32), dtype)
    b = _t((rng.standard_normal(cout) * 0.1).astype(np.float32), dtype)
    level = sparse.Level.from_coords(coords)
    got = sparse.conv(x, level.table, w, b).float().cpu().numpy()
    wt = ops.conv_weight(w.double().cpu().numpy())
    ref = ops.subm_conv(x.double().cpu().numpy(), ops.neighbour_table(coords), wt, b.double().cpu().numpy())
    tol = 2e-3 if dtype == torch.float16 else 1e-2
    assert rel_l2(got, ref) < tol
    # the reference's MLX surface: weight_t [27*Cin, Cout]
    got2 = sparse.sparse_conv(x, level, sparse.conv_weight(w), b).float().cpu().numpy()
    assert np.array_equal(got, got2)


def test_conv_isolated_voxels_and_ragged_tiles():
    coords = (np.arange(300)[:, None] * np.array([[3, 0, 0]]) % 240 + np.array([[0, 5, 7]])).astype(np.int32)
    coords = np.unique(coords, axis=0)  # isolated voxels: only the centre tap exists
    rng = np.random.default_rng(3)
    x = _t(rng.standard_normal((coords.shape[0], 64)).astype(np.float16))
    w = _t((rng.standard_normal((64, 3, 3, 3, 64)) * 0.05).astype(np.float16))
    got = sparse.conv(x, sparse.neighbour_table(coords), w).float().cpu().numpy()
    ref = x.double().cpu().numpy() @ w.double().cpu().numpy()[:, 1, 1, 1, :].T
    assert rel_l2(got, ref) < 2e-3
    far = np.array([[0, 0, 0], [100, 100, 100]], np.int32)  # tiles with only the centre tap
    out = sparse.conv(_t(rng.standard_normal((2, 64)).astype(np.float16)), sparse.neighbour_table(far), w)
    assert torch.isfinite(out.float()).all()


def test_stride2_conv_matches_dense_conv3d():
    import torch.nn.functional as F

    rng = np.random.default_rng(4)
    side = 18
    coords = np.argwhere(rng.random((side,) * 3) < 0.25).astype(np.int32)
    cin, cout = 32, 48
    x = rng.standard_normal((coords.shape[0], cin)).astype(np.float16)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) * 0.1).astype(np.float16)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float16)
    out, low = sparse.downsample_conv(_t(x), coords, _t(w), _t(b))
    low = low.cpu().numpy()
    dense = torch.zeros(1, cin, side, side, side, dtype=torch.float64)
    i, j, k = coords.T
    dense[0, :, i, j, k] = torch.from_numpy(x.astype(np.float64)).T
    wd = torch.from_numpy(w.astype(np.float64)).permute(0, 4, 1, 2, 3)
    ref = F.conv3d(dense, wd, torch.from_numpy(b.astype(np.float64)), stride=2, padding=1)[0]
    ref = ref[:, low[:, 0], low[:, 1], low[:, 2]].T.numpy()
    assert rel_l2(out.float().cpu().numpy(), ref) < 2e-3


def test_config5_conv_sampled_rows():
    """cfg5 size: 200k voxels, C=256 -> 256; sampled rows against a float64 gather."""
    rng = np.random.default_rng(5)
    coords = synthetic.shell_coords(200_000, 128, 48, 4, seed=5)
    x = _t(rng.standard_normal((coords.shape[0], 256)).astype(np.float16))
    w = _t((rng.standard_normal((256, 3, 3, 3, 256)) * 0.02).astype(np.float16))
    b = _t((rng.standard_normal(256) * 0.02).astype(np.float16))
    level = sparse.Level.from_coords(coords)
    got = sparse.conv(x, level.table, w, b)
    rows = np.sort(rng.choice(coords.shape[0], 2000, replace=False))
    tab = level.table[rows].long().cpu().numpy()
    xs = np.concatenate([x.double().cpu().numpy(), np.zeros((1, 256))], 0)
    wk = w.double().cpu().numpy().reshape(256, 27, 256)
    ref = np.einsum("rkc,okc->ro", xs[tab], wk) + b.double().cpu().numpy()
    assert rel_l2(got[rows].float().cpu().numpy(), ref) < 2e-3


def test_spconv_shim_matches_golden_and_dense_conv3d():
    """The spconv drop-in (tests/test_backends.py:21-67 of the reference): SubMConv3d against the
    reference shim's fp64 golden, the pair layout coords[dst] == coords[src] + 1 - r, and the
    k <-> 26 - k count symmetry of submanifold pairs."""
    from hi3d_b200.torch_backend import sparse_conv as sc

    g = np.load(GOLDEN / "sparse.npz")
    xyz = g["coords"]
    indices = _t(np.concatenate([np.zeros((xyz.shape[0], 1), np.int32), xyz], 1))
    conv = sc.SubMConv3d(8, 8, 3, bias=True, indice_key="subm3").to(DEV)
    w = np.zeros((8, 3, 3, 3, 8))
    w[:7, ..., :5] = g["weight"]
    b = np.zeros(8)
    b[:7] = g["bias"]
    with torch.no_grad():
        conv.weight.copy_(torch.from_numpy(w))
        conv.bias.copy_(torch.from_numpy(b))
    conv = conv.half()
    feats = np.zeros((xyz.shape[0], 8))
    feats[:, :5] = g["feats"]
    x = sc.SparseConvTensor(_t(feats, torch.float16), indices, [12, 12, 12], 1)
    out = conv(x)
    assert "subm3" in x.indice_dict
    assert rel_l2(out.features.float().cpu().numpy()[:, :7], g["conv_out"]) < 3e-3
    _, pairs, counts = sc.get_indice_pairs(indices, 1, [12, 12, 12], sc.ConvAlgo.Native, (3, 3, 3), (1, 1, 1),
                                           (1, 1, 1), (1, 1, 1), (0, 0, 0), True, False)
    coords = torch.from_numpy(xyz.astype(np.int64))
    for k in range(27):
        r = torch.tensor([k // 9, (k // 3) % 3, k % 3])
        n = int(counts[k])
        src, dst = pairs[0, k, :n].cpu(), pairs[1, k, :n].cpu()
        assert torch.equal(coords[dst], coords[src] + 1 - r)
        assert n == int(counts[26 - k])
    with pytest.raises(NotImplementedError):
        sc.get_indice_pairs(indices, 1, [12] * 3, sc.ConvAlgo.Native, (3, 3, 3), (2, 2, 2), (1, 1, 1), (1, 1, 1),
                            (0, 0, 0), True, False)


def test_spconv_shim_batches_do_not_mix():
    from hi3d_b200.torch_backend import sparse_conv as sc

    rng = np.random.default_rng(9)
    xyz = np.argwhere(rng.random((10, 10, 10)) < 0.4).astype(np.int32)
    n = xyz.shape[0]
    idx = np.concatenate([np.concatenate([np.zeros((n, 1), np.int32), xyz], 1),
                          np.concatenate([np.ones((n, 1), np.int32), xyz], 1)])
    feats = rng.standard_normal((2 * n, 16)).astype(np.float16)
    conv = sc.SubMConv3d(16, 16, 3).to(DEV).half()
    both = conv(sc.SparseConvTensor(_t(feats), _t(idx), [10] * 3, 2)).features
    one = conv(sc.SparseConvTensor(_t(feats[:n]), _t(idx[:n]), [10] * 3, 1)).features
    assert torch.equal(both[:n], one)
