"""The fp16 B200 block vs the fp32 CPU oracle (itself pinned to the upstream module).

Bound: relative L2 <= 2e-3 against the fp32 reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN, rel_l2

from hi3d_b200 import synthetic, transformer
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-3


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


def test_packed_block_matches_upstream_golden():
    g = np.load(GOLDEN / "block.npz")
    w = {k[2:]: g[k] for k in g.files if k.startswith("w:")}
    heads = 2
    lens = [int(n) for n in g["lens"]]
    cu = _t(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32))
    cos, sin = transformer.rope_tables(g["coords"][:, 1:], 64)
    wd = transformer.to_device(w, DEV)
    ck, cv = transformer.context_kv(wd, _t(g["ctx"], torch.float16), heads)
    y = transformer.block_forward_packed(wd, _t(g["x"], torch.float16), _t(g["mod"]), _t(cos), _t(sin), ck, cv,
                                         heads, cu, max(lens))
    assert rel_l2(y.float().cpu().numpy(), g["y"]) < TOL


def _config0(n=4096, c=1024, heads=16, L=1370, seed=0):
    coords = synthetic.shell_coords(n, 64, 24, 2, seed=seed)
    w = synthetic.block_weights(c, c, heads, seed=seed + 1)
    x = synthetic.features(n, c, seed=seed + 2)
    mod = synthetic.modulation(c, 0.6, seed=seed + 3).astype(np.float16)
    ctx = synthetic.features(L, c, seed=seed + 4)
    cos, sin = transformer.rope_tables(coords, c // heads)
    return coords, w, x, mod, ctx, cos, sin


def test_config0_block_matches_fp32_oracle():
    coords, w, x, mod, ctx, cos, sin = _config0()
    heads = 16
    wd = transformer.to_device(w, DEV)
    ck, cv = transformer.context_kv(wd, _t(ctx), heads)
    y = transformer.block_forward(wd, _t(x)[None], _t(mod), _t(cos), _t(sin), ck, cv, None, heads)
    ref = ops.block_forward_f32(w, x.astype(np.float32), mod, cos, sin, ctx, heads)
    assert rel_l2(y[0].float().cpu().numpy(), ref) < TOL


def test_block_with_strong_gates_and_update():
    """O(1) adaLN gates so every branch moves the output; also bound the error of the
    block's update (out - x) itself, which exposes any wrong branch."""
    coords, w, x, mod, ctx, cos, sin = _config0(n=2048, c=1024, heads=16, L=300, seed=30)
    rng = np.random.default_rng(31)
    w["modulation"] = rng.standard_normal((1, 6 * 1024)).astype(np.float32) * 0.5
    w["self_attn.q_rms_norm.gamma"] = rng.uniform(0.5, 1.5, (16, 64)).astype(np.float32)
    w["self_attn.k_rms_norm.gamma"] = rng.uniform(0.5, 1.5, (16, 64)).astype(np.float32)
    heads = 16
    wd = transformer.to_device(w, DEV)
    ck, cv = transformer.context_kv(wd, _t(ctx), heads)
    y = transformer.block_forward(wd, _t(x)[None], _t(mod), _t(cos), _t(sin), ck, cv, None, heads)[0]
    ref = ops.block_forward_f32(w, x.astype(np.float32), mod, cos, sin, ctx, heads)
    got = y.float().cpu().numpy()
    assert rel_l2(got, ref) < TOL
    xf = x.astype(np.float32)
    assert rel_l2(got - xf, ref - xf) < 5e-3


def test_cfg_batch_with_zero_condition_branch():
    coords, w, x, mod, ctx, cos, sin = _config0(n=1000, c=256, heads=4, L=77, seed=10)
    heads = 4
    wd = transformer.to_device(w, DEV)
    ck, cv = transformer.context_kv(wd, _t(ctx), heads)
    neg = transformer.negative_cross(wd)
    xb = _t(np.stack([x, x]))
    y = transformer.block_forward(wd, xb, _t(mod), _t(cos), _t(sin), ck, cv, neg, heads, n_pos=1)
    ref_pos = ops.block_forward_f32(w, x.astype(np.float32), mod, cos, sin, ctx, heads)
    ref_neg = ops.block_forward_f32(w, x.astype(np.float32), mod, cos, sin, np.zeros_like(ctx), heads)
    assert rel_l2(y[0].float().cpu().numpy(), ref_pos) < TOL
    assert rel_l2(y[1].float().cpu().numpy(), ref_neg) < TOL
    assert torch.equal(xb, _t(np.stack([x, x])))  # functional: input untouched


def test_two_block_stack():
    coords, w, x, mod, ctx, cos, sin = _config0(n=777, c=512, heads=8, L=100, seed=20)
    heads = 8
    w2 = synthetic.block_weights(512, 512, heads, seed=99)
    stack = transformer.BlockStack([transformer.to_device(w, DEV), transformer.to_device(w2, DEV)], heads)
    kvs = stack.prepare(_t(ctx))
    y = stack(_t(x)[None], _t(mod), _t(cos), _t(sin), kvs)
    ref = ops.block_forward_f32(w, x.astype(np.float32), mod, cos, sin, ctx, heads)
    ref = ops.block_forward_f32(w2, ref, mod, cos, sin, ctx, heads)
    assert rel_l2(y[0].float().cpu().numpy(), ref) < TOL


def test_w8a8_block_close_to_fp32_oracle():
    """cfg2 path: the six block projections through int8 (signed-H64 activations, rotated int8
    weights, exact int32 accumulation).  Bounded by int8 quantisation error."""
    coords, w, x, mod, ctx, cos, sin = _config0(n=2048, c=1024, heads=16, L=300, seed=40)
    rng = np.random.default_rng(41)
    w["modulation"] = rng.standard_normal((1, 6 * 1024)).astype(np.float32) * 0.5
    heads = 16
    wd = transformer.to_w8a8(transformer.to_device(w, DEV))
    assert wd["self_attn.to_qkv.weight"].dtype == torch.int8
    ck, cv = transformer.context_kv(wd, _t(ctx), heads)
    y = transformer.block_forward(wd, _t(x)[None], _t(mod), _t(cos), _t(sin), ck, cv, None, heads)[0]
    ref = ops.block_forward_f32(w, x.astype(np.float32), mod, cos, sin, ctx, heads)
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < 1e-2
    xf = x.astype(np.float32)
    assert rel_l2(got - xf, ref - xf) < 5e-2
