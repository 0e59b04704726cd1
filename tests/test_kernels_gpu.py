"""Row kernels (LayerNorm-modulate, RoPE + QK norm, gate/residual, GELU) vs the CPU oracle.

Tolerances are the reference's own (tests/test_mlx_kernels.py:27-60, tests/test_fast.py:14-32).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN, rel_l2

from hi3d_b200 import kernels
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("c", [1024, 2112, 256, 4096])
def test_layer_norm_modulate_matches_oracle(c):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((2, 50, c)) * 3 + 0.5).astype(np.float16)
    scale = (1 + 0.1 * rng.standard_normal((1, c))).astype(np.float16)
    shift = (0.1 * rng.standard_normal((1, c))).astype(np.float16)
    w, b = rng.standard_normal(c).astype(np.float32), rng.standard_normal(c).astype(np.float32)
    cases = (
        (dict(scale=scale, shift=shift), dict(scale=_t(scale), shift=_t(shift))),
        (dict(weight=w, bias=b), dict(weight=_t(w), bias=_t(b))),
        ({}, {}),
        (dict(weight=w, bias=b, scale=scale, shift=shift), dict(weight=_t(w), bias=_t(b), scale=_t(scale), shift=_t(shift))),
    )
    for ref_kw, kw in cases:
        ref = ops.layer_norm_modulate(x, 1e-6, **ref_kw)
        got = kernels.layer_norm_modulate(_t(x), 1e-6, **kw).cpu().numpy()
        equal = (ref == got).mean()
        assert equal > 0.999, equal  # the rest differ by one ulp (fp32 summation order)
        assert np.allclose(ref.astype(np.float32), got.astype(np.float32), atol=1e-2, rtol=1e-3)


def test_layer_norm_modulate_per_batch_and_bf16():
    rng = np.random.default_rng(6)
    c = 1024
    x = rng.standard_normal((2, 33, c)).astype(np.float32)
    scale = (1 + 0.1 * rng.standard_normal((2, c))).astype(np.float32)
    shift = (0.1 * rng.standard_normal((2, c))).astype(np.float32)
    got = kernels.layer_norm_modulate(_t(x, torch.float16), 1e-6, scale=_t(scale, torch.float16),
                                      shift=_t(shift, torch.float16)).cpu().numpy()
    for bb in range(2):
        ref = ops.layer_norm_modulate(x[bb].astype(np.float16), 1e-6, scale=scale[bb].astype(np.float16),
                                      shift=shift[bb].astype(np.float16))
        assert (ref == got[bb]).mean() > 0.999
    xb = _t(x, torch.bfloat16)
    got = kernels.layer_norm_modulate(xb, 1e-6).float().cpu().numpy()
    ref = ops.layer_norm32_f32(xb.float().cpu().numpy())
    assert np.allclose(got, ref, atol=2e-2, rtol=1e-2)


def test_layer_norm_modulate_golden_upstream():
    g = np.load(GOLDEN / "layernorm.npz")
    x = _t(g["x"])
    got = kernels.layer_norm_modulate(x, 1e-6, scale=_t((1 + g["scale"]).astype(np.float16)),
                                      shift=_t(g["shift"].astype(np.float16))).cpu().numpy()
    assert (got == g["modulated"]).mean() > 0.999
    got = kernels.layer_norm_modulate(x, 1e-6, weight=_t(g["w"]), bias=_t(g["b"])).cpu().numpy()
    assert (got == g["affine"]).mean() > 0.999


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 96, 128])
def test_qkv_rope_rms_float64_oracle(dtype, d):
    # odd sequence length and head count exercise partial groups (tests/test_fast.py:14-32)
    rng = np.random.default_rng(2026)
    b, n, h = 2, 37, 3
    raw = rng.normal(0, 2, (b * n, 3 * h * d)).astype(np.float32)
    phases = rng.uniform(-3, 3, (n, d // 2)).astype(np.float32)
    c, s = np.cos(phases), np.sin(phases)
    gq, gk = (rng.uniform(.5, 1.5, (h, d)).astype(np.float32) for _ in range(2))
    x = _t(raw, dtype)
    out = kernels.qkv_rope_rms(x, _t(c), _t(s), _t(gq), _t(gk), b, h, d)
    xin = x.float().cpu().numpy()
    yq, yk = ops.qkv_rope_rms_f64(xin, c, s, gq, gk, b, h, d)
    tol = 2.2e-4 if dtype == torch.float16 else 2e-3
    assert rel_l2(out[0].float().cpu().numpy(), yq) < tol
    assert rel_l2(out[1].float().cpu().numpy(), yk) < tol
    assert torch.equal(out[2].cpu(), x.view(b, n, 3, h, d)[:, :, 2].permute(0, 2, 1, 3).cpu())


def test_qkv_rope_rms_matches_composed_ops():
    """tests/test_mlx_kernels.py:27-45: fp16 tolerance 8e-3 vs the composed fp32 ops."""
    rng = np.random.default_rng(0)
    b, n, h, d = 2, 37, 3, 96
    x = (rng.standard_normal((b * n, 3 * h * d)) * 2).astype(np.float16)
    cos = rng.uniform(-1, 1, (n, d // 2)).astype(np.float32)
    sin = rng.uniform(-1, 1, (n, d // 2)).astype(np.float32)
    gq = rng.uniform(0.5, 1.5, (h, d)).astype(np.float32)
    gk = rng.uniform(0.5, 1.5, (h, d)).astype(np.float32)
    ref = ops.qkv_rope_rms(x, cos, sin, gq, gk, b, h, d)
    got = kernels.qkv_rope_rms(_t(x), _t(cos), _t(sin), _t(gq), _t(gk), b, h, d)
    for a, g in zip(ref, got):
        assert a.shape == tuple(g.shape)
        assert np.allclose(a.astype(np.float32), g.float().cpu().numpy(), atol=8e-3, rtol=8e-3)
    assert np.array_equal(ref[2], got[2].cpu().numpy())


def test_qkv_rope_rms_simd_rejects_bad_group():
    with pytest.raises(ValueError):
        kernels.qkv_rope_rms_simd(None, None, None, None, None, 1, 1, 64, group=12)


def test_gate_residual_bit_exact():
    rng = np.random.default_rng(8)
    x = rng.standard_normal((2, 70, 1024)).astype(np.float16)
    y = rng.standard_normal((2, 70, 1024)).astype(np.float16)
    gate = (0.3 * rng.standard_normal((1, 1024))).astype(np.float16)
    xt = _t(x)
    kernels.gate_residual(xt, _t(y), _t(gate))
    assert np.array_equal(xt.cpu().numpy(), ops.gate_residual(x, y, gate))
    gate2 = (0.3 * rng.standard_normal((2, 1024))).astype(np.float16)
    xt = _t(x)
    kernels.gate_residual(xt, _t(y), _t(gate2))
    for b in range(2):
        assert np.array_equal(xt[b].cpu().numpy(), ops.gate_residual(x[b], y[b], gate2[b]))
    xt = _t(x)
    kernels.gate_residual(xt, _t(y), None)
    assert np.array_equal(xt.cpu().numpy(), ops.gate_residual(x, y, None))


def test_gelu_tanh_matches_float64():
    """fp32 evaluation of the reference formula, rounded once.  ``1 + tanh(z)`` cancels for
    negative inputs, so the fp32 formula (here and in the reference) carries an absolute error
    of a few 1e-7 * |x| there; elsewhere the result is within one fp16 rounding of exact."""
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((300, 4096)) * 3).astype(np.float16)
    got = kernels.gelu_tanh(_t(x)).cpu().numpy().astype(np.float64)
    xd = x.astype(np.float64)
    exact = 0.5 * xd * (1 + np.tanh(np.sqrt(2 / np.pi) * (xd + 0.044715 * xd ** 3)))
    assert (np.abs(got - exact) <= 2.0 ** -11 * np.abs(exact) + 1e-6 * (1 + np.abs(xd))).all()
    ref = ops.gelu_tanh(x)
    assert (got.astype(np.float16) == ref).mean() > 0.95
