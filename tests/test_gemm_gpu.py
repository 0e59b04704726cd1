"""tcgen05 GEMM (16-bit and W8A8) vs CPU references.

W8A8 contract (the reference's tests/test_w8a8_inference.py:8-20): int32 accumulators exact,
output within rtol 5e-4 / atol 2e-6 of ``acc * sa * sw + bias`` in fp32; here additionally
bit-exact against the oracle, which evaluates the epilogue in the same order.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from hi3d_b200 import linear as lin
from hi3d_b200 import w8a8
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


def _ulp_diff(a16, b16):
    return np.abs(a16.view(np.int16).astype(np.int32) - b16.view(np.int16).astype(np.int32))


@pytest.mark.parametrize("m,n,k", [(300, 1024, 1024), (1, 17, 64), (129, 257, 200), (1000, 3072, 1024),
                                   (513, 1024, 4096), (77, 4096, 1024)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_linear_store_matches_fp32(m, n, k, dtype):
    rng = np.random.default_rng(m + n + k)
    x = _t(rng.standard_normal((m, k)).astype(np.float32), dtype)
    w = _t((rng.standard_normal((n, k)) * 0.02).astype(np.float32), dtype)
    b = _t((rng.standard_normal(n) * 0.02).astype(np.float32), dtype)
    got = lin.linear(x, w, b)
    ref = (x.float() @ w.float().t() + b.float()).to(dtype)
    g, r = got.float().cpu().numpy(), ref.float().cpu().numpy()
    scale = np.abs(r).max()
    tol = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    assert np.abs(g - r).max() <= tol * scale
    assert (got.cpu() == ref.cpu()).float().mean() > 0.97


def test_linear_gelu_and_residual_epilogues():
    rng = np.random.default_rng(1)
    m, n, k = 700, 1024, 1024
    x = _t(rng.standard_normal((m, k)).astype(np.float16))
    w = _t((rng.standard_normal((n, k)) * 0.02).astype(np.float16))
    b = _t((rng.standard_normal(n) * 0.02).astype(np.float16))
    y = lin.linear(x, w, b).cpu().numpy()  # store path, already validated above
    g = lin.linear(x, w, b, epilogue="gelu").cpu().numpy()
    assert (g == ops.gelu_tanh(y)).mean() > 0.95 and _ulp_diff(g, ops.gelu_tanh(y)).max() <= 8
    res0 = rng.standard_normal((2, m // 2, n)).astype(np.float16)
    gate = (0.5 * rng.standard_normal((2, n))).astype(np.float16)
    res = _t(res0)
    lin.linear(x.view(2, m // 2, k), w, b, epilogue="residual", residual=res, gate=_t(gate))
    want = np.stack([ops.gate_residual(res0[i], y.reshape(2, m // 2, n)[i], gate[i]) for i in range(2)])
    assert np.array_equal(res.cpu().numpy(), want)
    res = _t(res0)
    lin.linear(x.view(2, m // 2, k), w, b, epilogue="residual", residual=res)
    assert np.array_equal(res.cpu().numpy(), ops.gate_residual(res0, y.reshape(2, m // 2, n), None))


@pytest.mark.parametrize("rows,k", [(20003, 1024), (8195, 4096), (3001, 2112)])
def test_quantizer_bit_exact_many_tiles(rows, k):
    """Enough rows that every CTA of the tiled quantiser runs several tiles (both tile buffers
    refilled, the three row-maximum slots rotating) and the last tile is partial."""
    rng = np.random.default_rng(rows)
    x = (rng.standard_normal((rows, k)) * rng.uniform(0.1, 10, (rows, 1))).astype(np.float16)
    q, s = w8a8.quantize_activation(_t(x))
    q_ref, s_ref = ops.quantize_activation(x)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("k", [64, 1024, 2112, 4096, 8448])
def test_quantizer_bit_exact(k):
    rng = np.random.default_rng(k)
    x = (rng.standard_normal((37, k)) * rng.uniform(0.1, 10, (37, 1))).astype(np.float16)
    q, s = w8a8.quantize_activation(_t(x))
    q_ref, s_ref = ops.quantize_activation(x)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    q, s = w8a8.quantize_activation(_t(x), rotate=False)
    xf = x.astype(np.float32)
    s_ref = (np.maximum(np.abs(xf).max(-1), np.float32(1e-8)) / np.float32(127)).astype(np.float32)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), np.clip(np.rint(xf / s_ref[:, None]), -127, 127).astype(np.int8))


@pytest.mark.parametrize("m,n,k", [(3, 17, 64), (65, 131, 2112), (7, 33, 8448), (300, 3072, 1024),
                                   (1024, 4096, 4096), (4096, 1024, 4096)])
def test_int32_accumulators_bit_exact(m, n, k):
    rng = np.random.default_rng(m * 7 + n)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    w = rng.integers(-127, 128, (n, k), dtype=np.int8)
    acc = w8a8.gemm_accumulators(_t(a), _t(w)).cpu().numpy()
    exact = (a.astype(np.float64) @ w.astype(np.float64).T).astype(np.int64)  # exact: |sum| < 2^53
    assert np.array_equal(acc.astype(np.int64), exact)


@pytest.mark.parametrize("rows,columns,width", [(3, 17, 64), (65, 131, 2112), (7, 33, 8448)])
def test_integer_projection_matches_reference_contract(rows, columns, width):
    """tests/test_w8a8_inference.py:8-20 of the reference, on the B200 kernels."""
    rng = np.random.default_rng(7)
    x = rng.normal(size=(rows, width)).astype(np.float16)
    w = rng.integers(-127, 128, size=(columns, width), dtype=np.int8)
    sw = rng.uniform(.0001, .001, columns).astype(np.float32)
    bias = rng.normal(0, .01, columns).astype(np.float16)
    a, sa = w8a8.quantize_activation(_t(x))
    integer = a.cpu().numpy().astype(np.int64) @ w.astype(np.int64).T
    expected = integer.astype(np.float32) * sa.cpu().numpy()[:, None] * sw[None, :] + bias.astype(np.float32)
    result = w8a8.linear(_t(x), _t(w), _t(sw), _t(bias)).cpu().numpy().astype(np.float32)
    assert np.isfinite(result).all()
    np.testing.assert_allclose(result, expected, rtol=5e-4, atol=2e-6)
    assert np.array_equal(result.astype(np.float16), expected.astype(np.float16))  # same rounding points


def test_weight_quantization_matches_oracle():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((3072, 1024)) * 0.02).astype(np.float16)
    q, s = w8a8.quantize_weight(_t(w))
    q_ref, s_ref = ops.quantize_weight(w)
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)


def test_w8a8_projection_close_to_fp16():
    """The rotated int8 projection of N(0,1) activations through N(0, 0.02) weights stays
    within int8 quantisation error of the fp16 projection."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2048, 1024)).astype(np.float16)
    w = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float16)
    b = (rng.standard_normal(1024) * 0.02).astype(np.float16)
    qw, sw = w8a8.quantize_weight(_t(w))
    y8 = w8a8.linear(_t(x), qw, sw, _t(b)).float().cpu().numpy()
    y16 = (x.astype(np.float32) @ w.astype(np.float32).T + b.astype(np.float32))
    err = np.linalg.norm(y8 - y16) / np.linalg.norm(y16)
    assert err < 2e-2, err


def _rope_inputs(rng, batch, n, heads, k_dim, dtype):
    d = 64
    x = _t(rng.standard_normal((batch * n, k_dim)).astype(np.float32), dtype)
    w = _t((rng.standard_normal((3 * heads * d, k_dim)) * 0.05).astype(np.float32), dtype)
    b = _t((rng.standard_normal(3 * heads * d) * 0.1).astype(np.float32), dtype)
    ang = rng.uniform(0, 6.3, (n, d // 2)).astype(np.float32)
    cos, sin = _t(np.cos(ang)), _t(np.sin(ang))
    gq = _t(rng.uniform(0.5, 1.5, (heads, d)).astype(np.float32))
    gk = _t(rng.uniform(0.5, 1.5, (heads, d)).astype(np.float32))
    return x, w, b, cos, sin, gq, gk


@pytest.mark.parametrize("batch,n,heads,k_dim", [(1, 1000, 16, 1024), (2, 300, 4, 256), (3, 129, 8, 512)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("token_major", [False, True])
def test_linear_qkv_rope_matches_projection_then_rope(batch, n, heads, k_dim, dtype, token_major):
    """Fused QKV projection + RoPE + QK norm vs the unfused pair (linear then qkv_rope_rms) and the
    float64 rotation oracle: v bit-exact (both are the rounded projection), q/k within the rope
    kernel's own float64 bound."""
    from hi3d_b200 import kernels
    from conftest import rel_l2

    rng = np.random.default_rng(n + heads)
    x, w, b, cos, sin, gq, gk = _rope_inputs(rng, batch, n, heads, k_dim, dtype)
    q, k, v = lin.linear_qkv_rope(x, w, b, cos, sin, gq, gk, batch, heads, 64, token_major)
    qkv = lin.linear(x, w, b)
    q0, k0, v0 = kernels.qkv_rope_rms(qkv, cos, sin, gq, gk, batch, heads, 64, token_major=token_major)
    assert torch.equal(v, v0)
    qf, kf = ops.qkv_rope_rms_f64(qkv.float().cpu().numpy(), cos.cpu().numpy(), sin.cpu().numpy(),
                                  gq.cpu().numpy(), gk.cpu().numpy(), batch, heads, 64)
    perm = (0, 2, 1, 3) if token_major else (0, 1, 2, 3)
    tol = 2.2e-4 if dtype == torch.float16 else 2e-3
    for got, ref, unfused in ((q, qf, q0), (k, kf, k0)):
        g = got.permute(*perm).float().cpu().numpy()
        assert rel_l2(g, ref) < tol
        assert (got == unfused).float().mean() > 0.98


def test_w8a8_linear_qkv_rope_matches_projection_then_rope():
    from hi3d_b200 import kernels

    rng = np.random.default_rng(7)
    batch, n, heads, k_dim = 2, 200, 4, 512
    x, w, b, cos, sin, gq, gk = _rope_inputs(rng, batch, n, heads, k_dim, torch.float16)
    wq, sw = w8a8.quantize_weight(w)
    q, k, v = w8a8.linear_qkv_rope(x, wq, sw, b, cos, sin, gq, gk, batch, heads, 64)
    qkv = w8a8.linear(x, wq, sw, b)
    q0, k0, v0 = kernels.qkv_rope_rms(qkv, cos, sin, gq, gk, batch, heads, 64)
    assert torch.equal(v, v0)
    for got, ref in ((q, q0), (k, k0)):
        assert (got == ref).float().mean() > 0.98
        assert (got.float() - ref.float()).abs().max().item() <= 2 ** -8 * ref.float().abs().max().item()


def test_linear_qkv_rope_rejects_unsupported_layouts():
    x = torch.zeros(64, 256, device=DEV, dtype=torch.float16)
    w = torch.zeros(3 * 2 * 64, 256, device=DEV, dtype=torch.float16)   # heads * 64 = 128: not a tile multiple
    cos = torch.zeros(64, 32, device=DEV)
    g = torch.ones(2, 64, device=DEV)
    with pytest.raises(NotImplementedError):
        lin.linear_qkv_rope(x, w, None, cos, cos, g, g, 1, 2, 64)


@pytest.mark.parametrize("c", [64, 1024, 2112, 4096])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_layer_norm_quantize_bit_exact(c, dtype):
    """The fused LayerNorm(-modulate) + signed-H64 quantiser equals quantising the 16-bit
    LayerNorm output, codes and scales bit for bit (modulation per batch element, fp32 affine)."""
    from hi3d_b200 import kernels

    rng = np.random.default_rng(c)
    x = _t((rng.standard_normal((2, 150, c)) * 3 + 0.5).astype(np.float32), dtype)
    sc = _t((1 + 0.2 * rng.standard_normal((2, c))).astype(np.float32), dtype)
    sh = _t((0.1 * rng.standard_normal((2, c))).astype(np.float32), dtype)
    w = _t(rng.uniform(0.5, 1.5, c).astype(np.float32))
    b = _t(rng.normal(0, 0.1, c).astype(np.float32))
    for kw in (dict(scale=sc, shift=sh), dict(weight=w, bias=b), {}):
        fused = w8a8.layer_norm_quantize(x, 1e-6, **kw)
        q, s = w8a8.quantize_activation(kernels.layer_norm_modulate(x, 1e-6, **kw))
        assert torch.equal(fused.q, q) and torch.equal(fused.scale, s)
    # the projections accept the quantised rows in place of x
    wq, sw = w8a8.quantize_weight((torch.randn(256, c, device="cuda") * 0.02).half())
    bias = torch.zeros(256, dtype=torch.float16, device="cuda")
    h = kernels.layer_norm_modulate(x.half(), 1e-6, scale=sc.half(), shift=sh.half())
    fused = w8a8.layer_norm_quantize(x.half(), 1e-6, scale=sc.half(), shift=sh.half())
    assert torch.equal(w8a8.linear(fused, wq, sw, bias), w8a8.linear(h, wq, sw, bias))
    assert torch.equal(w8a8.linear(fused[1], wq, sw, bias), w8a8.linear(h[1], wq, sw, bias))
