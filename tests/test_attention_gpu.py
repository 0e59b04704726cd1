"""tcgen05 flash attention vs exact float64 attention (and the reference's shim outputs).

The bound is the reference's (tests/test_mlx_kernels.py:163-179): relative RMS error < 3e-4
for fp16 (output rounding alone is ~2e-4), and ``bnhd`` bit-identical to ``bhnd``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN, rel_rms

from hi3d_b200 import attention
from hi3d_b200.torch_backend import attention as shim
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


SHAPES = [(2, 333, 333, False), (1, 77, 291, True), (2, 300, 129, True), (1, 5, 3, False), (2, 1000, 31, False),
          (1, 256, 1370, True), (1, 129, 257, False)]


@pytest.mark.parametrize("batch,nq,nk,shared", SHAPES)
@pytest.mark.parametrize("h,d", [(22, 96), (16, 64), (4, 128)])
def test_flash_attention_matches_float64(batch, nq, nk, shared, h, d):
    rng = np.random.default_rng(0)
    q = (rng.standard_normal((batch, h, nq, d)) * 2).astype(np.float16)
    k = (rng.standard_normal((1 if shared else batch, h, nk, d)) * 2).astype(np.float16)
    v = rng.standard_normal(k.shape).astype(np.float16)
    exact = ops.attention_f64(q, k, v, d ** -0.5)
    qt, kt, vt = _t(q, torch.float16), _t(k, torch.float16), _t(v, torch.float16)
    out = attention.flash_attention(qt, kt, vt, d ** -0.5)
    got = out.float().cpu().numpy()
    err = rel_rms(got, exact)
    assert err < 3e-4, err
    bnhd = attention.flash_attention(qt.transpose(1, 2).contiguous(), kt, vt, d ** -0.5, q_layout="bnhd")
    assert torch.equal(bnhd, out)


@pytest.mark.parametrize("d", [64, 96])
def test_flash_attention_bf16(d):
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 8, 700, d)).astype(np.float32) * 2
    k = rng.standard_normal((1, 8, 900, d)).astype(np.float32) * 2
    v = rng.standard_normal((1, 8, 900, d)).astype(np.float32)
    qt, kt, vt = (_t(a, torch.bfloat16) for a in (q, k, v))
    exact = ops.attention_f64(*(t.float().cpu().numpy() for t in (qt, kt, vt)), d ** -0.5)
    got = attention.flash_attention(qt, kt, vt, d ** -0.5).float().cpu().numpy()
    assert rel_rms(got, exact) < 4e-3


def test_varlen_packed_with_empty_and_ragged_sequences():
    rng = np.random.default_rng(2)
    h, d = 16, 64
    cu = np.array([0, 100, 100, 357, 700, 701], np.int32)
    qkv = (rng.standard_normal((701, 3, h, d)) * 2).astype(np.float16)
    exact = ops.attention_varlen(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, cu, d ** -0.5)
    t = _t(qkv, torch.float16)
    got = shim.flash_attn_varlen_qkvpacked_func(t, _t(cu, torch.int32), 343).float().cpu().numpy()
    assert rel_rms(got, exact) < 3e-4


def test_cross_attention_shared_keys_varlen():
    rng = np.random.default_rng(3)
    h, d, L = 16, 64, 1370
    cu = np.array([0, 500, 1200], np.int32)
    q = (rng.standard_normal((1200, h, d)) * 2).astype(np.float16)
    kv = (rng.standard_normal((L, 2, h, d)) * 2).astype(np.float16)
    exact = ops.attention_varlen(q, kv[:, 0], kv[:, 1], cu, None, d ** -0.5)
    kvt = _t(kv, torch.float16)
    got = attention.flash_attn_varlen(_t(q, torch.float16), kvt[:, 0], kvt[:, 1], _t(cu, torch.int32), None, 700,
                                      d ** -0.5).float().cpu().numpy()
    assert rel_rms(got, exact) < 3e-4


def test_shim_matches_reference_golden():
    g = np.load(GOLDEN / "attention.npz")
    qkv = _t(g["qkv"], torch.float16)
    got = shim.flash_attn_varlen_qkvpacked_func(qkv, _t(g["cu"], torch.int32), 90).float().cpu().numpy()
    assert rel_rms(got, g["self_out"]) < 2e-3  # fp16 input rounding vs the fp32 reference
    got = shim.flash_attn_varlen_kvpacked_func(_t(g["q"], torch.float16), _t(g["kv"], torch.float16),
                                               torch.tensor([0, 70]), torch.tensor([0, 30]), 70, 30)
    assert rel_rms(got.float().cpu().numpy(), g["cross_out"]) < 2e-3
    with pytest.raises(NotImplementedError):
        shim.flash_attn_varlen_qkvpacked_func(qkv, _t(g["cu"], torch.int32), 90, causal=True)


def test_long_sequence_sampled_rows_and_determinism():
    """32k keys: check 192 sampled query rows against float64, and bit-identical reruns."""
    rng = np.random.default_rng(4)
    h, d, n = 2, 64, 32768
    q = (rng.standard_normal((1, h, n, d)) * 2).astype(np.float16)
    k = (rng.standard_normal((1, h, n, d)) * 2).astype(np.float16)
    v = rng.standard_normal((1, h, n, d)).astype(np.float16)
    qt, kt, vt = (_t(a, torch.float16) for a in (q, k, v))
    out = attention.flash_attention(qt, kt, vt, d ** -0.5)
    again = attention.flash_attention(qt, kt, vt, d ** -0.5)
    assert torch.equal(out, again)
    rows = np.sort(rng.choice(n, 192, replace=False))
    exact = ops.attention_f64(q[:, :, rows], k, v, d ** -0.5)
    got = out[:, rows].float().cpu().numpy()
    assert rel_rms(got, exact) < 3e-4


@pytest.mark.parametrize("splits", [2, 3, 4, 7])
@pytest.mark.parametrize("h,d,dtype", [(16, 64, torch.float16), (4, 128, torch.bfloat16), (6, 96, torch.float16)])
def test_key_split_attention_matches_single_pass_and_float64(splits, h, d, dtype):
    """Key ranges on separate CTAs merged by log2-sum-exp weights: within the float64 bound and
    within output rounding of the single-pass kernel (dense, batch 2, keys not a multiple of the
    key block)."""
    rng = np.random.default_rng(splits + d)
    q = (rng.standard_normal((2, h, 300, d)) * 2).astype(np.float32)
    k = (rng.standard_normal((2, h, 1111, d)) * 2).astype(np.float32)
    v = rng.standard_normal((2, h, 1111, d)).astype(np.float32)
    qt, kt, vt = (_t(a, dtype) for a in (q, k, v))
    exact = ops.attention_f64(*(t.float().cpu().numpy() for t in (qt, kt, vt)), d ** -0.5)
    one = attention.flash_attention(qt, kt, vt, d ** -0.5, k_splits=1)
    got = attention.flash_attention(qt, kt, vt, d ** -0.5, k_splits=splits)
    tol = 3e-4 if dtype == torch.float16 else 4e-3
    assert rel_rms(got.float().cpu().numpy(), exact) < tol
    ulp = 2.0 ** (-10 if dtype == torch.float16 else -7)
    assert (got.float() - one.float()).abs().max().item() <= 2 * ulp * one.float().abs().max().item()


def test_key_split_varlen_with_short_and_empty_sequences():
    """More splits than some sequences have key blocks (those splits are empty) and an empty
    sequence: still exact to the float64 bound."""
    rng = np.random.default_rng(9)
    h, d = 16, 64
    cu = np.array([0, 100, 100, 357, 1700, 1701], np.int32)
    qkv = (rng.standard_normal((1701, 3, h, d)) * 2).astype(np.float16)
    exact = ops.attention_varlen(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, cu, d ** -0.5)
    t = _t(qkv, torch.float16)
    cut = _t(cu, torch.int32)
    got = attention.flash_attn_varlen(t[:, 0], t[:, 1], t[:, 2], cut, cut, 1343, d ** -0.5, k_splits=6)
    assert rel_rms(got.float().cpu().numpy(), exact) < 3e-4


def test_auto_splits_fill_waves():
    assert attention.auto_splits(2048, 256, 148) == 1   # cfg1 on one GPU: 13.8 waves already
    assert attention.auto_splits(256, 256, 148) == 1    # one eighth of the queries per GPU: the partial
    assert attention.auto_splits(512, 256, 148) == 1    # kernel's cost outweighs the wave tail
    assert attention.auto_splits(16, 256, 148) == 8     # a short grid over long keys
    assert attention.auto_splits(64, 512, 148) == 2
    assert attention.auto_splits(256, 3, 148) == 1      # too few key blocks to split
    assert attention.auto_splits(256, 11, 148) == 1     # cross-attention at 8 GPUs: CTA set-up dominates


def test_attention_parts_over_disjoint_key_sets_match_single_pass():
    """Keys split into three disjoint sets added one at a time (as the sharded block does) and
    merged: within output rounding of one pass over all keys, and within the float64 bound."""
    rng = np.random.default_rng(11)
    h, d = 8, 64
    q = (rng.standard_normal((1, 500, h, d)) * 2).astype(np.float16)      # token-major queries
    k = (rng.standard_normal((1, h, 3000, d)) * 2).astype(np.float16)
    v = rng.standard_normal((1, h, 3000, d)).astype(np.float16)
    qt, kt, vt = _t(q, torch.float16), _t(k, torch.float16), _t(v, torch.float16)
    one = attention.flash_attention(qt, kt, vt, d ** -0.5, q_layout="bnhd", k_splits=1)
    parts = attention.AttentionParts(qt, d ** -0.5, slots=8, q_layout="bnhd")
    for lo, hi in ((1000, 2000), (0, 1000), (2000, 3000)):
        parts.add(kt[:, :, lo:hi], vt[:, :, lo:hi], k_splits=2 if lo == 0 else 1)
    got = parts.merge()
    assert (got.float() - one.float()).abs().max().item() <= 2 * 2 ** -10 * one.float().abs().max().item()
    exact = ops.attention_f64(q.transpose(0, 2, 1, 3), k, v, d ** -0.5)
    assert rel_rms(got.float().cpu().numpy(), exact) < 3e-4  # both [1, Nq, H * D]


@pytest.mark.parametrize("h,d,dtype", [(8, 64, torch.float16), (4, 128, torch.bfloat16), (6, 96, torch.float16)])
def test_last_key_set_merged_in_its_epilogue_equals_partial_plus_merge(h, d, dtype):
    """hi3d_flash_attn_fwd_partial_merge (the last key set attended in one pass and folded with
    the earlier partials in its epilogue) is bit-identical to adding it as a partial and running
    the merge kernel, and within the float64 bound."""
    rng = np.random.default_rng(12 + d)
    q = (rng.standard_normal((1, 500, h, d)) * 2).astype(np.float32)
    k = (rng.standard_normal((1, h, 3000, d)) * 2).astype(np.float32)
    v = rng.standard_normal((1, h, 3000, d)).astype(np.float32)
    qt, kt, vt = _t(q, dtype), _t(k, dtype), _t(v, dtype)
    sets = ((1000, 2000, 1), (0, 1000, 2), (2000, 3000, 1))
    ref_parts = attention.AttentionParts(qt, d ** -0.5, slots=8, q_layout="bnhd")
    for lo, hi, s in sets:
        ref_parts.add(kt[:, :, lo:hi], vt[:, :, lo:hi], k_splits=s)
    want = ref_parts.merge()
    parts = attention.AttentionParts(qt, d ** -0.5, slots=8, q_layout="bnhd")
    for lo, hi, s in sets[:-1]:
        parts.add(kt[:, :, lo:hi], vt[:, :, lo:hi], k_splits=s)
    got = parts.add_final(kt[:, :, 2000:3000], vt[:, :, 2000:3000])
    assert torch.equal(got, want)
    exact = ops.attention_f64(*(t.float().cpu().numpy() for t in (qt.transpose(1, 2), kt, vt)), d ** -0.5)
    assert rel_rms(got.float().cpu().numpy(), exact) < (3e-4 if dtype == torch.float16 else 4e-3)
    # no earlier partials: the merged launch is a plain single pass
    solo = attention.AttentionParts(qt, d ** -0.5, slots=1, q_layout="bnhd").add_final(kt, vt)
    assert torch.equal(solo, attention.flash_attention(qt, kt, vt, d ** -0.5, q_layout="bnhd", k_splits=1))


def test_partial_merge_varlen_with_empty_key_ranges():
    """Varlen sequences whose last key range is empty take their rows from the earlier
    partials alone; an empty sequence stays untouched, as with the merge kernel."""
    import ctypes

    from hi3d_b200 import _lib

    rng = np.random.default_rng(13)
    h, d = 4, 64
    cu_q = np.array([0, 200, 200, 450], np.int32)
    cu_k1 = np.array([0, 300, 300, 700], np.int32)      # first key set: keys of every sequence
    cu_k2 = np.array([0, 0, 0, 250], np.int32)          # last key set: sequence 0 has none
    q = (rng.standard_normal((450, h, d)) * 2).astype(np.float16)
    k1, v1 = (rng.standard_normal((700, h, d)) * 2).astype(np.float16), rng.standard_normal((700, h, d)).astype(np.float16)
    k2, v2 = (rng.standard_normal((250, h, d)) * 2).astype(np.float16), rng.standard_normal((250, h, d)).astype(np.float16)
    tq, tk1, tv1, tk2, tv2 = (_t(a, torch.float16) for a in (q, k1, v1, k2, v2))
    cq, c1, c2 = (_t(a, torch.int32) for a in (cu_q, cu_k1, cu_k2))
    part_o = torch.empty((1, 450, h, d), dtype=torch.float32, device=DEV)
    part_lse = torch.empty((1, 450, h), dtype=torch.float32, device=DEV)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream

    def args(k, v, ck, out):
        return _lib.AttnArgs(q=tq.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(),
                             q_row=h * d, q_head=d, k_row=h * d, k_head=d, v_row=h * d, v_head=d, o_row=h * d,
                             o_head=d, cu_seqlens_q=cq.data_ptr(), cu_seqlens_k=ck.data_ptr(), nq=450,
                             nk=k.shape[0], max_seqlen_q=250, num_seqs=3, heads=h, head_dim=d, dtype=_lib.F16,
                             scale=d ** -0.5)

    out = torch.full((450, h, d), 7.0, dtype=torch.float16, device=DEV)
    a1 = args(tk1, tv1, c1, out)
    assert lib.hi3d_flash_attn_fwd_partial(ctypes.byref(a1), 1, 0, part_o.data_ptr(), part_lse.data_ptr(), 450,
                                           stream) == _lib.OK
    a2 = args(tk2, tv2, c2, out)
    assert lib.hi3d_flash_attn_fwd_partial_merge(ctypes.byref(a2), 1, part_o.data_ptr(), part_lse.data_ptr(), 450,
                                                 stream) == _lib.OK
    got = out.float().cpu().numpy()
    kk = [np.concatenate([k1[0:300], k2[0:0]]), None, np.concatenate([k1[300:700], k2[0:250]])]
    vv = [np.concatenate([v1[0:300], v2[0:0]]), None, np.concatenate([v1[300:700], v2[0:250]])]
    for i, (lo, hi) in enumerate(((0, 200), (200, 200), (200, 450))):
        if hi == lo:
            continue
        exact = ops.attention_varlen(q[lo:hi], kk[i], vv[i], [0, hi - lo], [0, kk[i].shape[0]], d ** -0.5)
        assert rel_rms(got[lo:hi], exact) < 3e-4
    assert _lib.device_status()["code"] == 0
