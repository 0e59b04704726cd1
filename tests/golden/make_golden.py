"""Generate the golden fixtures in this directory from the reference's own code.

Run once in a container that has the reference source tree (read-only); name its
root in ``HI3D_REFERENCE`` (required):

    HI3D_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports the reference's runnable CPU code only:

* the upstream PyTorch modules (``sparc3d.nn``) with the reference's torch shims for
  ``flash_attn`` and ``spconv`` registered (src/hi3d_mac/torch_backend/__init__.py:34-64);
* the pure-numpy helpers of the MLX path (``neighbour_table``, ``downsample_structure``,
  ``rope_tables``, ``signs``), imported behind a stub ``mlx.core`` whose ``array`` is
  ``numpy.asarray`` (MLX itself is not installable here).

Every fixture is a small ``.npz`` (inputs and the reference's outputs).  The GPU box
never runs this script; tests read the committed fixtures.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if not os.environ.get("HI3D_REFERENCE"):
    raise SystemExit("set HI3D_REFERENCE to the root of the reference source tree")
REF = Path(os.environ["HI3D_REFERENCE"]) / "src"
sys.path.insert(0, str(HERE.parents[1] / "hi3dv1.0-mlx_b200"))


def _stub_mlx() -> None:
    mlx = types.ModuleType("mlx")
    core = types.ModuleType("mlx.core")
    core.array = np.asarray
    for n in ("float16", "float32", "int32", "int8"):
        setattr(core, n, getattr(np, n))
    core.bfloat16 = np.float32
    core.Dtype = object
    mlx.core = core
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = core


def main() -> None:
    sys.path.insert(0, str(REF))
    _stub_mlx()
    from hi3d_mac.torch_backend import _register_flash_attn, _register_spconv

    _register_spconv()
    _register_flash_attn()
    import torch

    from hi3d_mac.mlx_backend import sparse as ref_sparse
    from hi3d_mac.mlx_backend import transformer as ref_tf
    from hi3d_mac.torch_backend import attention as ref_attn
    from hi3d_mac.torch_backend import sparse_conv as ref_conv
    from sparc3d.nn.norm import LayerNorm32
    from sparc3d.nn.rope import RotaryPositionEmbedder
    from sparc3d.nn.sparse.attention.modules import SparseMultiHeadRMSNorm
    from sparc3d.nn.sparse.basic import SparseTensor
    from sparc3d.nn.sparse.transformer.modulated import ModulatedSparseTransformerCrossBlock

    from hi3d_b200 import synthetic

    torch.manual_seed(0)
    rng = np.random.default_rng(2026)

    # ---- rope tables and rope + qk-norm (fp32, upstream modules)
    ca = rng.integers(0, 60, (50, 3)).astype(np.int32)
    cb = rng.integers(0, 128, (50, 3)).astype(np.int32)
    out = {"coords_a": ca, "coords_b": cb}
    for tag, c in (("a", ca), ("b", cb)):
        for d in (64, 96):
            cos, sin = ref_tf.rope_tables(c, d)
            out[f"cos_{tag}{d}"], out[f"sin_{tag}{d}"] = np.asarray(cos), np.asarray(sin)
    h, d = 3, 64
    qkv = (rng.standard_normal((50, 3 * h * d)) * 2).astype(np.float32)
    gq = rng.uniform(0.5, 1.5, (h, d)).astype(np.float32)
    gk = rng.uniform(0.5, 1.5, (h, d)).astype(np.float32)
    rope = RotaryPositionEmbedder(d)
    t = torch.from_numpy(qkv).reshape(50, 3, h, d)
    q, k = rope(t[:, 0], t[:, 1], torch.from_numpy(cb.astype(np.int64)))
    nq, nk = SparseMultiHeadRMSNorm(d, h), SparseMultiHeadRMSNorm(d, h)
    nq.gamma.data = torch.from_numpy(gq)
    nk.gamma.data = torch.from_numpy(gk)
    out.update(qkv=qkv, gq=gq, gk=gk, q_ref=nq(q).detach().numpy(), k_ref=nk(k).detach().numpy())
    np.savez_compressed(HERE / "rope.npz", **out)

    # ---- LayerNorm32 (+affine) and the upstream fp16 adaLN modulation
    c = 512
    x = (rng.standard_normal((80, c)) * 3 + 0.5).astype(np.float16)
    scale = (0.1 * rng.standard_normal((1, c))).astype(np.float32)
    shift = (0.1 * rng.standard_normal((1, c))).astype(np.float32)
    w, b = rng.standard_normal(c).astype(np.float32), rng.standard_normal(c).astype(np.float32)
    coords = np.concatenate([np.zeros((80, 1), np.int32), rng.integers(0, 64, (80, 3)).astype(np.int32)], 1)
    st = SparseTensor(torch.from_numpy(x), torch.from_numpy(coords))
    ln = LayerNorm32(c, elementwise_affine=False, eps=1e-6)
    lna = LayerNorm32(c, elementwise_affine=True, eps=1e-6)
    lna.weight.data, lna.bias.data = torch.from_numpy(w), torch.from_numpy(b)
    hs = st.replace(ln(st.feats))
    mod = hs * (1 + torch.from_numpy(scale)) + torch.from_numpy(shift)  # modulated.py:57-58
    np.savez_compressed(HERE / "layernorm.npz", x=x, scale=scale, shift=shift, w=w, b=b,
                        plain=ln(st.feats).detach().numpy(), affine=lna(st.feats).detach().numpy(),
                        modulated=mod.feats.detach().numpy())

    # ---- attention through the reference's flash_attn shim (fp32)
    g = torch.Generator().manual_seed(0)
    qkv_t = torch.randn(150, 3, 2, 64, generator=g)
    cu = torch.tensor([0, 60, 150], dtype=torch.int32)
    self_out = ref_attn.flash_attn_varlen_qkvpacked_func(qkv_t, cu, 90)
    qc = torch.randn(70, 2, 64, generator=g)
    kv = torch.randn(30, 2, 2, 64, generator=g)
    cross_out = ref_attn.flash_attn_varlen_kvpacked_func(qc, kv, torch.tensor([0, 70]), torch.tensor([0, 30]), 70, 30)
    np.savez_compressed(HERE / "attention.npz", qkv=qkv_t.numpy(), cu=cu.numpy(), self_out=self_out.numpy(),
                        q=qc.numpy(), kv=kv.numpy(), cross_out=cross_out.numpy())

    # ---- sparse structure (MLX numpy helpers) and submanifold conv (spconv shim, fp64)
    occ = rng.random((12, 12, 12)) < 0.3
    xyz = np.argwhere(occ).astype(np.int32)
    xyz = xyz[rng.permutation(xyz.shape[0])]
    table = ref_sparse.neighbour_table(xyz)
    low, inverse, counts = ref_sparse.downsample_structure(xyz)
    feats = rng.standard_normal((xyz.shape[0], 5))
    conv = ref_conv.SubMConv3d(5, 7, 3, bias=True).double()
    torch.nn.init.normal_(conv.bias)
    ind = torch.from_numpy(np.concatenate([np.zeros((xyz.shape[0], 1), np.int32), xyz], 1))
    conv_out = conv(ref_conv.SparseConvTensor(torch.from_numpy(feats), ind, [12, 12, 12], 1)).features
    np.savez_compressed(HERE / "sparse.npz", coords=xyz, table=table, low=low, inverse=inverse, counts=counts,
                        feats=feats, weight=conv.weight.detach().numpy(), bias=conv.bias.detach().numpy(),
                        conv_out=conv_out.detach().numpy())

    # ---- one upstream block in fp32 (two packed objects, shared condition)
    c, cc, heads, L = 128, 96, 2, 20
    lens = [70, 50]
    wts = synthetic.block_weights(c, cc, heads, seed=7, gamma_random=True)
    blk = ModulatedSparseTransformerCrossBlock(c, cc, heads).float()
    sd = {k: torch.from_numpy(v.astype(np.float32)) for k, v in wts.items()}
    sd = {("self_attn.q_rms_norm.gamma" if k == "self_attn.q_rms_norm.gamma" else k): v for k, v in sd.items()}
    missing, unexpected = blk.load_state_dict(sd, strict=False)
    assert not unexpected and not [m for m in missing if "rope" not in m], (missing, unexpected)
    coords_b = [synthetic.shell_coords(n, 32, 10, 2, seed=11 + i) for i, n in enumerate(lens)]
    cb_all = np.concatenate([np.concatenate([np.full((n, 1), i, np.int32), co], 1)
                             for i, (n, co) in enumerate(zip(lens, coords_b))])
    xb = synthetic.features(sum(lens), c, seed=12, dtype=np.float32)
    modb = synthetic.modulation(c, 0.37, seed=13).reshape(1, 6 * c)
    ctx = synthetic.features(L, cc, seed=14, dtype=np.float32)
    with torch.no_grad():
        yb = blk(SparseTensor(torch.from_numpy(xb), torch.from_numpy(cb_all)), torch.from_numpy(modb),
                 torch.from_numpy(np.stack([ctx] * len(lens)))).feats.numpy()
    np.savez_compressed(HERE / "block.npz", x=xb, coords=cb_all, mod=modb, ctx=ctx, lens=np.array(lens), y=yb,
                        **{f"w:{k}": v for k, v in wts.items()})

    # ---- the whole upstream transformer in fp32 (one object, 2 blocks, one I/O stage)
    from sparc3d.models.transformers.config import Sparc3DTransformerConfig
    from sparc3d.models.transformers.sparc3d_transformer import Sparc3DTransformer

    c, cc, heads, nblk, io, L = 128, 96, 2, 2, 64, 24
    cfg = Sparc3DTransformerConfig(model_channels=c, cond_channels=cc, num_blocks=nblk, num_heads=heads,
                                   io_block_channels=(io,), use_fp16=False)
    model = Sparc3DTransformer(cfg).float()
    wts = synthetic.model_weights(c, cc, heads, nblk, io_channels=io, seed=21, std=None)
    missing, unexpected = model.load_state_dict({k: torch.from_numpy(v.astype(np.float32)) for k, v in wts.items()},
                                                strict=False)
    assert not unexpected and not [m for m in missing if "rope" not in m], (missing, unexpected)
    fine = synthetic.shell_coords(1500, 32, 10, 2, seed=22)
    feats = synthetic.features(fine.shape[0], 32, seed=23, dtype=np.float32)
    cond = synthetic.features(L, cc, seed=24, dtype=np.float32)
    t = np.float32(0.43)
    ind = torch.from_numpy(np.concatenate([np.zeros((fine.shape[0], 1), np.int32), fine], 1))
    with torch.no_grad():
        vel = model(SparseTensor(torch.from_numpy(feats), ind), torch.tensor([np.float32(1000.0) * t]),
                    torch.from_numpy(cond)[None]).feats.numpy()
    # the weights are regenerated by the tests from the same call (seeded numpy); a checksum pins them
    checksum = np.float64(sum(float(np.abs(v.astype(np.float64)).sum()) for v in wts.values()))
    np.savez_compressed(HERE / "forward.npz", coords=fine, feats=feats, cond=cond, t=t, velocity=vel,
                        config=np.array([c, cc, heads, nblk, io, 21]), weight_checksum=checksum)

    # ---- the upstream flow-matching schedule and guidance (sparc3d.schedulers)
    from sparc3d.schedulers.flow_match_heun import FlowMatchHeunScheduler
    from sparc3d.schedulers.schedule import effective_guidance_scale

    sched = {}
    for steps, tokens in ((25, 34316), (12, 4000), (25, 1000), (3, 1500), (40, 262144)):
        sch = FlowMatchHeunScheduler()
        hats = sch.set_timesteps(steps, num_tokens=tokens)
        sched[f"sigmas_{steps}_{tokens}"] = sch.sigmas.numpy()
        sched[f"hats_{steps}_{tokens}"] = hats.numpy()
    ts = np.array([1.2, 1.0, 0.99, 0.85, 0.7, 0.69999, 0.3], np.float32)
    sched["guidance_t"] = ts
    # the pipelines pass float32 model times: the tensor form compares and squares in float32
    sched["guidance"] = effective_guidance_scale(torch.from_numpy(ts)).numpy().astype(np.float64)
    np.savez_compressed(HERE / "schedule.npz", **sched)

    # ---- VAE decoder index structures: the MLX helpers (octree child table, serialization, windows)
    core = sys.modules["mlx.core"]
    core.take = np.take
    core.take_along_axis = np.take_along_axis
    core.eval = lambda *a, **k: None
    from hi3d_mac.mlx_backend import vae as ref_vae

    occ = rng.random((10, 10, 10)) < 0.35
    pc = np.argwhere(occ).astype(np.int32)
    pc = pc[rng.permutation(pc.shape[0])]
    ptable = ref_sparse.neighbour_table(pc)
    cmask = rng.random((pc.shape[0], 8)) < 0.4
    ctable, cparent, cslot = ref_sparse.child_neighbour_table(ptable, cmask)
    scoords = synthetic.shell_coords(1000, 40, 12, 3, seed=41)
    serial = ref_vae.serialization(scoords)
    vae_out = dict(parent_coords=pc, parent_table=ptable, child_mask=cmask, child_table=np.asarray(ctable),
                   child_parent=np.asarray(cparent), child_slot=np.asarray(cslot), serial_coords=scoords)
    for i, (perm, inverse) in enumerate(serial):
        gather, scatter = ref_vae.window_index(perm, inverse)
        vae_out.update({f"perm{i}": perm, f"inverse{i}": inverse, f"gather{i}": gather, f"scatter{i}": scatter})
    np.savez_compressed(HERE / "vae.npz", **vae_out)

    # ---- W8A8 sign tables of the signed H64 rotation
    from hi3d_mac.mlx_backend import w8a8 as ref_w8a8

    np.savez_compressed(HERE / "w8a8.npz", **{f"signs{k}": np.asarray(ref_w8a8.signs(k)) for k in (64, 1024, 2112, 4096)})
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
