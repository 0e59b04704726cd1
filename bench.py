"""Benchmark of the sparse-DiT refinement torso on B200 (BASELINE configs[1] by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extras]
                    [--workload stack|stack_w8a8|block|attention|attention262k|conv|forward|vae]

One step = one forward of the 24-block stack (C=1024, 16 heads x 64, GELU MLP 4x,
1370 condition tokens) over T=32,768 voxel tokens of one object in fp16, inputs
resident in HBM.  ``value`` is block tokens/s = blocks * T / step time (whole job,
max over ranks).  With N>1 GPUs (torchrun) the T tokens are split into N query
slices and every block all-gathers K/V over NCCL (strong scaling).

Beside the headline (outside its timed region) the default line carries the other BASELINE
configurations: ``cfg4_attention`` (262,144 bf16 tokens as 4 objects of 65,536, query-sharded
over the N GPUs), and at N=1 ``cfg2_w8a8`` (the W8A8 stack and its int8 GEMMs) and
``cfg5_conv`` (neighbour map, submanifold and stride-2 conv), each with its roofline fraction
and CPU baseline.  At N>1 it adds the per-phase breakdown of a step (maximum over ranks) and
``sharded_rel_l2``, the sharded stack's first two blocks against the same blocks on one GPU.

``--workload attention`` times the self-attention kernel alone at the same size
(T=32,768, 16x64 heads, fp16); ``--workload attention262k`` the high-resolution
config (cfg4), query-sharded over the GPUs.  Both report attention TFLOP/s
(4 * Nq * Nk * H * D per object).  ``--workload conv`` times the cfg5 submanifold
convolution; ``--workload forward`` the whole refinement transformer around the same stack;
``--workload vae`` the VAE decoder's kernels.

Rank 0 prints one JSON line.  ``--impl reference`` times the reference's CPU path instead, on
every host thread: the upstream PyTorch block with the reference's flash_attn shim, restated in
torch (oracle/torch_block.py, pinned to the upstream module) because the reference itself cannot
travel to the GPU box; one whole block of the stack per step.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "hi3dv1.0-mlx_b200"))

T_TOKENS = 32768
CHANNELS = 1024
HEADS = 16
COND = 1370
BLOCKS = 24
GRID, RADIUS, THICK = 64, 24.0, 3.0
# the released model's block: C = 2112, 22 heads x 96, condition 2917 x 2048
# (src/sparc3d/models/transformers/config.py:101-111)
REL_C, REL_HEADS, REL_CC, REL_L = 2112, 22, 2048, 2917
# whole-transformer workload: fine voxels on a shell in 128^3 (R=48 +-4) -> 34,316 low tokens
FWD_FINE, FWD_GRID, FWD_RADIUS, FWD_THICK, FWD_IO, FWD_T = 120000, 128, 48.0, 4.0, 256, 0.37


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _profile_traffic(name: str) -> float | None:
    """DRAM bytes per launch recorded from an ncu capture in profiles/<name>.md (or None)."""
    p = REPO / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None
        self.skip = 0

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: wait (at most 5 s) for its first sample, so that a
        # short timed region (a few hundred ms at 8 GPUs) is sampled too
        t0 = time.time()
        while time.time() - t0 < 5.0 and self.proc.poll() is None:
            if Path(self.file.name).stat().st_size > 0:
                break
            time.sleep(0.02)
        self.skip = len(Path(self.file.name).read_text().splitlines())  # samples taken before the region
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        lines = Path(self.file.name).read_text().splitlines()
        os.unlink(self.file.name)
        # the samples taken during the region; the one just before it when the region was shorter
        # than the sampling interval
        lines = lines[self.skip:] or lines[-1:]
        rows = [r.split(",") for r in lines if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- inputs


def make_inputs(seed: int = 0):
    from hi3d_b200 import synthetic, transformer

    coords = synthetic.shell_coords(T_TOKENS, GRID, RADIUS, THICK, seed=seed)
    cos, sin = transformer.rope_tables(coords, CHANNELS // HEADS)
    x = synthetic.features(T_TOKENS, CHANNELS, seed=seed + 1)
    mod = synthetic.modulation(CHANNELS, 0.5, seed=seed + 2).astype(np.float16)
    cond = synthetic.features(COND, CHANNELS, seed=seed + 3)
    return coords, cos, sin, x, mod, cond


def device_weights(device, seed: int = 100, blocks: int = BLOCKS, c: int = CHANNELS, cc: int = CHANNELS,
                   heads: int = HEADS) -> list[dict]:
    """``blocks`` blocks of N(0, 0.02) fp16 weights generated on the device (seeded): hidden
    width ``c``, condition width ``cc``, ``heads`` heads."""
    import torch

    from hi3d_b200.synthetic import BLOCK_LINEARS

    g = torch.Generator(device=device).manual_seed(seed)
    d = c // heads
    out = []
    for _ in range(blocks):
        w = {}
        for name, i_mult, o_mult in BLOCK_LINEARS:
            w[f"{name}.weight"] = (torch.randn((o_mult * c, i_mult * c), generator=g, device=device) * 0.02).half()
            w[f"{name}.bias"] = (torch.randn(o_mult * c, generator=g, device=device) * 0.02).half()
        w["cross_attn.to_kv.weight"] = (torch.randn((2 * c, cc), generator=g, device=device) * 0.02).half()
        w["cross_attn.to_kv.bias"] = (torch.randn(2 * c, generator=g, device=device) * 0.02).half()
        w["modulation"] = torch.randn((1, 6 * c), generator=g, device=device) / c ** 0.5
        w["norm2.weight"] = torch.ones(c, device=device)
        w["norm2.bias"] = torch.zeros(c, device=device)
        w["self_attn.q_rms_norm.gamma"] = torch.ones((heads, d), device=device)
        w["self_attn.k_rms_norm.gamma"] = torch.ones((heads, d), device=device)
        out.append(w)
    return out


# ----------------------------------------------------------------------------- configs
#
# One config dict per workload, used verbatim by both arms so that their lines describe the
# same workload.


def stack_config(workload: str, nblocks: int, world: int, transport: str = "nccl") -> dict:
    if workload == "stack_w8a8":
        name = (f"cfg2: W8A8 {BLOCKS}-block stack fwd (int8 signed-H64 activations, int8 rotated weights, int32 "
                f"accumulate, fp16 dequant), T={T_TOKENS}, C={CHANNELS}, {HEADS}x{CHANNELS // HEADS} heads, "
                f"{COND} cond tokens")
    else:
        name = (f"cfg1: {nblocks}-block sparse-DiT stack fwd, T={T_TOKENS} shell tokens in {GRID}^3, C={CHANNELS}, "
                f"{HEADS}x{CHANNELS // HEADS} heads, {COND} cond tokens, fp16")
    if transport == "auto":
        import torch

        from hi3d_b200.dist import auto_transport

        transport = auto_transport(world, torch.device("cuda", 0) if torch.cuda.is_available() else None)
    kv = {"nccl": "NCCL all-gather", "peer": "QKV epilogue stores into peers' symmetric buffers",
          "multicast": "QKV epilogue multimem stores into every GPU's symmetric buffer"}[transport]
    return {"workload": name, "blocks": nblocks, "tokens": T_TOKENS,
            "parallelism": f"query-sharded x{world}, K/V by {kv}" if world > 1 else "none",
            "l2": "inputs larger than L2 (705 MB of weights + activations per step)"}


def attention_config(big: bool, world: int) -> dict:
    d = CHANNELS // HEADS
    if big:
        return {"workload": f"cfg4: self-attention, 4 objects x 65536 tokens varlen, {HEADS}x{d} heads, bf16, K/V "
                            f"shards exchanged between the ranks of each object",
                "tokens": 4 * 65536, "parallelism": f"query-sharded x{world}" if world > 1 else "none",
                "l2": "inputs larger than L2"}
    return {"workload": f"cfg1: self-attention, T={T_TOKENS}, {HEADS}x{d} heads, fp16", "tokens": T_TOKENS,
            "parallelism": f"query-sharded x{world}" if world > 1 else "none", "l2": "inputs larger than L2"}


CONV_N, CONV_C = 200_000, 256


def conv_config() -> dict:
    return {"workload": f"cfg5: submanifold 3x3x3 conv, {CONV_N} shell voxels in 128^3, {CONV_C}->{CONV_C} channels, "
                        f"fp16", "l2": "inputs larger than L2 (102 MB features + 102 MB output)"}


# ----------------------------------------------------------------------------- CPU baseline
#
# The reference's CPU path for this hot path is its upstream PyTorch block with the reference's
# torch shims (fp32; attention by SDPA over bounded query blocks).  The reference itself cannot
# travel to the GPU box; oracle/torch_block.py restates that path in torch and is pinned to the
# upstream module's output (tests/test_oracle_golden.py), so the CPU arm times the restatement,
# on every host thread the process may use.

_CPU_CACHE: dict = {}


def cpu_threads() -> int:
    """Use every host thread this process may run on (torchrun sets OMP_NUM_THREADS=1)."""
    import torch

    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return n


def _cpu_block_inputs(seed: int = 0, released: bool = False):
    from hi3d_b200 import synthetic, transformer
    from oracle import torch_block

    key = ("block", released)
    if key not in _CPU_CACHE:
        if released:
            coords = synthetic.shell_coords(T_TOKENS, GRID, RADIUS, THICK, seed=seed)
            cos, sin = transformer.rope_tables(coords, REL_C // REL_HEADS)
            x = synthetic.features(T_TOKENS, REL_C, seed=seed + 1)
            mod = synthetic.modulation(REL_C, 0.5, seed=seed + 2).astype(np.float16)
            cond = synthetic.features(REL_L, REL_CC, seed=seed + 3)
            w = synthetic.block_weights(REL_C, REL_CC, REL_HEADS, seed=seed + 5)
        else:
            coords, cos, sin, x, mod, cond = make_inputs(seed)
            w = synthetic.block_weights(CHANNELS, CHANNELS, HEADS, seed=seed + 5)
        _CPU_CACHE[key] = (torch_block.weights_f32(w), x, mod, cos, sin, cond)
    return _CPU_CACHE[key]


def cpu_block_seconds(rows: int | None = None, released: bool = False) -> float:
    """Wall seconds of one whole fp32 block of the reference's CPU path over the first ``rows``
    tokens (all T by default); ``released``: at the released model's shape."""
    from oracle import torch_block

    w, x, mod, cos, sin, cond = _cpu_block_inputs(released=released)
    r = slice(0, rows or x.shape[0])
    t0 = time.perf_counter()
    torch_block.block_forward(w, x[r], mod, cos[r], sin[r], cond, REL_HEADS if released else HEADS)
    return time.perf_counter() - t0


def cpu_attention_tflops(big: bool, sample: int = 512) -> tuple[float, str]:
    """The reference's shim attention (fp32 SDPA, torch_backend/attention.py:20-38) of ``sample``
    query rows against one whole object, scaled to TFLOP/s with the GPU arm's 4 Nq Nk H D count."""
    import torch

    from oracle import torch_block

    per = 65536 if big else T_TOKENS
    d = CHANNELS // HEADS
    if ("attn", big) not in _CPU_CACHE:
        g = torch.Generator().manual_seed(7)
        _CPU_CACHE[("attn", big)] = tuple(torch.randn((n, HEADS, d), generator=g) for n in (sample, per, per))
    q, k, v = _CPU_CACHE[("attn", big)]
    t0 = time.perf_counter()
    torch_block.attend(q, k, v, d ** -0.5)
    secs = time.perf_counter() - t0
    return 4.0 * sample * per * HEADS * d / secs / 1e12, (f"{sample} query rows x {per} keys x {HEADS} heads, fp32 "
                                                          f"SDPA (the reference's flash_attn shim)")


def forward_inputs():
    from hi3d_b200 import synthetic

    if "fwd" not in _CPU_CACHE:
        coords = synthetic.shell_coords(FWD_FINE, FWD_GRID, FWD_RADIUS, FWD_THICK, seed=1)
        feats = synthetic.features(coords.shape[0], 32, seed=4, dtype=np.float32)
        cond = synthetic.features(COND, CHANNELS, seed=5, dtype=np.float32)
        _CPU_CACHE["fwd"] = (coords, feats, cond)
    return _CPU_CACHE["fwd"]


def cpu_forward_seconds() -> tuple[float, float, str]:
    """One fp32 CPU forward of the whole transformer: the embedding and I/O stages in full at the
    workload size (numpy oracle port), plus one whole block of the reference's CPU path on the
    low-level tokens whose time counts 24 times (the 24 blocks have one shape).  Returns
    ``(estimated forward seconds, wall seconds spent, description)``."""
    from hi3d_b200 import synthetic
    from oracle import ops, torch_block

    t_wall = time.perf_counter()
    coords, feats, cond = forward_inputs()
    w = synthetic.model_weights(CHANNELS, CHANNELS, HEADS, 1, io_channels=FWD_IO, seed=3)
    io_only = {k: v for k, v in w.items() if not k.startswith("blocks.")}
    t0 = time.perf_counter()
    ops.forward_f32(io_only, feats, coords, FWD_T, cond, HEADS)
    io_s = time.perf_counter() - t0
    low, _, _ = ops.downsample_structure(coords)
    cos, sin = ops.rope_tables(low, CHANNELS // HEADS)
    x = synthetic.features(low.shape[0], CHANNELS, seed=6, dtype=np.float32)
    mod = synthetic.modulation(CHANNELS, FWD_T, seed=7)
    bw = torch_block.weights_f32({k[len("blocks.0."):]: v for k, v in w.items() if k.startswith("blocks.0.")})
    t0 = time.perf_counter()
    torch_block.block_forward(bw, x, mod, cos, sin, cond, HEADS)
    blk_s = time.perf_counter() - t0
    desc = (f"whole transformer fp32: embedding + I/O stages in full on {coords.shape[0]} fine voxels (numpy oracle "
            f"port, {io_s:.1f} s) plus one whole block of the reference's CPU path (torch restatement) on "
            f"{low.shape[0]} low tokens ({blk_s:.1f} s), counted {BLOCKS} times")
    return io_s + BLOCKS * blk_s, time.perf_counter() - t_wall, desc


def cpu_conv_tflops(sample: int = 20000) -> tuple[float, str]:
    """fp32 numpy gather-GEMM of ``sample`` output rows of the cfg5 convolution (TFLOP/s over the
    present neighbour pairs, as the GPU arm counts them)."""
    from hi3d_b200 import synthetic
    from oracle import ops

    if "conv" not in _CPU_CACHE:
        n, c = CONV_N, CONV_C
        coords = synthetic.shell_coords(n, 128, 48, 4, seed=5)
        rng = np.random.default_rng(3)
        table = ops.neighbour_table(coords)[:sample]
        x = np.concatenate([rng.standard_normal((n, c)).astype(np.float32), np.zeros((1, c), np.float32)])
        wt = (rng.standard_normal((27, c, c)) * 0.02).astype(np.float32)
        _CPU_CACHE["conv"] = (table, x, wt, n)
    table, x, wt, n = _CPU_CACHE["conv"]
    t0 = time.perf_counter()
    out = np.zeros((table.shape[0], wt.shape[2]), np.float32)
    for k in range(27):
        out += x[table[:, k]] @ wt[k]
    secs = time.perf_counter() - t0
    pairs = int((table < n).sum())
    return 2.0 * wt.shape[1] * wt.shape[2] * pairs / secs / 1e12, f"{sample} output rows of cfg5, fp32 gather-GEMM"


W8A8_GEMMS = (("self_attn.to_qkv", 1024, 3072), ("self_attn.to_out", 1024, 1024), ("cross_attn.to_q", 1024, 1024),
              ("cross_attn.to_out", 1024, 1024), ("mlp.mlp.0", 1024, 4096), ("mlp.mlp.2", 4096, 1024))


def cpu_w8a8_tops(rows: int = 64) -> tuple[float, str]:
    """The reference's CPU statement of the W8A8 GEMM (its contract test, int64 numpy,
    tests/test_w8a8_inference.py:15) over ``rows`` rows of each of a block's six projections."""
    rng = np.random.default_rng(9)
    ops_total, secs = 0.0, 0.0
    for _, k, n in W8A8_GEMMS:
        a = rng.integers(-127, 128, (rows, k), dtype=np.int8)
        w = rng.integers(-127, 128, (n, k), dtype=np.int8)
        t0 = time.perf_counter()
        _ = a.astype(np.int64) @ w.astype(np.int64).T
        secs += time.perf_counter() - t0
        ops_total += 2.0 * rows * k * n
    return ops_total / secs / 1e12, f"{rows} rows of each of a block's six projections, int64 numpy GEMM"


# ----------------------------------------------------------------------------- reference arm


def run_reference(args) -> None:
    """The CPU path of the reference, timed on the host's cores (rank 0 only under torchrun)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = cpu_threads()
    world = args.gpus
    secs = []

    def steps(fn):
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            r = fn()
            if i >= args.warmup:
                secs.append(time.perf_counter() - t0)
        return r

    if args.workload == "released":
        _cpu_block_inputs(released=True)
        steps(lambda: cpu_block_seconds(released=True))
        metric, unit = "block_tokens_per_s", "tokens/s"
        value = T_TOKENS * len(secs) / sum(secs)
        d = REL_C // REL_HEADS
        config = {"workload": f"released shape: {BLOCKS}-block stack fwd, T={T_TOKENS}, C={REL_C}, "
                              f"{REL_HEADS}x{d} heads, {REL_L} cond tokens of width {REL_CC}, fp16"}
        desc = (f"one whole fp32 block at the released shape, T={T_TOKENS}, per step: the reference's CPU "
                f"path (upstream block + flash_attn shim) restated in torch")
    elif args.workload in ("stack", "stack_w8a8", "block"):
        nblocks = 1 if args.workload == "block" else BLOCKS
        _cpu_block_inputs()
        steps(cpu_block_seconds)
        metric, unit = "block_tokens_per_s", "tokens/s"
        value = T_TOKENS * len(secs) / sum(secs)
        config = stack_config(args.workload, nblocks, world, args.kv_transport)
        desc = (f"one whole fp32 block at T={T_TOKENS} per step (each of the stack's {nblocks} blocks has this "
                f"shape): the reference's CPU path, upstream block + flash_attn shim (SDPA over query blocks), "
                f"restated in torch and pinned to the upstream module")
        if args.workload == "stack_w8a8":
            desc += "; the reference's W8A8 GEMM exists only as a Metal kernel, so its CPU path is this fp32 block"
    elif args.workload == "forward":
        from oracle import ops

        est = []
        steps(lambda: est.append(cpu_forward_seconds()))
        n_low = ops.downsample_structure(forward_inputs()[0])[0].shape[0]
        fwd_s = statistics.median(e[0] for e in est[args.warmup:])
        desc = est[-1][2]
        metric, unit, value = "forward_tokens_per_s", "tokens/s", n_low / fwd_s
        config = {"workload": f"whole refinement transformer fwd: {FWD_FINE} fine shell voxels, {n_low} low tokens, "
                              f"{BLOCKS} blocks", "low_tokens": n_low}
    elif args.workload == "kernels":
        import torch

        x = torch.randn((T_TOKENS, CHANNELS))
        sc, sh = torch.randn(CHANNELS), torch.randn(CHANNELS)

        def ln():
            # the reference's CPU LayerNorm32 + modulation (norm.py:12-17, modulated.py:55-56), fp32
            torch.nn.functional.layer_norm(x, (CHANNELS,), eps=1e-6) * (1 + sc) + sh

        steps(ln)
        value, unit, metric = 2.0 * T_TOKENS * CHANNELS * 4 * len(secs) / sum(secs) / 1e9, "GB/s", "layer_norm_modulate_gbs"
        desc = f"fp32 LayerNorm32 + modulation of {T_TOKENS} x {CHANNELS} rows on the host (the reference's CPU path)"
        config = {"workload": f"row kernels and projection epilogues at T={T_TOKENS}, C={CHANNELS} (quantiser also "
                              f"at width 4096), fp16, each timed alone"}
    elif args.workload in ("conv", "vae"):
        vals = []
        steps(lambda: vals.append(cpu_conv_tflops()))
        value, unit = statistics.median(v[0] for v in vals[args.warmup:]), "TFLOP/s"
        desc = vals[-1][1]
        metric = "sparse_conv_tflops" if args.workload == "conv" else "vae_conv_gn_swish_tflops"
        config = conv_config()
    else:
        big = args.workload == "attention262k"
        vals = []
        steps(lambda: vals.append(cpu_attention_tflops(big)))
        value, unit, metric = statistics.median(v[0] for v in vals[args.warmup:]), "TFLOP/s", "attention_tflops"
        desc = vals[-1][1]
        config = attention_config(big, world)
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sum(secs) / len(secs) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm: helpers


def _timed(fn, steps: int, warmup: int) -> float:
    """Milliseconds per call of ``fn`` (CUDA events on the current stream, after ``warmup`` calls)."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _timed_graph(fn, steps: int, warmup: int, per_graph: int = 16) -> float:
    """Milliseconds per call of ``fn`` on the device alone: ``per_graph`` calls captured in one
    CUDA graph, replayed ``steps`` times between CUDA events (after ``warmup`` eager calls and one
    replay).  For kernels of a few tens of microseconds, whose eager launches through Python
    would leave the GPU waiting on the host."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for _ in range(per_graph):
                fn()
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (steps * per_graph)
    del graph
    return ms


def _max_over_ranks(ms: float, world: int, dev) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return ms
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure_w8a8(weights, inputs, steps: int, warmup: int, fp16_ms: float) -> dict:
    """cfg2 beside the headline: the W8A8 24-block stack (weights quantised on the GPU from the
    same fp16 weights) and each int8 projection GEMM of a block at M = T."""
    import torch

    from hi3d_b200 import transformer, w8a8

    x_dev, mod_d, cos_d, sin_d, cond_d = inputs
    w8 = [transformer.to_w8a8(w) for w in weights]
    stack = transformer.BlockStack(w8, HEADS)
    kvs = [transformer.context_kv(w, cond_d, HEADS) for w in w8]
    ms = _timed(lambda: stack(x_dev[None], mod_d, cos_d, sin_d, kvs), steps, warmup)
    g = torch.Generator(device=x_dev.device).manual_seed(11)
    per, ops_all, t_all = {}, 0.0, 0.0
    for name, k, n in W8A8_GEMMS:
        a = torch.randint(-127, 128, (T_TOKENS, k), generator=g, device=x_dev.device, dtype=torch.int8)
        sa = torch.rand(T_TOKENS, generator=g, device=x_dev.device) * 0.01 + 1e-3
        qa = w8a8.Quantized(a, sa, (T_TOKENS, k), torch.float16)
        wq, sw, b = w8[0][f"{name}.weight"], w8[0][f"{name}.w8_scale"], w8[0][f"{name}.bias"]
        t = _timed(lambda: w8a8.linear(qa, wq, sw, b), steps, warmup)
        per[name] = 2.0 * T_TOKENS * k * n / (t / 1e3) / 1e12
        ops_all += 2.0 * T_TOKENS * k * n
        t_all += t
    del w8, stack, kvs
    tops = ops_all / (t_all / 1e3) / 1e12
    peaks = _peaks()
    peak = 2 * peaks["bf16_tflops"]
    cv, cdesc = cpu_w8a8_tops()
    return {"ms_per_step": ms, "tokens_per_s": BLOCKS * T_TOKENS / (ms / 1e3), "fp16_over_w8a8_time": fp16_ms / ms,
            "int8_gemm_tops": tops, "int8_gemm_tops_per_projection": per,
            "roofline": {"bound": "tensor", "achieved": tops, "peak": peak, "unit": "TOP/s", "frac": tops / peak,
                         "peak_source": f"2 x {peaks['source']} bf16_tflops burst (the dense int8 rate is twice "
                                        f"the bf16 rate); GEMMs timed alone"},
            "cpu_baseline": {"value": cv, "unit": "TOP/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": cdesc}}


def measure_conv(dev, steps: int, warmup: int) -> dict:
    """cfg5: neighbour map, submanifold conv and the stride-2 conv at 200,000 voxels, 256 -> 256."""
    import torch

    from hi3d_b200 import sparse, synthetic

    n, c = CONV_N, CONV_C
    coords = synthetic.shell_coords(n, 128, 48, 4, seed=5)
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn((n, c), generator=g, device=dev).half()
    w = (torch.randn((c, 3, 3, 3, c), generator=g, device=dev) * 0.02).half()
    b = (torch.randn(c, generator=g, device=dev) * 0.02).half()
    cdev = torch.from_numpy(coords).to(dev)
    level = sparse.Level(cdev, sparse.neighbour_table(cdev))
    map_ms = _timed(lambda: sparse.neighbour_table(cdev), steps, warmup)
    mask = level.tap_mask
    pairs = int((level.table < n).sum().item())
    conv_ms = _timed(lambda: sparse.conv(x, level.table, w, b, tap_mask=mask), steps, warmup)
    low, _, _ = sparse.downsample_structure(cdev)
    table2 = sparse.neighbour_table(cdev, query=low, stride=2)
    mask2 = sparse.conv_tap_mask(table2, n)
    pairs2 = int((table2 < n).sum().item())
    down_ms = _timed(lambda: sparse.conv(x, table2, w, b, n_in=n, tap_mask=mask2), steps, warmup)
    struct_ms = _timed(lambda: sparse.downsample_structure(cdev), steps, warmup)
    tflops = 2.0 * c * c * pairs / (conv_ms / 1e3) / 1e12
    peaks = _peaks()
    cv, cdesc = cpu_conv_tflops()
    return {"value": tflops, "unit": "TFLOP/s", "ms": conv_ms, "pairs": pairs,
            "dense_equivalent_tflops": 2.0 * 27 * n * c * c / (conv_ms / 1e3) / 1e12,
            "neighbour_map_ms": map_ms, "lookups_per_s": 27 * n / (map_ms / 1e3),
            "stride2_conv_ms": down_ms, "stride2_low_voxels": int(low.shape[0]), "stride2_pairs": pairs2,
            "stride2_tflops": 2.0 * c * c * pairs2 / (down_ms / 1e3) / 1e12,
            "downsample_structure_ms": struct_ms,
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tflops / peaks["bf16_tflops"], "traffic": _profile_traffic("sparse_conv_cfg5"),
                         "peak_source": f"{peaks['source']} bf16_tflops (burst; kernel timed alone)"},
            "cpu_baseline": {"value": cv, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": cdesc}}


def measure_cfg4(dev, world: int, rank: int, steps: int, warmup: int, sub) -> dict:
    """cfg4: bf16 self-attention over 4 objects x 65,536 tokens, the packed tokens split into
    contiguous slices over the ranks.  With at most 4 ranks each rank holds whole objects and
    attends them alone; with more, the ranks of one object all-gather its K/V shards (``sub``, from
    ``dist.object_group``), then attend all its keys.  Every rank times its own slice; the
    step time is the maximum over ranks."""
    import torch

    from hi3d_b200 import attention, dist as hdist

    objects, per, d = 4, 65536, CHANNELS // HEADS
    tl = objects * per // world
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    # RoPE'd, RMS-normalised queries/keys have per-head norm sqrt(D): unit-variance entries
    q, k, v = (torch.randn((tl, HEADS, d), generator=g, device=dev).bfloat16() for _ in range(3))
    scale = d ** -0.5
    if sub is None:
        n_obj = objects // world
        cu = torch.arange(n_obj + 1, device=dev, dtype=torch.int32) * per
        out = torch.empty_like(q)
        step = lambda: attention.flash_attn_varlen(q, k, v, cu, cu, per, scale, out=out)
        exchange = 0
    else:
        # this rank's keys/values in its slot of the gather buffers (where the projection writes them)
        kvb = hdist.kv_gather_buffers(tl, HEADS, d, q.dtype, dev, sub)
        hdist.own_rows(kvb[0], sub)[0].copy_(k)
        hdist.own_rows(kvb[1], sub)[0].copy_(v)
        step = lambda: hdist.sharded_self_attention(q[None], kvb[0], kvb[1], scale, sub)
        exchange = 2 * (per - tl) * HEADS * d * 2
    ms = _timed(step, steps, warmup)
    ms = _max_over_ranks(ms, world, dev)
    flops = 4.0 * objects * per * per * HEADS * d
    tflops = flops / (ms / 1e3) / 1e12
    peaks = _peaks()
    peak = peaks["bf16_tflops_sustained"]
    line = {"value": tflops, "unit": "TFLOP/s", "ms_per_layer": ms, "tflops_per_gpu": tflops / world,
            "kv_bytes_received_per_rank": exchange,
            "roofline": {"bound": "tensor", "achieved": tflops / world, "peak": peak, "unit": "TFLOP/s",
                         "frac": tflops / world / peak,
                         "peak_source": f"{peaks['source']} bf16_tflops_sustained (burst {peaks['bf16_tflops']})"}}
    if rank == 0 and world == 1:
        cv, cdesc = cpu_attention_tflops(True)
        line["cpu_baseline"] = {"value": cv, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                                "sample": cdesc}
    return line


def sharded_parity(weights, inputs_local, inputs_full, world: int, rank: int, dev,
                   transport: str = "nccl") -> float | None:
    """Relative L2 between the first two blocks run query-sharded over the ranks and the same two
    blocks on one GPU (rank 0), on the bench inputs; None on ranks other than 0."""
    import torch

    from hi3d_b200 import dist as hdist, transformer

    x_l, mod_d, cos_l, sin_l, cond_d = inputs_local
    two = weights[:2]
    kvs = [transformer.context_kv(w, cond_d, HEADS) for w in two]
    stack = hdist.ShardedBlockStack(two, HEADS, transport=transport)
    y_local = stack(x_l, mod_d, cos_l, sin_l, kvs)
    y_all = hdist.gather_rows(y_local)
    stack.close()  # collective: no rank releases its buffers while another still stores into them
    if rank != 0:
        return None
    x_f, cos_f, sin_f = inputs_full
    ref = transformer.BlockStack(two, HEADS)(x_f[None], mod_d, cos_f, sin_f, kvs)[0]
    return float((y_all.float() - ref.float()).norm() / ref.float().norm())


# ----------------------------------------------------------------------------- GPU arm: stack


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from hi3d_b200 import _lib, attention, dist as hdist, transformer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        hdist.init_nccl(dev)
    _lib.load()
    cpu_threads()

    coords, cos, sin, x, mod, cond = make_inputs(0)
    if T_TOKENS % world:
        raise ValueError("T must divide by the number of GPUs")
    tl = T_TOKENS // world
    rows = slice(rank * tl, (rank + 1) * tl)
    nblocks = 1 if args.workload == "block" else BLOCKS
    weights = device_weights(dev, blocks=nblocks)
    if args.workload == "stack_w8a8":
        weights = [transformer.to_w8a8(w) for w in weights]
    x_host = torch.from_numpy(x[rows]).pin_memory()
    x_dev = x_host.to(dev)
    cos_d, sin_d = torch.from_numpy(cos[rows]).to(dev), torch.from_numpy(sin[rows]).to(dev)
    mod_d = torch.from_numpy(mod).to(dev)
    cond_d = torch.from_numpy(cond).to(dev)
    if world == 1:
        stack = transformer.BlockStack(weights, HEADS)
        run = lambda xin: stack(xin[None], mod_d, cos_d, sin_d, kvs)[0]
    else:
        stack = hdist.ShardedBlockStack(weights, HEADS, transport=args.kv_transport)
        run = lambda xin: stack(xin, mod_d, cos_d, sin_d, kvs)
    kvs = [transformer.context_kv(w, cond_d, HEADS) for w in weights]

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        run(x_dev)
    torch.cuda.synchronize()
    barrier()

    # ---- device-resident timed region (attention launches timed live with events)
    stream = torch.cuda.current_stream()
    attention.TIMER.start()
    _lib.LAUNCHES[0] = 0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        barrier()
        start.record(stream)
        for _ in range(args.steps):
            run(x_dev)
        end.record(stream)
        torch.cuda.synchronize()
        barrier()
    launches = _lib.LAUNCHES[0]
    attn = attention.TIMER.stop()
    # host time to enqueue one step onto an idle stream: below the device step time, the
    # step is device-bound
    h0 = time.perf_counter()
    run(x_dev)
    host_ms = (time.perf_counter() - h0) * 1e3
    torch.cuda.synchronize()
    barrier()
    ms = _max_over_ranks(start.elapsed_time(end), world, dev)
    ms_per_step = ms / args.steps
    value = nblocks * T_TOKENS / (ms_per_step / 1e3)

    # ---- end to end through the public API: pinned host input -> stack -> host output
    out_host = torch.empty_like(x_host).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        xin = x_host.to(dev, non_blocking=True)
        out_host.copy_(run(xin), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    e2e_value = nblocks * T_TOKENS / (e2e_ms / args.steps / 1e3)

    # ---- roofline of the dominant kernel (self-attention)
    peaks = _peaks()
    # Self-attention: one launch per block over all keys, or (sharded) the partial launches over the
    # rank's own and the gathered keys; every block has exactly one cross-attention launch.
    self_launches = [r for r in attn if r["nk"] != COND and r["flops"]]
    n_blocks_seen = max(1, sum(1 for r in attn if r["nk"] == COND))
    avg_s = sum(r["ms"] for r in self_launches) / n_blocks_seen / 1e3
    flops = sum(r["flops"] for r in self_launches) / n_blocks_seen
    achieved = flops / avg_s / 1e12 if avg_s > 0 else 0.0
    peak = peaks["bf16_tflops_sustained"]
    attn_share = sum(r["ms"] for r in attn) / ms if ms > 0 else None
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": _profile_traffic("flash_attn_fwd_cfg1"), "kernel": "hi3d::attn::flash_fwd_kernel<half,64,false>",
                "peak_source": f"{peaks['source']} bf16_tflops_sustained (burst {peaks['bf16_tflops']})",
                "flops_per_launch": flops, "avg_launch_ms": avg_s * 1e3, "attention_time_share": attn_share}

    line = {
        "metric": "block_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": stack_config(args.workload, nblocks, world,
                               stack.transport if world > 1 else args.kv_transport),
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": x_host.numel() * 2,
                "d2h_bytes_per_step": out_host.numel() * 2},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "attention_tflops": achieved,
        "host_enqueue_ms_per_step": host_ms,
    }
    extra = args.workload == "stack" and not args.no_extras
    if world > 1:
        # per-phase breakdown of one step on every rank (outside the timed region), the maximum
        # over ranks per phase, then the sharded stack's parity against one GPU
        timer = hdist.PhaseTimer()
        torch.cuda.synchronize()
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(2):
            stack(x_dev, mod_d, cos_d, sin_d, kvs, timer=timer)
        t1.record()
        phases = timer.totals()
        names = sorted(phases)
        vals = torch.tensor([phases[n] / 2 for n in names] + [t0.elapsed_time(t1) / 2], device=dev)
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        bd = {n: float(v) for n, v in zip(names + ["step_with_marks"], vals.tolist())}
        line["breakdown_ms_per_step"] = bd
        if args.workload in ("stack", "block"):
            x_full = torch.from_numpy(x).to(dev) if rank == 0 else None
            cos_f = torch.from_numpy(cos).to(dev) if rank == 0 else None
            sin_f = torch.from_numpy(sin).to(dev) if rank == 0 else None
            err = sharded_parity(weights, (x_dev, mod_d, cos_d, sin_d, cond_d), (x_full, cos_f, sin_f), world, rank,
                                 dev, args.kv_transport)
            if rank == 0:
                line["sharded_rel_l2"] = err
                line["sharded_rel_l2_case"] = "first 2 blocks query-sharded vs one GPU on the bench inputs"
        barrier()
    if extra:
        # the north-star's multi-GPU configuration beside the headline (outside its timed region)
        sub = hdist.object_group(4) if world > 1 else None
        line["cfg4_attention"] = measure_cfg4(dev, world, rank, max(3, args.steps // 4), 2, sub)
        line["extra_keys"] = ["cfg4_attention"]
    if extra and world == 1:
        line["cfg2_w8a8"] = measure_w8a8(weights, (x_dev, mod_d, cos_d, sin_d, cond_d), max(3, args.steps // 2),
                                         args.warmup, ms_per_step)
        line["cfg5_conv"] = measure_conv(dev, args.steps, args.warmup)
        line["extra_keys"] += ["cfg2_w8a8", "cfg5_conv"]
    if rank == 0 and world == 1:
        cpu_block_seconds(rows=4096)  # warm the thread pool and allocator
        secs = cpu_block_seconds()
        line["cpu_baseline"] = {"value": T_TOKENS / secs, "unit": "tokens/s", "cores": torch.get_num_threads(),
                                "kind": "port",
                                "sample": f"one whole fp32 block at T={T_TOKENS} (one of the stack's {nblocks}): the "
                                          f"reference's CPU path (upstream block + flash_attn shim), restated in torch",
                                "seconds_per_block": secs}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        # every rank drops its symmetric K/V buffers (and their multicast binding) at the same
        # point, with no kernel in flight, before the process group goes away
        stack.close()  # collective: every rank drops its symmetric buffers at the same point
        dist.barrier()
        dist.destroy_process_group()


def run_attention(args, big: bool) -> None:
    """Self-attention kernel alone: cfg1 (T=32768 fp16, one object) or cfg4 (4 x 65536 bf16 varlen,
    query-sharded over the GPUs with per-object K/V exchange)."""
    import torch
    import torch.distributed as dist

    from hi3d_b200 import _lib, attention, dist as hdist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        hdist.init_nccl(dev)
    _lib.load()
    cpu_threads()
    d = CHANNELS // HEADS
    peaks = _peaks()
    _lib.LAUNCHES[0] = 0
    if big:
        sub = hdist.object_group(4) if world > 1 else None
        with ClockSampler(local) as clocks:
            r = measure_cfg4(dev, world, rank, args.steps, args.warmup, sub)
        launches = _lib.LAUNCHES[0]
        ms_step, tflops = r["ms_per_layer"], r["value"]
        roof = dict(r["roofline"], traffic=_profile_traffic("flash_attn_fwd_cfg4"))
        # end to end: this rank's q/k/v slice from pinned host memory, the output back to the host
        tl = 4 * 65536 // world
        g = torch.Generator().manual_seed(8 + rank)
        hq, hk, hv = (torch.randn((tl, HEADS, d), generator=g).bfloat16().pin_memory() for _ in range(3))
        hout = torch.empty((tl, HEADS, d), dtype=torch.bfloat16).pin_memory()
        kvb = hdist.kv_gather_buffers(tl, HEADS, d, torch.bfloat16, dev, sub) if sub is not None else None

        def e2e_step():
            dq = hq.to(dev, non_blocking=True)
            if sub is None:
                dk, dv = (t.to(dev, non_blocking=True) for t in (hk, hv))
                n_obj = 4 // world
                cu = torch.arange(n_obj + 1, device=dev, dtype=torch.int32) * 65536
                o = attention.flash_attn_varlen(dq, dk, dv, cu, cu, 65536, d ** -0.5)
            else:  # keys/values straight into this rank's slot of the gather buffers
                hdist.own_rows(kvb[0], sub)[0].copy_(hk, non_blocking=True)
                hdist.own_rows(kvb[1], sub)[0].copy_(hv, non_blocking=True)
                o = hdist.sharded_self_attention(dq[None], kvb[0], kvb[1], d ** -0.5, sub)[0].view(tl, HEADS, d)
            hout.copy_(o, non_blocking=True)

        e2e_ms = _max_over_ranks(_timed(e2e_step, args.steps, 1), world, dev)
        flops_all = 4.0 * 4 * 65536 * 65536 * HEADS * d
        e2e = {"value": flops_all / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": 3 * tl * HEADS * d * 2, "d2h_bytes_per_step": tl * HEADS * d * 2}
        cpu = r.get("cpu_baseline")
        extra = {"kv_bytes_received_per_rank": r["kv_bytes_received_per_rank"]}
    else:
        g = torch.Generator(device=dev).manual_seed(7)
        per = T_TOKENS
        k = torch.randn((per, HEADS, d), generator=g, device=dev).half()
        v = torch.randn((per, HEADS, d), generator=g, device=dev).half()
        if per % world:
            raise ValueError("tokens must divide by the number of GPUs")
        ql = per // world
        q = torch.randn((ql, HEADS, d), generator=g, device=dev).half()
        cu_q = torch.tensor([0, ql], device=dev, dtype=torch.int32)
        cu_k = torch.tensor([0, per], device=dev, dtype=torch.int32)
        out = torch.empty_like(q)
        with ClockSampler(local) as clocks:
            ms_step = _timed(lambda: attention.flash_attn_varlen(q, k, v, cu_q, cu_k, ql, d ** -0.5, out=out),
                             args.steps, args.warmup)
        launches = _lib.LAUNCHES[0]
        ms_step = _max_over_ranks(ms_step, world, dev)
        flops = 4.0 * ql * per * HEADS * d
        tflops = flops * world / (ms_step / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": tflops / world, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": tflops / world / peaks["bf16_tflops"], "traffic": _profile_traffic("flash_attn_fwd_cfg1"),
                "peak_source": f"{peaks['source']} bf16_tflops (burst; kernel timed alone)"}
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hout = torch.empty_like(hq).pin_memory()

        def e2e_step():
            dq, dk, dv = (t.to(dev, non_blocking=True) for t in (hq, hk, hv))
            hout.copy_(attention.flash_attn_varlen(dq, dk, dv, cu_q, cu_k, ql, d ** -0.5), non_blocking=True)

        e2e_ms = _max_over_ranks(_timed(e2e_step, args.steps, 1), world, dev)
        e2e = {"value": flops * world / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": (q.numel() + k.numel() + v.numel()) * 2, "d2h_bytes_per_step": out.numel() * 2}
        cpu = None
        if rank == 0 and world == 1:
            cv, cdesc = cpu_attention_tflops(False)
            cpu = {"value": cv, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port", "sample": cdesc}
        extra = {}
    line = {
        "metric": "attention_tflops", "value": tflops, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if big else "f16", "data": "synthetic",
        "config": attention_config(big, world), "roofline": roof, "e2e": e2e, "gpu_launches": launches,
        "clocks": clocks.summary(), **extra,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_conv(args) -> None:
    """cfg5: submanifold 3x3x3 conv, 200,000 shell voxels in 128^3, C_in = C_out = 256, fp16.
    A step = one convolution over all voxels (the neighbour map is built once per level, as in
    the reference, and timed separately).  Reports TFLOP/s over the actual neighbour pairs
    (2 * Cin * Cout per present pair); the dense-equivalent count is in the config."""
    import torch

    from hi3d_b200 import _lib, sparse, synthetic

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _lib.load()
    cpu_threads()
    _lib.LAUNCHES[0] = 0
    with ClockSampler(0) as clocks:
        r = measure_conv(dev, args.steps, args.warmup)
    launches = _lib.LAUNCHES[0]
    n, c = CONV_N, CONV_C
    coords = synthetic.shell_coords(n, 128, 48, 4, seed=5)
    cdev = torch.from_numpy(coords).to(dev)
    level = sparse.Level(cdev, sparse.neighbour_table(cdev))
    g = torch.Generator(device=dev).manual_seed(3)
    w = (torch.randn((c, 3, 3, 3, c), generator=g, device=dev) * 0.02).half()
    b = (torch.randn(c, generator=g, device=dev) * 0.02).half()
    hx = torch.randn((n, c), generator=g).half().pin_memory()
    hout = torch.empty((n, c), dtype=torch.float16).pin_memory()
    mask = level.tap_mask
    e2e_ms = _timed(lambda: hout.copy_(sparse.conv(hx.to(dev, non_blocking=True), level.table, w, b, tap_mask=mask),
                                       non_blocking=True), args.steps, 1)
    flops = 2.0 * c * c * r["pairs"]
    cfg = dict(conv_config(), **{k: r[k] for k in ("pairs", "dense_equivalent_tflops", "neighbour_map_ms",
                                                    "lookups_per_s", "stride2_conv_ms", "stride2_tflops",
                                                    "downsample_structure_ms")})
    line = {
        "metric": "sparse_conv_tflops", "value": r["value"], "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "f16", "data": "synthetic", "config": cfg,
        "roofline": r["roofline"],
        "e2e": {"value": flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": n * c * 2,
                "d2h_bytes_per_step": n * c * 2},
        "gpu_launches": launches, "clocks": clocks.summary(), "cpu_baseline": r["cpu_baseline"],
    }
    print(json.dumps(line), flush=True)


def run_forward(args) -> None:
    """The whole refinement transformer (one conditioned branch) on one GPU: a step is one
    velocity evaluation, inputs resident; ``value`` = low-level tokens / step time."""
    import torch

    from hi3d_b200 import _lib, attention, model, synthetic

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _lib.load()
    cpu_threads()
    coords, feats, cond = forward_inputs()
    cfg = model.ModelConfig(model_channels=CHANNELS, cond_channels=CHANNELS, num_heads=HEADS, num_blocks=BLOCKS,
                            io_channels=FWD_IO)
    m = model.Sparc3DTransformer(cfg, synthetic.model_weights(CHANNELS, CHANNELS, HEADS, BLOCKS, io_channels=FWD_IO,
                                                              seed=3), device=dev)
    geo = model.Geometry(coords, cfg.head_dim, device=dev)
    n_low = geo.low.n
    kvs = m.prepare(torch.from_numpy(cond).to(dev))
    f_host = torch.from_numpy(feats).pin_memory()
    f_dev = f_host.to(dev)
    step = lambda f: m(f, FWD_T, geo, kvs)[0]
    for _ in range(args.warmup):
        step(f_dev)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    attention.TIMER.start()
    _lib.LAUNCHES[0] = 0
    with ClockSampler(0) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step(f_dev)
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.LAUNCHES[0]
    attn = attention.TIMER.stop()
    ms = e0.elapsed_time(e1) / args.steps
    # the I/O stages alone (same calls as inside a step), for the split of the step time
    emb, _ = m.embed(FWD_T)
    e0.record(stream)
    for _ in range(args.steps):
        h, skip0 = m.input_stage(f_dev, emb, geo)
        m.output_stage(h, h, skip0, emb, geo)
    e1.record(stream)
    torch.cuda.synchronize()
    io_ms = e0.elapsed_time(e1) / args.steps
    # a guided evaluation: the [condition, zero condition] batch, first block's self-attention shared
    e0.record(stream)
    for _ in range(args.steps):
        m(f_dev, FWD_T, geo, kvs, negative=True)
    e1.record(stream)
    torch.cuda.synchronize()
    guided_ms = e0.elapsed_time(e1) / args.steps
    out_host = torch.empty((coords.shape[0], 32), dtype=torch.float32).pin_memory()
    e0.record(stream)
    for _ in range(args.steps):
        out_host.copy_(step(f_host.to(dev, non_blocking=True)), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    peaks = _peaks()
    self_launches = [r for r in attn if r["nk"] == n_low and r["flops"]]
    avg_s = sum(r["ms"] for r in self_launches) / max(1, len(self_launches)) / 1e3
    flops = sum(r["flops"] for r in self_launches) / max(1, len(self_launches))
    achieved = flops / avg_s / 1e12 if avg_s > 0 else 0.0
    peak = peaks["bf16_tflops_sustained"]
    line = {
        "metric": "forward_tokens_per_s", "value": n_low / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"whole refinement transformer fwd: {FWD_FINE} fine shell voxels, {n_low} low tokens, "
                               f"{BLOCKS} blocks", "low_tokens": n_low,
                   "detail": (f"{coords.shape[0]} fine shell voxels in {FWD_GRID}^3 -> {n_low} low tokens, I/O stage "
                              f"{FWD_IO} channels, {BLOCKS} blocks C={CHANNELS} {HEADS}x{CHANNELS // HEADS} heads, "
                              f"{COND} cond tokens, fp16 torso"),
                   "io_stages_ms": io_ms, "stack_ms": ms - io_ms, "guided_batch2_ms": guided_ms,
                   "l2": "inputs larger than L2 (705 MB of weights per step)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None,
                     "kernel": "hi3d::attn::flash_fwd_kernel<half,64,false>",
                     "peak_source": f"{peaks['source']} bf16_tflops_sustained", "flops_per_launch": flops,
                     "avg_launch_ms": avg_s * 1e3},
        "e2e": {"value": n_low / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": f_host.numel() * 4,
                "d2h_bytes_per_step": out_host.numel() * 4},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }
    secs, _, desc = cpu_forward_seconds()
    line["cpu_baseline"] = {"value": n_low / secs, "unit": "tokens/s", "cores": torch.get_num_threads(),
                            "kind": "port", "sample": desc}
    print(json.dumps(line), flush=True)


def run_released(args) -> None:
    """The 24-block stack at the released model's shape, T = 32,768 tokens (fp16, one GPU).
    At head dim 96 the QKV projection runs as a plain GEMM followed by the RoPE + QK-norm row
    kernel (the fused epilogue needs head dim 64); the line reports block tokens/s, the
    self-attention TFLOP/s and the per-block split of projections, norms and attention."""
    import torch

    from hi3d_b200 import _lib, attention, synthetic, transformer

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _lib.load()
    cpu_threads()
    d = REL_C // REL_HEADS
    coords = synthetic.shell_coords(T_TOKENS, GRID, RADIUS, THICK, seed=0)
    cos, sin = transformer.rope_tables(coords, d)
    x = synthetic.features(T_TOKENS, REL_C, seed=1)
    mod = synthetic.modulation(REL_C, 0.5, seed=2).astype(np.float16)
    cond = synthetic.features(REL_L, REL_CC, seed=3)
    weights = device_weights(dev, blocks=BLOCKS, c=REL_C, cc=REL_CC, heads=REL_HEADS)
    stack = transformer.BlockStack(weights, REL_HEADS)
    x_dev = torch.from_numpy(x).to(dev)
    cos_d, sin_d = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    mod_d = torch.from_numpy(mod).to(dev)
    kvs = stack.prepare(torch.from_numpy(cond).to(dev))
    run = lambda xin: stack(xin[None], mod_d, cos_d, sin_d, kvs)[0]
    attention.TIMER.start()
    _lib.LAUNCHES[0] = 0
    with ClockSampler(0) as clocks:
        ms = _timed(lambda: run(x_dev), args.steps, args.warmup)
    launches = _lib.LAUNCHES[0]
    attn = attention.TIMER.stop()
    self_l = [r for r in attn if r["nk"] == T_TOKENS and r["flops"]]
    cross_l = [r for r in attn if r["nk"] == REL_L and r["flops"]]
    a_ms = sum(r["ms"] for r in self_l) / max(1, len(self_l))
    a_tflops = sum(r["flops"] for r in self_l) / max(1, len(self_l)) / (a_ms / 1e3) / 1e12 if a_ms else 0.0
    c_ms = sum(r["ms"] for r in cross_l) / max(1, len(cross_l))
    peaks = _peaks()
    value = BLOCKS * T_TOKENS / (ms / 1e3)
    x_host = torch.from_numpy(x).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    e2e_ms = _timed(lambda: out_host.copy_(run(x_host.to(dev, non_blocking=True)), non_blocking=True), args.steps, 1)
    line = {
        "metric": "block_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"released shape: {BLOCKS}-block stack fwd, T={T_TOKENS}, C={REL_C}, "
                               f"{REL_HEADS}x{d} heads, {REL_L} cond tokens of width {REL_CC}, fp16",
                   "self_attention_ms_per_block": a_ms, "cross_attention_ms_per_block": c_ms,
                   "other_ms_per_block": ms / BLOCKS - a_ms - c_ms,
                   "l2": "inputs larger than L2 (weights 2.4 GB per step)"},
        "roofline": {"bound": "tensor", "achieved": a_tflops, "peak": peaks["bf16_tflops_sustained"],
                     "unit": "TFLOP/s", "frac": a_tflops / peaks["bf16_tflops_sustained"],
                     "kernel": "hi3d::attn::flash_fwd_kernel<half,96,false>",
                     "peak_source": f"{peaks['source']} bf16_tflops_sustained"},
        "e2e": {"value": BLOCKS * T_TOKENS / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": out_host.numel() * 2},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_kernels(args) -> None:
    """The block's row kernels and projection epilogues alone at cfg1/cfg2 sizes (one GPU): the
    two LayerNorm forms (T x 1024, inputs rotated over 8 copies so every launch reads HBM), the
    W8A8 activation quantiser at widths 1024 and 4096, and the K = 1024 projection with each
    epilogue (store, residual, gated residual).  ``value`` is the modulated LayerNorm's fraction of
    the measured HBM bandwidth; every kernel's time and fraction is in ``config``."""
    import torch

    from hi3d_b200 import _lib, kernels, linear, w8a8

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _lib.load()
    peaks = _peaks()
    g = torch.Generator(device=dev).manual_seed(5)
    R, C = T_TOKENS, CHANNELS
    xs = [torch.randn((R, C), generator=g, device=dev).half() for _ in range(8)]
    sc, sh = torch.randn(C, generator=g, device=dev).half(), torch.randn(C, generator=g, device=dev).half()
    wln, bln = torch.rand(C, generator=g, device=dev) + 0.5, torch.randn(C, generator=g, device=dev) * 0.1
    res = {}
    _lib.LAUNCHES[0] = 0
    it = [0]

    def rot():
        it[0] += 1
        return xs[it[0] % 8]

    xqs = {k: [torch.randn((R, k), generator=g, device=dev).half() for _ in range(8 if k == 1024 else 2)]
           for k in (1024, 4096)}
    wt = (torch.randn((C, C), generator=g, device=dev) * 0.02).half()
    bt = (torch.randn(C, generator=g, device=dev) * 0.02).half()
    resids = [torch.randn((R, C), generator=g, device=dev).half() for _ in range(8)]
    gate = (torch.randn(C, generator=g, device=dev) * 0.1).half()

    def ln(**kw):
        return lambda: kernels.layer_norm_modulate(rot(), 1e-6, **kw)

    def quant(k):
        def call():
            it[0] += 1
            return w8a8.quantize_activation(xqs[k][it[0] % len(xqs[k])])
        return call

    def gemm(**kw):
        def call():
            a = rot()  # activations and residuals rotated over 8 copies each (> L2)
            extra = dict(residual=resids[it[0] % 8]) if kw["epilogue"] == "residual" else {}
            return linear.linear(a, wt, bt, **kw, **extra)
        return call

    hbm = lambda nbytes: lambda ms: {"gbs": nbytes / (ms / 1e3) / 1e9,
                                     "hbm_frac": nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
    tensor = lambda flop: lambda ms: {"tflops": flop / (ms / 1e3) / 1e12,
                                      "tensor_frac": flop / (ms / 1e3) / 1e12 / peaks["bf16_tflops"]}
    table = [  # name, call, algorithmic rate from the per-launch time
        ("layer_norm_modulate", ln(scale=sc, shift=sh), hbm(4.0 * R * C)),
        ("layer_norm_affine", ln(weight=wln, bias=bln), hbm(4.0 * R * C)),
        ("quantize_act_i8_k1024", quant(1024), hbm(3.0 * R * 1024 + 4 * R)),
        ("quantize_act_i8_k4096", quant(4096), hbm(3.0 * R * 4096 + 4 * R)),
        ("gemm_store", gemm(epilogue="store"), tensor(2.0 * R * C * C)),
        ("gemm_residual", gemm(epilogue="residual"), tensor(2.0 * R * C * C)),
        ("gemm_gated_residual", gemm(epilogue="residual", gate=gate), tensor(2.0 * R * C * C)),
    ]
    if args.only:
        table = [t for t in table if t[0] == args.only]
        if not table:
            raise SystemExit(f"--only {args.only}: not a kernel of this workload")
    # every kernel's launches captured in a CUDA graph (_timed_graph): eager launches through
    # Python take longer on the host than these kernels take on the device
    with ClockSampler(0) as clocks:
        for name, call, rate in table:
            ms = _timed_graph(call, args.steps, args.warmup)
            res[name] = {"us": ms * 1e3, **rate(ms)}
    launches = _lib.LAUNCHES[0]
    head = table[0][0]
    v = res[head].get("gbs", res[head].get("tflops"))
    unit = "GB/s" if "gbs" in res[head] else "TFLOP/s"
    line = {
        "metric": f"{head}_{'gbs' if unit == 'GB/s' else 'tflops'}", "value": v, "unit": unit, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res[head]["us"] / 1e3,
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"row kernels and projection epilogues at T={R}, C={C} (quantiser also at width "
                               f"4096), fp16, each timed alone (16 launches per CUDA graph replay)", "kernels": res,
                   "l2": "every kernel's inputs rotated over copies totalling more than L2",
                   "peak_source": f"{peaks['source']} hbm_gbs {peaks['hbm_gbs']}, bf16_tflops {peaks['bf16_tflops']}"},
        "roofline": {"bound": "hbm" if unit == "GB/s" else "tensor", "achieved": v,
                     "peak": peaks["hbm_gbs"] if unit == "GB/s" else peaks["bf16_tflops"], "unit": unit,
                     "frac": res[head].get("hbm_frac", res[head].get("tensor_frac")), "traffic": None},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_vae(args) -> None:
    """The VAE decoder's kernels at decoder sizes (one line; value = conv(swish(GN(x))) TFLOP/s):
    a 256-channel level of 200,000 voxels (cfg5's shell) through GroupNorm statistics + swish +
    the 3x3x3 conv; the octree child table of that level at 40 % occupancy; serialization and
    48-point window attention over 32,768 latent points with 512 channels in 32 heads (fp16)."""
    import torch

    from hi3d_b200 import _lib, sparse, synthetic, vae

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _lib.load()
    n, c = 200_000, 256
    coords = synthetic.shell_coords(n, 128, 48, 4, seed=5)
    level = sparse.Level.from_coords(coords)
    g = torch.Generator(device=dev).manual_seed(3)
    x = (torch.randn((n, c), generator=g, device=dev) * 2).half()
    nw, nb = torch.rand(c, device=dev) + 0.5, torch.randn(c, device=dev) * 0.1
    w = (torch.randn((c, 3, 3, 3, c), generator=g, device=dev) * 0.02).half()
    b = (torch.randn(c, generator=g, device=dev) * 0.02).half()
    mask = torch.rand((n, 8), device=dev) < 0.4
    lat = synthetic.shell_coords(32768, 64, 24, 3, seed=6)
    lat_d = torch.from_numpy(lat).to(dev)
    qkv = torch.randn((lat.shape[0], 3 * 512), generator=g, device=dev).half()
    pairs = int((level.table < n).sum().item())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    _lib.LAUNCHES[0] = 0
    with ClockSampler(0) as clocks:
        conv_ms = timed(lambda: vae.conv_gn_swish(x, level, nw, nb, w, b))
        stats_ms = timed(lambda: vae.group_stats(x))
        mean, inv = vae.group_stats(x)
        swish_ms = timed(lambda: vae.group_norm_swish(x, mean, inv, nw, nb))
        child_ms = timed(lambda: vae.child_neighbour_table(level.table, mask))
        serial_ms = timed(lambda: vae.serialization(lat_d))
        gather = vae.window_index(vae.serialization(lat_d)[0][0])
        win_ms = timed(lambda: vae.window_attention(qkv, gather, 32))
    launches = _lib.LAUNCHES[0]
    flops = 2.0 * c * c * pairs
    peaks = _peaks()
    win_flops = 4.0 * gather.shape[0] * vae.PATCH * 512  # QK^T + PV over each window, all heads
    line = {
        "metric": "vae_conv_gn_swish_tflops", "value": flops / (conv_ms / 1e3) / 1e12, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": conv_ms, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"VAE decoder kernels: conv(swish(GN(x))) on {n} voxels x {c} channels; child "
                               f"table at 40 % occupancy; window attention over {lat.shape[0]} points, 512 ch, "
                               f"32 heads, windows of {vae.PATCH}",
                   "group_stats_ms": stats_ms, "group_norm_swish_ms": swish_ms,
                   "group_norm_swish_gbs": n * c * 4 / (swish_ms / 1e3) / 1e9,
                   "child_table_ms": child_ms, "serialization_ms": serial_ms, "window_attention_ms": win_ms,
                   "window_attention_tflops": win_flops / (win_ms / 1e3) / 1e12,
                   "l2": "inputs larger than L2 (102 MB features + weights per step)"},
        "roofline": {"bound": "tensor", "achieved": flops / (conv_ms / 1e3) / 1e12, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": flops / (conv_ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                     "traffic": None, "peak_source": f"{peaks['source']} bf16_tflops (burst)",
                     "note": "whole conv_gn_swish step (stats + swish + conv) against the conv's FLOPs"},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="headline only (no cfg2/cfg4/cfg5 extras)")
    ap.add_argument("--kv-transport", choices=["auto", "nccl", "peer", "multicast"], default="auto",
                    help="N > 1: K/V of each block by NCCL all-gather, or by the QKV projection's own stores into "
                         "the peers' symmetric buffers (one per peer, or one multimem store through NVSwitch)")
    ap.add_argument("--only", default=None, help="--workload kernels: time this one kernel (e.g. layer_norm_affine)")
    ap.add_argument("--workload", choices=["stack", "stack_w8a8", "block", "attention", "attention262k", "conv",
                                           "forward", "vae", "released", "kernels"], default="stack")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in ("stack", "stack_w8a8", "block"):
        run_ours(args)
    elif args.workload == "conv":
        run_conv(args)
    elif args.workload == "forward":
        run_forward(args)
    elif args.workload == "vae":
        run_vae(args)
    elif args.workload == "released":
        run_released(args)
    elif args.workload == "kernels":
        run_kernels(args)
    else:
        run_attention(args, big=args.workload == "attention262k")


if __name__ == "__main__":
    main()
