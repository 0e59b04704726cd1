"""Benchmark of the sparse-DiT refinement torso on B200 (BASELINE configs[1] by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload stack|stack_w8a8|block|attention|attention262k|conv|forward|vae]

One step = one forward of the 24-block stack (C=1024, 16 heads x 64, GELU MLP 4x,
1370 condition tokens) over T=32,768 voxel tokens of one object in fp16, inputs
resident in HBM.  ``value`` is block tokens/s = blocks * T / step time (whole job,
max over ranks).  With N>1 GPUs (torchrun) the T tokens are split into N query
slices and every block all-gathers K/V over NCCL (strong scaling).

``--workload attention`` times the self-attention kernel alone at the same size
(T=32,768, 16x64 heads, fp16); ``--workload attention262k`` the high-resolution
config (262,144 tokens packed as 4 objects of 65,536, bf16, varlen), query-sharded
over the GPUs.  Both report attention TFLOP/s (4 * Nq * Nk * H * D per object).

``--workload conv`` times the cfg5 submanifold convolution; ``--workload forward`` the whole
refinement transformer around the same stack (input layer, two fine/low res blocks, the
24 blocks, the upsampling and output res blocks, LayerNorm + output layer) on a fine shell
whose downsampled level holds ~34k tokens, reporting transformer tokens/s.

Rank 0 prints one JSON line.  ``--impl reference`` times the CPU path instead: the
oracle port of the reference block (the reference itself is Python that cannot travel
to the GPU box), on the host's cores, on a row-sampled bounded sample of the same
workload.
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

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
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
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
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


def device_weights(device, seed: int = 100, blocks: int = BLOCKS) -> list[dict]:
    """``blocks`` blocks of N(0, 0.02) fp16 weights generated on the device (seeded)."""
    import torch

    from hi3d_b200.synthetic import BLOCK_LINEARS

    g = torch.Generator(device=device).manual_seed(seed)
    c, d = CHANNELS, CHANNELS // HEADS
    out = []
    for _ in range(blocks):
        w = {}
        for name, i_mult, o_mult in BLOCK_LINEARS:
            w[f"{name}.weight"] = (torch.randn((o_mult * c, i_mult * c), generator=g, device=device) * 0.02).half()
            w[f"{name}.bias"] = (torch.randn(o_mult * c, generator=g, device=device) * 0.02).half()
        w["cross_attn.to_kv.weight"] = (torch.randn((2 * c, c), generator=g, device=device) * 0.02).half()
        w["cross_attn.to_kv.bias"] = (torch.randn(2 * c, generator=g, device=device) * 0.02).half()
        w["modulation"] = torch.randn((1, 6 * c), generator=g, device=device) / c ** 0.5
        w["norm2.weight"] = torch.ones(c, device=device)
        w["norm2.bias"] = torch.zeros(c, device=device)
        w["self_attn.q_rms_norm.gamma"] = torch.ones((HEADS, d), device=device)
        w["self_attn.k_rms_norm.gamma"] = torch.ones((HEADS, d), device=device)
        out.append(w)
    return out


# ----------------------------------------------------------------------------- CPU baseline


_CPU_CACHE: dict = {}


def cpu_block_seconds(sample: int, seed: int = 0) -> tuple[float, dict]:
    """One fp32 CPU block at the full workload size, estimated from a row sample (oracle port)."""
    from hi3d_b200 import synthetic
    from oracle import ops

    if "block" not in _CPU_CACHE:
        coords, cos, sin, x, mod, cond = make_inputs(seed)
        w = synthetic.block_weights(CHANNELS, CHANNELS, HEADS, seed=seed + 5)
        _CPU_CACHE["block"] = (w, x, mod, cos, sin, cond)
    w, x, mod, cos, sin, cond = _CPU_CACHE["block"]
    return ops.block_seconds_sampled(w, x, mod, cos, sin, cond, HEADS, sample=sample, seed=seed)


def cpu_attention_tflops(big: bool, sample: int = 256) -> tuple[float, str]:
    """fp32 numpy attention of ``sample`` query rows against one whole object (all heads),
    scaled to TFLOP/s with the same 4 * Nq * Nk * H * D count as the GPU arm."""
    per = 65536 if big else T_TOKENS
    d = CHANNELS // HEADS
    if ("attn", big) not in _CPU_CACHE:
        rng = np.random.default_rng(7)
        _CPU_CACHE[("attn", big)] = tuple(rng.standard_normal((HEADS, n, d)).astype(np.float32)
                                          for n in (sample, per, per))
    q, k, v = _CPU_CACHE[("attn", big)]
    t0 = time.perf_counter()
    for h in range(HEADS):
        s = q[h] @ k[h].T * np.float32(d ** -0.5)
        p = np.exp(s - s.max(-1, keepdims=True))
        _ = (p / p.sum(-1, keepdims=True)) @ v[h]
    secs = time.perf_counter() - t0
    return 4.0 * sample * per * HEADS * d / secs / 1e12, f"{sample} query rows x {per} keys x {HEADS} heads, fp32"


def forward_inputs():
    from hi3d_b200 import synthetic

    if "fwd" not in _CPU_CACHE:
        coords = synthetic.shell_coords(FWD_FINE, FWD_GRID, FWD_RADIUS, FWD_THICK, seed=1)
        feats = synthetic.features(coords.shape[0], 32, seed=4, dtype=np.float32)
        cond = synthetic.features(COND, CHANNELS, seed=5, dtype=np.float32)
        _CPU_CACHE["fwd"] = (coords, feats, cond)
    return _CPU_CACHE["fwd"]


def cpu_forward_seconds(sample: int = 512) -> tuple[float, str]:
    """One fp32 CPU forward of the whole transformer (oracle port): the embedding and I/O stages
    run in full at the workload size; the 24 blocks are the row-sampled block estimate on the
    low level, times 24."""
    from hi3d_b200 import synthetic
    from oracle import ops

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
    bw = {k[len("blocks.0."):]: v for k, v in w.items() if k.startswith("blocks.0.")}
    blk_s, _ = ops.block_seconds_sampled(bw, x, mod, cos, sin, cond, HEADS, sample=sample, seed=0)
    desc = (f"whole transformer fp32 (numpy oracle port): embedding + I/O stages in full on {coords.shape[0]} fine "
            f"voxels ({io_s:.1f} s), plus {BLOCKS} x one block on {low.shape[0]} low tokens estimated from "
            f"{sample} sampled query rows ({blk_s:.1f} s each)")
    return io_s + BLOCKS * blk_s, desc


def cpu_conv_tflops(sample: int = 20000) -> tuple[float, str]:
    """fp32 numpy gather-GEMM of ``sample`` output rows of the cfg5 convolution (TFLOP/s over the
    present neighbour pairs, as the GPU arm counts them)."""
    from hi3d_b200 import synthetic
    from oracle import ops

    if "conv" not in _CPU_CACHE:
        n, c = 200_000, 256
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


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count()
    if args.workload in ("stack", "stack_w8a8", "block"):
        sample = 512
        secs = []
        for i in range(args.warmup + args.steps):
            s, _ = cpu_block_seconds(sample, seed=0)
            if i >= args.warmup:
                secs.append(s)
        per_block = statistics.median(secs)
        value, unit, metric = T_TOKENS / per_block, "tokens/s", "block_tokens_per_s"
        ms_step = per_block * BLOCKS * 1e3
        desc = (f"one fp32 block at T={T_TOKENS} per step (numpy oracle port of the reference block): K/V side on "
                f"all rows, {sample} sampled query rows for the rest, scaled by T/{sample}")
        workload = f"cfg1 block on CPU: T={T_TOKENS}, C={CHANNELS}, H={HEADS}x64, L={COND}"
    elif args.workload == "forward":
        secs = []
        for i in range(args.warmup + args.steps):
            sec, desc = cpu_forward_seconds()
            if i >= args.warmup:
                secs.append(sec)
        from oracle import ops

        n_low = ops.downsample_structure(forward_inputs()[0])[0].shape[0]
        per = statistics.median(secs)
        value, unit, metric, ms_step = n_low / per, "tokens/s", "forward_tokens_per_s", per * 1e3
        workload = f"whole transformer on CPU: {FWD_FINE} fine voxels, {n_low} low tokens, {BLOCKS} blocks"
    elif args.workload in ("conv", "vae"):
        vals = []
        for i in range(args.warmup + args.steps):
            v, desc = cpu_conv_tflops()
            if i >= args.warmup:
                vals.append(v)
        value, unit, ms_step = statistics.median(vals), "TFLOP/s", None
        metric = "sparse_conv_tflops" if args.workload == "conv" else "vae_conv_gn_swish_tflops"
        workload = "cfg5 submanifold conv on CPU (the convolution that dominates both workloads)"
    else:
        big = args.workload == "attention262k"
        vals = []
        for i in range(args.warmup + args.steps):
            v, desc = cpu_attention_tflops(big)
            if i >= args.warmup:
                vals.append(v)
        value, unit, metric = statistics.median(vals), "TFLOP/s", "attention_tflops"
        ms_step = None
        workload = "cfg4 self-attention on CPU" if big else "cfg1 self-attention on CPU"
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "blocks": BLOCKS},
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm


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
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()

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
        stack = hdist.ShardedBlockStack(weights, HEADS)
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
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
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
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
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
        "config": {"workload": (f"cfg2: W8A8 {BLOCKS}-block stack fwd (int8 signed-H64 activations, int8 rotated "
                                f"weights, int32 accumulate, fp16 dequant), T={T_TOKENS}, C={CHANNELS}, "
                                f"{HEADS}x{CHANNELS // HEADS} heads, {COND} cond tokens"
                                if args.workload == "stack_w8a8" else
                                f"cfg1: {nblocks}-block sparse-DiT stack fwd, T={T_TOKENS} shell tokens in {GRID}^3, "
                                f"C={CHANNELS}, {HEADS}x{CHANNELS // HEADS} heads, {COND} cond tokens, fp16"),
                   "blocks": nblocks, "tokens": T_TOKENS, "parallelism": f"query-sharded x{world}" if world > 1 else "none",
                   "l2": "inputs larger than L2 (705 MB of weights + activations per step)"},
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": x_host.numel() * 2,
                "d2h_bytes_per_step": out_host.numel() * 2},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "attention_tflops": achieved,
    }
    if rank == 0 and world == 1:
        secs, phases = cpu_block_seconds(1024, seed=0)
        cpu_value = T_TOKENS / secs
        line["cpu_baseline"] = {"value": cpu_value, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"one fp32 block at T={T_TOKENS} (numpy oracle port): K/V side on all "
                                          f"rows, 1024 sampled query rows for the rest, scaled by T/1024",
                                "seconds_per_block": secs}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_attention(args, big: bool) -> None:
    """Self-attention kernel alone: cfg1 (T=32768 fp16, one object) or cfg4 (4 x 65536 bf16 varlen)."""
    import torch
    import torch.distributed as dist

    from hi3d_b200 import _lib, attention

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()
    d = CHANNELS // HEADS
    if big:
        objects, per, dtype = 4, 65536, torch.bfloat16
    else:
        objects, per, dtype = 1, T_TOKENS, torch.float16
    total = objects * per
    g = torch.Generator(device=dev).manual_seed(7)
    # RoPE'd, RMS-normalised queries/keys have per-head norm sqrt(D): unit-variance entries
    k = torch.randn((total, HEADS, d), generator=g, device=dev).to(dtype)
    v = torch.randn((total, HEADS, d), generator=g, device=dev).to(dtype)
    # query rows of this rank: a contiguous slice of every object (keys stay per object)
    if per % world:
        raise ValueError("tokens per object must divide by the number of GPUs")
    ql = per // world
    q = torch.randn((objects * ql, HEADS, d), generator=g, device=dev).to(dtype)
    cu_q = torch.arange(0, objects + 1, device=dev, dtype=torch.int32) * ql
    cu_k = torch.arange(0, objects + 1, device=dev, dtype=torch.int32) * per
    out = torch.empty_like(q)
    flops = 4.0 * objects * ql * per * HEADS * d  # per rank per launch

    def step():
        attention.flash_attn_varlen(q, k, v, cu_q, cu_k, ql, d ** -0.5, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    _lib.LAUNCHES[0] = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    launches = _lib.LAUNCHES[0]
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    tflops = flops * world / (ms_step / 1e3) / 1e12
    per_gpu = flops / (ms_step / 1e3) / 1e12
    peaks = _peaks()
    # end to end: q/k/v from pinned host memory, output back to the host
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty_like(hq).pin_memory()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        dq, dk, dv = (t.to(dev, non_blocking=True) for t in (hq, hk, hv))
        hout.copy_(attention.flash_attn_varlen(dq, dk, dv, cu_q, cu_k, ql, d ** -0.5), non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    name = "flash_attn_fwd_cfg4" if big else "flash_attn_fwd_cfg1"
    cpu = None
    if rank == 0 and world == 1:
        cv, cdesc = cpu_attention_tflops(big)
        cpu = {"value": cv, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port", "sample": cdesc}
    line = {
        "metric": "attention_tflops", "value": tflops, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16" if big else "f16", "data": "synthetic",
        "config": {"workload": (f"cfg4: self-attention, {objects} objects x {per} tokens varlen, {HEADS}x{d} heads, bf16"
                                if big else f"cfg1: self-attention, T={per}, {HEADS}x{d} heads, fp16"),
                   "tokens": total, "parallelism": f"query-sharded x{world}" if world > 1 else "none",
                   "l2": "inputs larger than L2" if total * HEADS * d * 2 * 3 > 126e6 else "inputs fit in L2"},
        "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": per_gpu / peaks["bf16_tflops"], "traffic": _profile_traffic(name),
                     "peak_source": f"{peaks['source']} bf16_tflops (burst; kernel timed alone)"},
        "e2e": {"value": flops * world / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": (q.numel() + k.numel() + v.numel()) * 2,
                "d2h_bytes_per_step": out.numel() * 2},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
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
    n, c = 200_000, 256
    coords = synthetic.shell_coords(n, 128, 48, 4, seed=5)
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn((n, c), generator=g, device=dev).half()
    w = (torch.randn((c, 3, 3, 3, c), generator=g, device=dev) * 0.02).half()
    b = (torch.randn(c, generator=g, device=dev) * 0.02).half()
    cdev = torch.from_numpy(coords).to(dev)
    for _ in range(3):
        level = sparse.Level(cdev, sparse.neighbour_table(cdev))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        table = sparse.neighbour_table(cdev)
    e1.record()
    torch.cuda.synchronize()
    map_ms = e0.elapsed_time(e1) / args.steps
    mask = level.tap_mask
    pairs = int((level.table < n).sum().item())
    step = lambda: sparse.conv(x, level.table, w, b, tap_mask=mask)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.LAUNCHES[0] = 0
    with ClockSampler(0) as clocks:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    launches = _lib.LAUNCHES[0]
    ms = e0.elapsed_time(e1) / args.steps
    flops = 2.0 * c * c * pairs
    dense_flops = 2.0 * 27 * n * c * c
    peaks = _peaks()
    hx = x.cpu().pin_memory()
    hout = torch.empty((n, c), dtype=torch.float16).pin_memory()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        hout.copy_(sparse.conv(hx.to(dev, non_blocking=True), level.table, w, b, tap_mask=mask), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    line = {
        "metric": "sparse_conv_tflops", "value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"cfg5: submanifold 3x3x3 conv, {n} shell voxels in 128^3, {c}->{c} channels, fp16",
                   "pairs": pairs, "dense_equivalent_tflops": dense_flops / (ms / 1e3) / 1e12,
                   "neighbour_map_ms": map_ms, "lookups_per_s": 27 * n / (map_ms / 1e3),
                   "l2": "inputs larger than L2 (102 MB features + 102 MB output)"},
        "roofline": {"bound": "tensor", "achieved": flops / (ms / 1e3) / 1e12, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                     "traffic": _profile_traffic("sparse_conv_cfg5"),
                     "peak_source": f"{peaks['source']} bf16_tflops (burst)"},
        "e2e": {"value": flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": n * c * 2,
                "d2h_bytes_per_step": n * c * 2},
        "gpu_launches": launches, "clocks": clocks.summary(),
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
        "config": {"workload": (f"whole refinement transformer fwd: {coords.shape[0]} fine shell voxels in "
                                f"{FWD_GRID}^3 -> {n_low} low tokens, I/O stage {FWD_IO} channels, {BLOCKS} blocks "
                                f"C={CHANNELS} {HEADS}x{CHANNELS // HEADS} heads, {COND} cond tokens, fp16 torso"),
                   "fine_voxels": int(coords.shape[0]), "low_tokens": n_low, "io_stages_ms": io_ms,
                   "stack_ms": ms - io_ms, "guided_batch2_ms": guided_ms,
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
    secs, desc = cpu_forward_seconds()
    line["cpu_baseline"] = {"value": n_low / secs, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                            "sample": desc}
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
    ap.add_argument("--workload", choices=["stack", "stack_w8a8", "block", "attention", "attention262k", "conv",
                                           "forward", "vae"], default="stack")
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
    else:
        run_attention(args, big=args.workload == "attention262k")


if __name__ == "__main__":
    main()
