"""The flow-matching sampler: schedule and guidance against the upstream scheduler (CPU), and
a guided Heun pass on the B200 model against the fp32 oracle sampler (GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN, rel_l2

from hi3d_b200 import sampler
from oracle import ops

CASES = ((25, 34316), (12, 4000), (25, 1000), (3, 1500), (40, 262144))


@pytest.mark.parametrize("steps,tokens", CASES)
def test_schedule_bit_exact_vs_upstream(steps, tokens):
    g = np.load(GOLDEN / "schedule.npz")
    sigmas, hats = sampler.flow_schedule(steps, tokens)
    assert np.array_equal(sigmas, g[f"sigmas_{steps}_{tokens}"])
    assert np.array_equal(hats, g[f"hats_{steps}_{tokens}"])


def test_guidance_scale_vs_upstream():
    """The reference evaluates the upstream guidance in float32 (pipeline.py:75-82), as the
    upstream tensor form does on float32 model times (t = float32(0.7) is guided)."""
    g = np.load(GOLDEN / "schedule.npz")
    ours = np.array([sampler.guidance_scale(t) for t in g["guidance_t"]])
    assert np.array_equal(np.float32(ours), np.float32(g["guidance"]))
    assert [sampler.guidance_scale(t) for t in (1.0, 0.7, 0.6999)] == [4.0, float(np.float32(10) * np.float32(0.7) ** 2), 1.0]
    assert ops.guidance_scale_f32(0.85) == sampler.guidance_scale(0.85)


def test_schedule_rejects_bad_arguments():
    with pytest.raises(ValueError):
        sampler.flow_schedule(0, 100)
    with pytest.raises(ValueError):
        sampler.flow_schedule(5, 0)


@pytest.mark.gpu
@pytest.mark.parametrize("scheduler", ["heun", "euler"])
def test_guided_pass_matches_oracle(scheduler):
    from test_model_gpu import _forward_setup

    g, w, heads, m, geo = _forward_setup()
    steps = 2
    noise = np.random.default_rng(31).standard_normal(g["feats"].shape).astype(np.float32)
    kvs = m.prepare(torch.from_numpy(g["cond"]).cuda())
    got = sampler.sample(m, kvs, geo, torch.from_numpy(noise), steps=steps, scheduler=scheduler).cpu().numpy()
    sigmas, hats = sampler.flow_schedule(steps, noise.shape[0])
    assert hats[0] >= 1.0  # the first evaluation is guided (both branches)
    want = ops.sample_f32(w, noise, g["coords"], g["cond"], heads, sigmas, hats, scheduler=scheduler)
    assert rel_l2(got, want) < 2e-3
    assert rel_l2(got - noise, want - noise) < 1e-2
