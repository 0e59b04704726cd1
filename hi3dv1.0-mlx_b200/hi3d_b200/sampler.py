"""Flow-matching sampler around the B200 transformer: the caller of the hot path.

Mirrors ``Hi3DPipelineMLX.sample`` (src/hi3d_mac/mlx_backend/pipeline.py:156-229) with the
upstream schedule (``FlowMatchSchedule.set_timesteps``,
src/sparc3d/schedulers/schedule.py:132-190, 241-242) and integrators (Heun:
src/sparc3d/schedulers/flow_match_heun.py:20-80; Euler; and the reference's two-step
Adams-Bashforth variant):

* the token-count-dependent sigma schedule, ``sigma_hat = sigma * (1 + gamma)`` model times;
* classifier-free guidance with the zero condition, scale 4 at t >= 1, ``10 t^2`` on [0.7, 1)
  and 1 below (no zero-condition branch then), evaluated in float32 as the reference does
  (pipeline.py:75-82);
* one velocity evaluation = one call of :class:`hi3d_b200.model.Sparc3DTransformer` on the
  ``[condition, zero condition]`` batch (the stack runs both branches as one batch, sharing
  the first block's self-attention, whose input is identical in both branches).

The sample updates are fp32 element-wise operations on ``[N, 32]`` tensors (torch; about
1e-5 of a velocity evaluation).  The condition K/V of every block are projected once per
pass (:meth:`Sparc3DTransformer.prepare`).
"""

from __future__ import annotations

import numpy as np
import torch

SIGMA_MIN = 0.002
TIME_RESCALE_FACTOR = 2.0
GUIDANCE_START = 0.7


def _rational_rescale(t: torch.Tensor, factor: float) -> torch.Tensor:
    return factor * t / (1.0 + (factor - 1.0) * t)


def flow_schedule(steps: int, num_tokens: int, sigma_min: float = SIGMA_MIN,
                  time_rescale_factor: float = TIME_RESCALE_FACTOR) -> tuple[np.ndarray, np.ndarray]:
    """``(sigmas [steps + 1], sigma_hats [steps])`` float32 of the token-dependent schedule
    (schedule.py:132-190, 241-242): base times ``linspace(1, 0)`` rescaled by
    ``time_rescale_factor``, warped by the token-count factor ``clamp((19 n - 20000) / (3 n + 60000), 1, 5)``,
    ``sigma = sigma_min + (1 - sigma_min) * warped``, and the model times inflated by
    ``gamma = 0.04`` while ``warped > 0.985``, else 0.002."""
    if steps <= 0 or num_tokens <= 0:
        raise ValueError("steps and num_tokens must be positive")
    warp = max(1.0, min(5.0, (19.0 * num_tokens - 20000.0) / (3.0 * num_tokens + 60000.0)))
    base = torch.linspace(1.0, 0.0, steps + 1, dtype=torch.float32)
    warped = _rational_rescale(_rational_rescale(base, float(time_rescale_factor)), warp)
    sigmas = sigma_min + (1.0 - sigma_min) * warped
    gammas = torch.where(warped[:-1] > 0.985, torch.full_like(warped[:-1], 0.04),
                         torch.full_like(warped[:-1], 0.002))
    sigma_hats = sigmas[:-1] * (1.0 + gammas)
    return sigmas.numpy().astype(np.float32), sigma_hats.numpy().astype(np.float32)


def guidance_scale(t: float) -> float:
    """Effective zero-condition guidance scale at model time ``t`` in float32 (pipeline.py:75-82)."""
    t32 = np.float32(t)
    if t32 >= 1.0:
        return 4.0
    if t32 >= GUIDANCE_START:
        return float(np.float32(10.0) * (t32 * t32))
    return 1.0


def sample(model, kvs, geo, noise: torch.Tensor, steps: int = 25, scheduler: str = "heun",
           corrector_guidance: str = "full", latent_mean=None, latent_std=None) -> torch.Tensor:
    """Integrate the flow from ``noise [N, 32]`` (fp32) to latents, as ``Hi3DPipelineMLX.sample``
    (pipeline.py:156-229): ``scheduler`` ``heun`` (two evaluations per step), ``euler`` or ``ab2``;
    ``corrector_guidance`` ``full`` (the Heun corrector evaluates both branches) or ``reuse``
    (it reuses the predictor's guidance difference).  Returns ``x * latent_std + latent_mean``
    (identity when not given)."""
    if scheduler not in ("heun", "euler", "ab2") or corrector_guidance not in ("full", "reuse"):
        raise ValueError("scheduler in {heun, euler, ab2}, corrector_guidance in {full, reuse}")
    n = noise.shape[0]
    sigmas, sigma_hats = flow_schedule(steps, n)
    x = noise.to(model.device, torch.float32)
    last_delta = None

    def velocity(xs: torch.Tensor, t: np.float32, reuse: bool = False) -> torch.Tensor:
        nonlocal last_delta
        if t < GUIDANCE_START:
            return model(xs, float(t), geo, kvs)[0]
        if reuse and last_delta is not None:
            (pos,) = model(xs, float(t), geo, kvs)
            return pos + (guidance_scale(t) - 1.0) * last_delta
        pos, neg = model(xs, float(t), geo, kvs, negative=True)
        last_delta = pos - neg
        return neg + guidance_scale(t) * (pos - neg)

    previous = None
    for i in range(steps):
        t, t_next = sigma_hats[i], sigmas[i + 1]
        dt = float(np.float32(t - t_next))
        last_delta = None
        v1 = velocity(x, t)
        if scheduler == "heun":
            predicted = x - dt * v1
            v2 = velocity(predicted, t_next, reuse=corrector_guidance == "reuse")
            x = x - dt * (0.5 * (v1 + v2))
        elif scheduler == "ab2" and previous is not None:
            v0, t0 = previous
            ratio = dt / (2.0 * float(np.float32(t0 - t)))
            x = x - dt * (v1 + ratio * (v1 - v0))
        else:
            x = x - dt * v1
        previous = (v1, t)
    if latent_std is not None:
        x = x * torch.as_tensor(latent_std, dtype=torch.float32, device=x.device)
    if latent_mean is not None:
        x = x + torch.as_tensor(latent_mean, dtype=torch.float32, device=x.device)
    return x
