"""Samplers that call the denoiser forward, restated (checker only).

* ``euler_cfg``: the Turbo deterministic flow-Euler loop of
  ``generate_few_step`` (``src/iris3b/sampling.py:98-138``) with the CFG
  combine of ``FlowDPMSolver._model_out`` (``src/iris3b/flow/solver.py:58-74``)
  on the doubled batch ``[uncond; cond]``; returns the pre-clamp sample.
* ``FlowDPMSolverOracle``: ``src/iris3b/flow/solver.py:36-141``.
"""

from __future__ import annotations

import math
from collections.abc import Callable

import torch

ModelFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
TURBO_SIGMAS = (1.0, 0.938, 0.833, 0.625)  # src/iris_metal/turbo.py:12


def cfg_velocity(model_fn: ModelFn, x, t_model: float, cond, uncond, cfg_scale: float):
    """``solver.py:67-74``: one call on ``[x; x]`` with text ``[uncond; cond]``."""
    if uncond is None or cfg_scale == 1.0:
        t = torch.full((x.shape[0],), t_model, device=x.device, dtype=torch.float32)
        return model_fn(x, t, cond)
    t = torch.full((2 * x.shape[0],), t_model, device=x.device, dtype=torch.float32)
    # one negative prompt serves every image, as the pipeline expands it (pipeline.py:297-300)
    uncond = uncond.expand(cond.shape[0], *uncond.shape[1:]) if uncond.shape[0] == 1 else uncond
    out = model_fn(torch.cat([x, x], dim=0), t, torch.cat([uncond, cond], dim=0))
    out_u, out_c = out.chunk(2, dim=0)
    return out_u + cfg_scale * (out_c - out_u)


def euler_cfg(
    model_fn: ModelFn,
    noise,
    cond,
    uncond,
    cfg_scale=3.0,
    sigmas=TURBO_SIGMAS,
    num_timesteps=1000,
    cfg_interval=(0.0, 1.5),
):
    """``sampling.py:125-137`` per sigma: ``clean = x - sigma v``; re-noise to the
    next sigma with the implied noise. Returns the pre-clamp final ``clean``.
    CFG applies at sigma strictly inside ``cfg_interval`` (``solver.py:62-63``)."""
    x = noise.float()
    sigma = torch.full((x.shape[0], 1, 1, 1), sigmas[0], device=x.device, dtype=torch.float32)
    clean = x
    lo, hi = cfg_interval
    for i in range(len(sigmas)):
        guided = uncond if lo < float(sigmas[i]) < hi else None
        out = cfg_velocity(model_fn, x, float(sigmas[i]) * num_timesteps, cond, guided, cfg_scale)
        # sigma.flatten() * 1000 in the reference is an fp32 product; float(s)*1000 rounds alike
        clean = x - sigma * out
        if i + 1 < len(sigmas):
            implied_noise = (x - (1 - sigma) * clean) / sigma
            sigma = torch.full_like(sigma, sigmas[i + 1])
            x = (1 - sigma) * clean + sigma * implied_noise
    return clean


def _lambda(t: float) -> float:
    """``solver.py:30-33``."""
    if t <= 0.0:
        return math.inf
    return math.log((1.0 - t) / t)


def shift_sigma(sigma, shift: float):
    """``src/iris3b/flow/schedule.py:24-25``."""
    return shift * sigma / (1 + (shift - 1) * sigma)


class FlowDPMSolverOracle:
    """``FlowDPMSolver`` (v-prediction), ``solver.py:36-141``."""

    def __init__(self, model_fn: ModelFn, num_timesteps=1000, cfg_scale=1.0, cfg_interval=(0.0, 1.0)):
        self.model_fn = model_fn
        self.num_timesteps = num_timesteps
        self.cfg_scale = cfg_scale
        self.cfg_interval = cfg_interval

    def _pred_x0(self, x, t, cond, uncond):
        lo, hi = self.cfg_interval
        use_cfg = uncond is not None and self.cfg_scale != 1.0 and lo < t < hi
        out = cfg_velocity(self.model_fn, x, t * self.num_timesteps, cond, uncond if use_cfg else None, self.cfg_scale)
        return x - t * out

    @staticmethod
    def time_grid(steps: int, shift: float) -> list[float]:
        sigma = 1.0 - torch.linspace(1.0, 0.001, steps + 1, dtype=torch.float64)
        return shift_sigma(sigma, shift).flip(0).tolist()

    @staticmethod
    def first_order(x, s, t, x0):
        h = _lambda(t) - _lambda(s)
        phi1 = math.expm1(-h)
        return (t / s) * x - (1.0 - t) * phi1 * x0

    @staticmethod
    def second_order(x, prev1, prev0, t):
        (s1, x0_1), (s0, x0_0) = prev1, prev0
        lam_t, lam_0, lam_1 = _lambda(t), _lambda(s0), _lambda(s1)
        h, h0 = lam_t - lam_0, lam_0 - lam_1
        r0 = h0 / h
        d = (x0_0 - x0_1) / r0
        phi1 = math.expm1(-h)
        return (t / s0) * x - (1.0 - t) * phi1 * x0_0 - 0.5 * (1.0 - t) * phi1 * d

    @torch.no_grad()
    def sample(self, z, cond, uncond=None, steps=50, order=2, shift=1.0):
        grid = self.time_grid(steps, shift)
        x = z
        history = []
        for i in range(1, steps + 1):
            s, t = grid[i - 1], grid[i]
            x0 = self._pred_x0(x, s, cond, uncond)
            history.append((s, x0))
            step_order = min(i, order, steps + 1 - i)
            if step_order == 1:
                x = self.first_order(x, s, t, x0)
            else:
                x = self.second_order(x, history[-2], history[-1], t)
            if len(history) > 2:
                history.pop(0)
        return x
