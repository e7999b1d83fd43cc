"""Samplers that call the denoiser once per step.

* :func:`euler_cfg`: the Turbo deterministic flow-Euler loop of
  ``generate_few_step`` (``src/iris3b/sampling.py:98-138``) with the CFG
  combine of ``FlowDPMSolver._model_out`` (``src/iris3b/flow/solver.py:58-74``)
  on the doubled batch ``[uncond; cond]``. The combine and the Euler update are
  one fused kernel per step (``iris_cfg_euler``).
* :class:`FlowDPMSolver`: ``src/iris3b/flow/solver.py:36-141`` with the same
  API; it drives any ``model_fn`` (e.g. :class:`iris_b200.model.CudaIris`) on
  CUDA tensors. The CFG combine, the x0 prediction and the first- or
  second-order update of each step are one fused kernel (``iris_dpm_update``),
  whose coefficients come from the host in double precision.
"""

from __future__ import annotations

import math
from collections.abc import Callable

import torch

from iris_b200 import _lib
from iris_b200.kernels import stream_of

TURBO_SIGMAS = (1.0, 0.938, 0.833, 0.625)  # src/iris_metal/turbo.py:12
ModelFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


@torch.no_grad()
def euler_cfg(
    model_fn: ModelFn,
    noise: torch.Tensor,
    cond: torch.Tensor,
    uncond: torch.Tensor | None,
    cfg_scale: float = 3.0,
    sigmas=TURBO_SIGMAS,
    num_timesteps: int = 1000,
    cfg_interval=(0.0, 1.5),
    check: Callable[[torch.Tensor], object] | None = None,
) -> torch.Tensor:
    """Pre-clamp final sample of the few-step Euler loop. CFG applies at sigmas
    strictly inside ``cfg_interval`` (``solver.py:62-63``); ``cond``/``uncond`` are
    adapted text ``[k, T, D]`` (``uncond`` may be ``[1, T, D]``). ``text`` is built
    once and reused by every guided call (``reuse_cfg_text``)."""
    x = noise.to(torch.float32).contiguous()
    images = x.shape[0]
    per_image = x[0].numel()
    lo, hi = cfg_interval
    guided_text = None
    if uncond is not None and cfg_scale != 1.0:
        guided_text = torch.cat([uncond.expand(images, -1, -1), cond], dim=0).contiguous()
    x_in = torch.empty((2 * images, *x.shape[1:]), device=x.device, dtype=torch.float32)
    for i, sigma in enumerate(sigmas):
        guided = guided_text is not None and lo < float(sigma) < hi
        t_model = float(sigma) * num_timesteps
        if guided:
            x_in[:images].copy_(x)
            x_in[images:].copy_(x)
            v = model_fn(x_in, torch.full((2 * images,), t_model, device=x.device, dtype=torch.float32), guided_text)
        else:
            v = model_fn(x, torch.full((images,), t_model, device=x.device, dtype=torch.float32), cond)
        sigma_next = float(sigmas[i + 1]) if i + 1 < len(sigmas) else -1.0
        x_next = torch.empty_like(x)
        _lib.call(
            "iris_cfg_euler", v.data_ptr(), x.data_ptr(), x_next.data_ptr(), images, per_image, float(cfg_scale),
            float(sigma), sigma_next, int(guided), stream_of(x),
        )  # fmt: skip
        x = x_next
    if check is not None:
        check(x)
    return x


def _lambda(t: float) -> float:
    return math.inf if t <= 0.0 else math.log((1.0 - t) / t)


def shift_sigma(sigma, shift: float):
    """``src/iris3b/flow/schedule.py:24-25``."""
    return shift * sigma / (1 + (shift - 1) * sigma)


class FlowDPMSolver:
    """Multistep DPM-Solver++ on the rectified-flow schedule (v-prediction),
    ``src/iris3b/flow/solver.py:36-141``."""

    def __init__(
        self,
        model_fn: ModelFn,
        num_timesteps: int = 1000,
        cfg_scale: float = 1.0,
        cfg_interval: tuple[float, float] = (0.0, 1.0),
        prediction: str = "v",
        reuse_cfg_text: bool = False,
    ):
        if prediction not in ("v", "x"):
            raise ValueError(f"unknown prediction type '{prediction}'")
        self.model_fn = model_fn
        self.num_timesteps = num_timesteps
        self.cfg_scale = cfg_scale
        self.cfg_interval = cfg_interval
        self.prediction = prediction
        self.reuse_cfg_text = reuse_cfg_text
        self._cfg_text: torch.Tensor | None = None

    def _model_call(self, x, t: float, cond, uncond) -> tuple[torch.Tensor, bool]:
        """The model output for ``x`` at ``t``: ``[uncond; cond]`` rows (and True)
        when CFG applies at ``t`` (``solver.py:58-74``), else the plain rows."""
        lo, hi = self.cfg_interval
        use_cfg = uncond is not None and self.cfg_scale != 1.0 and lo < t < hi
        rows = 2 * x.shape[0] if use_cfg else x.shape[0]
        t_model = torch.full((rows,), t * self.num_timesteps, device=x.device, dtype=torch.float32)
        if not use_cfg:
            return self.model_fn(x, t_model, cond), False
        text = self._cfg_text
        if text is None:
            text = torch.cat([uncond, cond], dim=0)
            if self.reuse_cfg_text:
                self._cfg_text = text
        return self.model_fn(torch.cat([x, x], dim=0), t_model, text), True

    @staticmethod
    def time_grid(steps: int, shift: float) -> list[float]:
        sigma = 1.0 - torch.linspace(1.0, 0.001, steps + 1, dtype=torch.float64)
        return shift_sigma(sigma, shift).flip(0).tolist()

    @staticmethod
    def coefficients(s: float, t: float, prev_s: float | None) -> tuple[float, float, float]:
        """``(a, b, c)`` of ``x_next = a x + b x0 + c (x0 - x0_prev)``: the first-order
        update (``prev_s`` None, ``solver.py:84-88``) or the second-order one with
        the previous step at ``prev_s`` (``solver.py:90-109``), in double precision."""
        if prev_s is None:
            phi1 = math.expm1(-(_lambda(t) - _lambda(s)))
            return t / s, -(1.0 - t) * phi1, 0.0
        lam_t, lam_0, lam_1 = _lambda(t), _lambda(s), _lambda(prev_s)
        h, h0 = lam_t - lam_0, lam_0 - lam_1
        phi1 = math.expm1(-h)
        return t / s, -(1.0 - t) * phi1, -0.5 * (1.0 - t) * phi1 / (h0 / h)

    @torch.no_grad()
    def sample(self, z, cond, uncond=None, steps: int = 50, order: int = 2, shift: float = 1.0):
        """Integrate from noise ``z`` (CUDA, fp32 ``[k, ...]``) to a sample; the
        order ramps up over the first steps and back down at the end, so the
        last (t = 0) update is the first-order x <- x0 projection."""
        if not z.is_cuda:
            raise ValueError("FlowDPMSolver.sample runs on CUDA tensors")
        grid = self.time_grid(steps, shift)
        x = z.to(torch.float32).contiguous()
        self._cfg_text = None
        images, per_image = x.shape[0], x[0].numel()
        x0_prev, s_prev = None, None
        for i in range(1, steps + 1):
            s, t = grid[i - 1], grid[i]
            out, guided = self._model_call(x, s, cond, uncond)
            step_order = min(i, order, steps + 1 - i)
            a, b, c = self.coefficients(s, t, s_prev if step_order == 2 else None)
            x0 = torch.empty_like(x)
            x_next = torch.empty_like(x)
            _lib.call(
                "iris_dpm_update", out.contiguous().data_ptr(), x.data_ptr(),
                x0_prev.data_ptr() if (c != 0.0 and x0_prev is not None) else None, x0.data_ptr(),
                x_next.data_ptr(), images, per_image, float(self.cfg_scale), int(guided), float(s),
                int(self.prediction == "x"), float(a), float(b), float(c), stream_of(x),
            )  # fmt: skip
            x, x0_prev, s_prev = x_next, x0, s
        self._cfg_text = None
        return x
