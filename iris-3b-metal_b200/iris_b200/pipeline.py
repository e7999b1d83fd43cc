"""End-to-end text-state -> image-sample entry point on one GPU.

The reference's ``IrisPipeline.__call__`` (``src/iris_metal/pipeline.py:265-330``)
encodes prompts with Qwen3-VL, adapts them once, draws CPU-seeded noise, runs
the sampler and returns images. Prompt encoding is outside this build; this
pipeline starts from text-encoder states (or adapted text) and keeps the rest:
host noise copied in, text adapted once per call, the sampler on the device
(the Turbo few-step guided Euler loop, or with ``steps`` the Original model's
multistep DPM-Solver++), ``require_finite`` on the pre-clamp sample, the
result copied back.
"""

from __future__ import annotations

import torch

from iris_b200.model import CudaIris, require_finite
from iris_b200.sampling import TURBO_SIGMAS, FlowDPMSolver, euler_cfg


class DenoisePipeline:
    def __init__(
        self,
        engine: CudaIris,
        cfg_scale: float = 3.0,
        sigmas=TURBO_SIGMAS,
        cfg_interval=(0.0, 1.5),
        *,
        steps: int | None = None,
        order: int = 2,
        shift: float = 1.0,
    ):
        """``steps=None``: the few-step Euler loop at ``sigmas`` (Turbo,
        ``src/iris3b/sampling.py:98-138``). ``steps=N``: ``FlowDPMSolver.sample``
        with ``N`` steps of ``order`` on the ``shift``-ed grid (the Original
        model's loop, ``src/iris3b/flow/solver.py:112-141``; its default CFG
        interval there is ``(0, 1)``)."""
        self.engine = engine
        self.cfg_scale = cfg_scale
        self.sigmas = tuple(sigmas)
        self.cfg_interval = cfg_interval
        self.steps, self.order, self.shift = steps, order, shift

    @torch.no_grad()
    def __call__(
        self,
        noise: torch.Tensor,
        cond_states: torch.Tensor,
        uncond_states: torch.Tensor | None,
        *,
        adapted: bool = False,
        out: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """``noise``: ``[k, 3, H, W]`` (host or device); text: encoder states
        ``[k, T, text_dim]`` / ``[1, T, text_dim]`` (or adapted ``[.., T, D]`` with
        ``adapted=True``). Returns the clamped sample, in ``out`` when given
        (e.g. pinned host memory), else on the noise's device."""
        if self.steps is not None and self.steps < 1:
            raise ValueError("DenoisePipeline: steps must be at least 1")
        if self.steps is None and not self.sigmas:
            raise ValueError("DenoisePipeline: sigmas must not be empty")
        dev = self.engine.device
        x = noise.to(dev, non_blocking=True)
        images = x.shape[0]
        if adapted:
            cond = cond_states.to(dev)
            uncond = None if uncond_states is None else uncond_states.to(dev)
        else:
            cond = self.engine.encode_text(cond_states)
            uncond = None if uncond_states is None else self.engine.encode_text(uncond_states)
        # one prompt (or one unconditional row) for every image, as the reference expands them
        # (src/iris_metal/pipeline.py:297-298)
        if cond.shape[0] not in (1, images):
            raise ValueError(f"cond text has {cond.shape[0]} rows for {images} images")
        cond = cond.expand(images, -1, -1)
        if uncond is not None:
            if uncond.shape[0] not in (1, images):
                raise ValueError(f"uncond text has {uncond.shape[0]} rows for {images} images")
            uncond = uncond.expand(images, -1, -1)
        if self.steps is None:
            sample = euler_cfg(
                self.engine, x, cond, uncond, cfg_scale=self.cfg_scale, sigmas=self.sigmas,
                cfg_interval=self.cfg_interval, check=require_finite,
            )  # fmt: skip
        else:
            solver = FlowDPMSolver(self.engine, cfg_scale=self.cfg_scale, cfg_interval=self.cfg_interval)
            sample = require_finite(solver.sample(x, cond, uncond, steps=self.steps, order=self.order, shift=self.shift))
        sample = sample.clamp(-1, 1)  # out of place: never the caller's noise tensor
        if out is not None:
            out.copy_(sample, non_blocking=True)
            return out
        return sample.to(noise.device)
