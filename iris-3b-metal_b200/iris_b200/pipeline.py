"""End-to-end text-state -> image-sample entry point on one GPU.

The reference's ``IrisPipeline.__call__`` (``src/iris_metal/pipeline.py:265-330``)
encodes prompts with Qwen3-VL, adapts them once, draws CPU-seeded noise, runs
the sampler and returns images. Prompt encoding is outside this build; this
pipeline starts from text-encoder states (or adapted text) and keeps the rest:
host noise copied in, text adapted once per call, the guided Euler loop on the
device, ``require_finite`` on the pre-clamp sample, the result copied back.
"""

from __future__ import annotations

import torch

from iris_b200.model import CudaIris, require_finite
from iris_b200.sampling import TURBO_SIGMAS, euler_cfg


class DenoisePipeline:
    def __init__(self, engine: CudaIris, cfg_scale: float = 3.0, sigmas=TURBO_SIGMAS, cfg_interval=(0.0, 1.5)):
        self.engine = engine
        self.cfg_scale = cfg_scale
        self.sigmas = tuple(sigmas)
        self.cfg_interval = cfg_interval

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
        dev = self.engine.device
        x = noise.to(dev, non_blocking=True)
        if adapted:
            cond = cond_states.to(dev)
            uncond = None if uncond_states is None else uncond_states.to(dev)
        else:
            cond = self.engine.encode_text(cond_states)
            uncond = None if uncond_states is None else self.engine.encode_text(uncond_states)
        sample = euler_cfg(
            self.engine, x, cond, uncond, cfg_scale=self.cfg_scale, sigmas=self.sigmas,
            cfg_interval=self.cfg_interval, check=require_finite,
        )  # fmt: skip
        sample = sample.clamp_(-1, 1)
        if out is not None:
            out.copy_(sample, non_blocking=True)
            return out
        return sample.to(noise.device)
