"""CPU-baseline timing of the oracle (the reference's fp32 PyTorch path,
restated) on a bounded sample of the benchmark workload. Used only by
``bench.py``'s CPU-baseline leg and its ``--impl reference`` arm.

A full 1024^2 step is ~68 TFLOP in fp32, minutes on host cores, so the sample
is one dual-stream block, one single-stream block and one pixel block at the
benchmark's batch and resolution; a forward is extrapolated as
``dual_depth * t_dual + (depth - dual_depth) * t_single + pixel_depth * t_pixel``
(the blocks are >99% of the FLOPs).
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from oracle import ops
from oracle.config import OracleConfig
from oracle.model import OracleModel
from oracle.params import STD, param_spec


def _sample_params(cfg: OracleConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    wanted = ("blocks.0.", f"blocks.{cfg.dual_depth}.", "pixel_blocks.0.", "modulation_cores.", "t_embedder.")
    gen = torch.Generator().manual_seed(seed)
    params = {}
    for name, shape, kind in param_spec(cfg):
        if name.startswith(wanted):
            v = torch.randn(shape, generator=gen) * STD
            params[name] = v + 1.0 if kind == "g" else v
    return params


class BlockSampler:
    """Inputs and parameters for timing one block of each kind on the CPU."""

    def __init__(self, cfg: OracleConfig, batch: int, height: int, width: int):
        self.cfg = cfg
        self.model = OracleModel(cfg, _sample_params(cfg))
        p = cfg.patch_size
        self.grid = (height // p, width // p)
        L = self.grid[0] * self.grid[1]
        gen = torch.Generator().manual_seed(1)
        d = cfg.hidden_size
        self.x = torch.randn(batch, L, d, generator=gen)
        self.y = torch.randn(batch, cfg.text_len, d, generator=gen)
        self.pixels = torch.randn(batch * L, p * p, cfg.pixel.hidden_size, generator=gen)
        self.s_cond = torch.randn(batch * L, d, generator=gen)
        t_emb = self.model.t_embed(torch.full((batch,), 625.0))
        self.cond = F.silu(t_emb)
        self.shared = {
            "img": self.model._lin(self.cond, "modulation_cores.adaln_img"),
            "txt": self.model._lin(self.cond, "modulation_cores.adaln_txt"),
        }
        self.rope_img, self.rope_txt, self.rope_pix = self.model.rope_tables(self.grid, cfg.text_len, "cpu")

    def dual(self):
        return self.model.dual_block(0, self.x, self.y, self.cond, self.rope_img, self.rope_txt, self.shared)

    def single(self):
        i = self.cfg.dual_depth
        return self.model.single_block(i, self.x, self.y, self.cond, self.rope_img, self.rope_txt, self.shared)

    def pixel(self):
        return self.model.pixel_block(0, self.pixels, self.s_cond, self.rope_pix, self.grid)

    def forward_seconds(self, repeats: int = 1) -> dict:
        """Seconds per block kind (median of ``repeats`` after one warm-up) and the
        extrapolated forward time."""
        out = {}
        with torch.no_grad():
            for name in ("dual", "single", "pixel"):
                fn = getattr(self, name)
                fn()
                times = []
                for _ in range(repeats):
                    start = time.perf_counter()
                    fn()
                    times.append(time.perf_counter() - start)
                out[name] = sorted(times)[len(times) // 2]
        cfg = self.cfg
        out["forward"] = (
            cfg.dual_depth * out["dual"] + (cfg.depth - cfg.dual_depth) * out["single"] + cfg.pixel.depth * out["pixel"]
        )
        return out


def sincos_check() -> bool:
    """Cheap self-test used by callers to confirm the oracle imports."""
    return ops.sincos_pos_embed_2d(16, 2, 2).shape == (4, 16)
