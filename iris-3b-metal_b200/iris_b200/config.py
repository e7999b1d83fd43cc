"""Model configuration with the reference's field names and defaults.

Mirrors ``ModelConfig`` / ``PixelStageConfig`` of ``src/iris3b/config.py:25-120``
(the fields the per-step forward reads), so a config built for the upstream
model and one built here are interchangeable by field name.
"""

from __future__ import annotations

from dataclasses import dataclass, field, fields, replace


@dataclass
class PixelStageConfig:
    enabled: bool = True
    depth: int = 4
    hidden_size: int = 16
    attn_hidden_size: int = 1280
    num_heads: int = 10
    mlp_ratio: float = 4.0
    modulation: str = "post"
    abs_pos_embed: bool = True


@dataclass
class ModelConfig:
    block: str = "single_stream"
    dual_depth: int = 8
    final_block_text: str = "keep"
    hidden_size: int = 2560
    depth: int = 24
    num_heads: int = 20
    num_kv_heads: int | None = 5
    gated_attention: bool = True
    sandwich_norm: bool = True
    patch_size: int = 16
    in_channels: int = 3
    mlp_ratio: float = 4.0
    qkv_bias: bool = False
    qk_norm: bool = True
    norm_eps: float = 1e-6
    modulation: str = "shared_bias"
    timestep_max_period: float = 10.0
    rope_theta: float = 10000.0
    rope_scale: float = 16.0
    rope_aspect: str = "isotropic"
    rope_frame_pairs: int = 0
    text_rope: bool = True
    text_rope_theta: float = 10000.0
    text_abs_pos_embed: bool = True
    text_dim: int = 2560
    text_len: int = 300
    text_adapter: str = "lap_blocks2"
    text_lap_num_layers: int = 12
    text_lap_num_heads: int = 32
    text_lap_mlp_ratio: float = 1.3
    pixel: PixelStageConfig = field(default_factory=PixelStageConfig)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def kv_heads(self) -> int:
        return self.num_heads if self.num_kv_heads is None else self.num_kv_heads

    @property
    def swiglu_hidden(self) -> int:
        # SwiGLU 2/3 width rule, src/iris3b/nn/mlp.py:33
        return int(2 * int(self.hidden_size * self.mlp_ratio) / 3)


def baseline_step_config() -> ModelConfig:
    """The benchmark model: the released hybrid topology (8 dual + 16 single-stream
    blocks, gated, sandwich-normed, shared-bias adaLN, post-modulated PiT) at
    d = 3072 with 24 MHA heads of 128 (fused QKV), SwiGLU 8192, 256 text tokens
    through the linear adapter."""
    return ModelConfig(hidden_size=3072, num_heads=24, num_kv_heads=None, text_len=256, text_adapter="linear")


def from_any(cfg) -> ModelConfig:
    """A ``ModelConfig`` from any object with the reference's field names."""
    if isinstance(cfg, ModelConfig):
        return cfg
    pix = cfg.pixel
    pixel = PixelStageConfig(**{f.name: getattr(pix, f.name) for f in fields(PixelStageConfig) if hasattr(pix, f.name)})
    values = {f.name: getattr(cfg, f.name) for f in fields(ModelConfig) if f.name != "pixel" and hasattr(cfg, f.name)}
    return replace(ModelConfig(), **values, pixel=pixel)
