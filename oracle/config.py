"""Model configuration restated for the oracle.

Field names and defaults follow ``ModelConfig`` / ``PixelStageConfig`` in
``src/iris3b/config.py:25-120`` (only the fields the per-step forward reads).
"""

from dataclasses import dataclass, field, replace


@dataclass
class PixelConfig:
    """``PixelStageConfig``, ``src/iris3b/config.py:25-38``."""

    enabled: bool = True
    depth: int = 4
    hidden_size: int = 16
    attn_hidden_size: int = 1280
    num_heads: int = 10
    mlp_ratio: float = 4.0
    modulation: str = "post"
    abs_pos_embed: bool = True


@dataclass
class OracleConfig:
    """``ModelConfig``, ``src/iris3b/config.py:41-120``."""

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
    text_rope: bool = True
    text_rope_theta: float = 10000.0
    text_abs_pos_embed: bool = True
    text_dim: int = 2560
    text_len: int = 300
    text_adapter: str = "linear"
    text_lap_num_layers: int = 12
    text_lap_num_heads: int = 32
    text_lap_mlp_ratio: float = 1.3
    pixel: PixelConfig = field(default_factory=PixelConfig)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def kv_heads(self) -> int:
        return self.num_heads if self.num_kv_heads is None else self.num_kv_heads

    @property
    def swiglu_hidden(self) -> int:
        # src/iris3b/nn/mlp.py:33
        return int(2 * int(self.hidden_size * self.mlp_ratio) / 3)


def baseline_step_config() -> OracleConfig:
    """the released hybrid at d=3072, 24 MHA heads x 128,
    linear text adapter, 256 text tokens: ``replace(ModelConfig(), hidden_size=3072,
    num_heads=24, num_kv_heads=None, text_len=256, text_adapter="linear")`` over the
    released defaults of ``src/iris3b/config.py``."""
    return OracleConfig(hidden_size=3072, num_heads=24, num_kv_heads=None, text_len=256)


def tiny_cpu_config() -> OracleConfig:
    """``tests/tiny_config.py:7-26`` with d=256, 4 mmdit
    blocks, 4 heads x 64, patch 16, text 32 x 2560 (SwiGLU width 682)."""
    return OracleConfig(
        block="mmdit",
        dual_depth=0,
        hidden_size=256,
        depth=4,
        num_heads=4,
        num_kv_heads=None,
        gated_attention=False,
        sandwich_norm=False,
        patch_size=16,
        modulation="per_block",
        rope_aspect="square",
        text_dim=2560,
        text_len=32,
        text_adapter="linear",
        pixel=PixelConfig(depth=1, hidden_size=8, attn_hidden_size=64, num_heads=4, modulation="pre"),
    )


def released_topology(**overrides) -> OracleConfig:
    """``RELEASED_TOPOLOGY`` of ``tests/test_metal_engine.py:28-48`` (toy width,
    128-wide heads) with a linear text adapter; GQA 2:1 unless overridden."""
    base = OracleConfig(
        block="single_stream",
        dual_depth=1,
        hidden_size=256,
        depth=3,
        num_heads=2,
        num_kv_heads=1,
        gated_attention=True,
        sandwich_norm=True,
        patch_size=4,
        modulation="shared_bias",
        rope_aspect="isotropic",
        text_dim=64,
        text_len=16,
        text_adapter="linear",
        pixel=PixelConfig(depth=2, hidden_size=16, attn_hidden_size=256, num_heads=2, modulation="post"),
    )
    return replace(base, **overrides)
