"""Weight sources for :class:`iris_b200.model.CudaIris`.

``CudaIris`` reads parameters by the reference's ``state_dict`` names from any
object with ``.cfg`` and ``.state_dict()`` -- the upstream ``IrisDiT`` or the
``IrisWeights`` container below, which loads a released checkpoint's
``model.safetensors`` (same key layout, ``src/iris_metal/loading.py:41-77``)
or synthesises random weights for benchmarking.
"""

from __future__ import annotations

from dataclasses import fields, replace
from pathlib import Path

import torch

from iris_b200.config import ModelConfig, PixelStageConfig, from_any


class IrisWeights:
    def __init__(self, cfg, state: dict[str, torch.Tensor]):
        self.cfg = from_any(cfg)
        self._state = state

    def state_dict(self) -> dict[str, torch.Tensor]:
        return self._state

    @classmethod
    def from_safetensors(cls, path: str | Path, cfg, device: torch.device | str = "cuda") -> "IrisWeights":
        """Every tensor of a ``model.safetensors`` file, moved to ``device`` one at a
        time (the engine repacks the matrices to BF16 once; gains, biases and
        tables stay as stored)."""
        from safetensors import safe_open

        state = {}
        with safe_open(str(path), framework="pt", device="cpu") as reader:
            for key in reader.keys():
                state[key] = reader.get_tensor(key).to(device)
        return cls(cfg, state)

    @classmethod
    def from_checkpoint(cls, checkpoint: str | Path, device: torch.device | str = "cuda") -> "IrisWeights":
        """A released checkpoint directory: ``config.yaml`` (its ``model`` section)
        and ``model.safetensors``, the layout ``load_config`` + ``load_dit`` read
        (``src/iris_metal/loading.py:15-17,67-77``)."""
        root = Path(checkpoint)
        return cls.from_safetensors(root / "model.safetensors", load_model_config(root / "config.yaml"), device)


def load_model_config(path: str | Path) -> ModelConfig:
    """The ``model`` section of a checkpoint's ``config.yaml`` over the defaults;
    keys the schema does not define are dropped, as ``inference_config`` does
    (``src/iris3b/config.py:539-568``)."""
    import yaml

    with open(path) as f:
        raw = yaml.safe_load(f) or {}
    model = dict(raw.get("model") or {})
    known = {f.name for f in fields(ModelConfig)}
    pixel_known = {f.name for f in fields(PixelStageConfig)}
    pixel = {k: v for k, v in dict(model.pop("pixel", None) or {}).items() if k in pixel_known}
    values = {k: v for k, v in model.items() if k in known}
    return replace(ModelConfig(), **values, pixel=replace(PixelStageConfig(), **pixel))


def synthetic_state(cfg: ModelConfig, device, seed: int = 0, std: float = 0.02, dtype=torch.bfloat16) -> dict:
    """Random weights for every parameter the per-step forward reads: N(0, std)
    for matrices and biases, 1 + N(0, std) for RMSNorm gains (so no branch is
    zero, unlike the zero-init head and adaLN of a fresh model). Drawn on the
    device; matrices are created directly in ``dtype`` (the engine's storage
    type), everything else in FP32."""
    gen = torch.Generator(device=device).manual_seed(seed)
    state: dict[str, torch.Tensor] = {}

    def mat(name, out_f, in_f, bias=False):
        state[f"{name}.weight"] = (torch.randn(out_f, in_f, generator=gen, device=device) * std).to(dtype)
        if bias:
            state[f"{name}.bias"] = torch.randn(out_f, generator=gen, device=device) * std

    def gain(name, dim):
        state[f"{name}.weight"] = 1.0 + torch.randn(dim, generator=gen, device=device) * std

    d, p, hd, hkv = cfg.hidden_size, cfg.patch_size, cfg.head_dim, cfg.kv_heads
    ffn = cfg.swiglu_hidden
    state["y_pos_embedding"] = torch.randn(1, cfg.text_len, d, generator=gen, device=device) * std
    mat("s_embedder.proj", d, p * p * cfg.in_channels, True)
    mat("t_embedder.mlp.0", d, 256, True)
    mat("t_embedder.mlp.2", d, d, True)
    mat("y_embedder.proj", d, cfg.text_dim, True)
    gain("y_embedder.norm", d)
    mat("modulation_cores.adaln_img", 6 * d, d, True)
    mat("modulation_cores.adaln_txt", 6 * d, d, True)
    mha = hkv == cfg.num_heads
    for i in range(cfg.depth):
        b = f"blocks.{i}"
        if i < cfg.dual_depth:
            for n in ("norm_x1", "norm_x2", "norm_y1", "norm_y2"):
                gain(f"{b}.{n}", d)
            for s in ("x", "y"):
                if mha:
                    mat(f"{b}.attn.qkv_{s}", 3 * d, d)
                else:
                    mat(f"{b}.attn.q_proj_{s}", d, d)
                    mat(f"{b}.attn.k_proj_{s}", hkv * hd, d)
                    mat(f"{b}.attn.v_proj_{s}", hkv * hd, d)
                gain(f"{b}.attn.q_norm_{s}", hd)
                gain(f"{b}.attn.k_norm_{s}", hd)
                mat(f"{b}.attn.proj_{s}", d, d, True)
                mat(f"{b}.attn_gate_{s}", d, d)
                gain(f"{b}.attn_post_norm_{s}", d)
                mat(f"{b}.mlp_{s}.w1", ffn, d)
                mat(f"{b}.mlp_{s}.w3", ffn, d)
                mat(f"{b}.mlp_{s}.w2", d, ffn)
                gain(f"{b}.mlp_post_norm_{s}", d)
            state[f"{b}.adaln_img.bias"] = torch.randn(6 * d, generator=gen, device=device) * std
            state[f"{b}.adaln_txt.bias"] = torch.randn(6 * d, generator=gen, device=device) * std
        else:
            gain(f"{b}.norm1", d)
            gain(f"{b}.norm2", d)
            if mha:
                mat(f"{b}.qkv", 3 * d, d)
            else:
                mat(f"{b}.q_proj", d, d)
                mat(f"{b}.k_proj", hkv * hd, d)
                mat(f"{b}.v_proj", hkv * hd, d)
            gain(f"{b}.q_norm", hd)
            gain(f"{b}.k_norm", hd)
            mat(f"{b}.attn_gate", d, d)
            mat(f"{b}.attn_proj", d, d, True)
            gain(f"{b}.attn_post_norm", d)
            mat(f"{b}.mlp.w1", ffn, d)
            mat(f"{b}.mlp.w3", ffn, d)
            mat(f"{b}.mlp.w2", d, ffn)
            gain(f"{b}.mlp_post_norm", d)
            state[f"{b}.adaln.bias"] = torch.randn(6 * d, generator=gen, device=device) * std
    pix = cfg.pixel
    dp, pp, da = pix.hidden_size, p * p, pix.attn_hidden_size
    phd = da // pix.num_heads
    mat("pixel_embedder.proj", dp, cfg.in_channels, True)
    for i in range(pix.depth):
        b = f"pixel_blocks.{i}"
        gain(f"{b}.norm1", dp)
        gain(f"{b}.norm2", dp)
        mat(f"{b}.adaln", 4 * dp * pp, d, True)
        mat(f"{b}.compress", da, pp * dp, True)
        mat(f"{b}.expand", pp * dp, da, True)
        mat(f"{b}.attn.qkv", 3 * da, da)
        gain(f"{b}.attn.q_norm", phd)
        gain(f"{b}.attn.k_norm", phd)
        mat(f"{b}.attn.proj", da, da, True)
        mat(f"{b}.mlp.fc1", int(dp * pix.mlp_ratio), dp, True)
        mat(f"{b}.mlp.fc2", dp, int(dp * pix.mlp_ratio), True)
    gain("final_layer.norm", dp)
    mat("final_layer.linear", cfg.in_channels, dp, True)
    return state
