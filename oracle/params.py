"""Parameter inventory and the seeded random-init recipe.

``param_spec`` lists ``IrisDiT.named_parameters()`` for a config, in the same
order and with the same names and shapes: the model's own parameter
(``y_pos_embedding``) first, then the submodules in registration order
(``src/iris3b/models/dit.py:66-194``; blocks ``mmdit.py:37-82``,
``single_stream.py:22-69``, ``pit.py:32-64``; attention
``attention.py:97-115,149-189``; shared cores ``modulation.py:288-334``).
The golden script checks this list against the reference itself.

Init recipe (all configs): walk ``named_parameters()`` in order; RMSNorm gains
become ``1 + N(0, 0.02)``, every other tensor ``N(0, 0.02)``. This replaces the
zero-init head and adaLN, whose default would make the output exactly zero
(``tests/test_model.py:39-44``).
"""

from __future__ import annotations

import torch

from oracle.config import OracleConfig

STD = 0.02


def _linear(prefix: str, out_f: int, in_f: int, bias: bool) -> list[tuple[str, tuple, str]]:
    items = [(f"{prefix}.weight", (out_f, in_f), "w")]
    if bias:
        items.append((f"{prefix}.bias", (out_f,), "b"))
    return items


def _norm(prefix: str, dim: int) -> list[tuple[str, tuple, str]]:
    return [(f"{prefix}.weight", (dim,), "g")]


def param_spec(cfg: OracleConfig) -> list[tuple[str, tuple, str]]:
    """``[(name, shape, kind)]`` with kind ``g`` (RMSNorm gain), ``w``, ``b`` or ``p``."""
    d, p, c = cfg.hidden_size, cfg.patch_size, cfg.in_channels
    hd, hkv = cfg.head_dim, cfg.kv_heads
    ffn = cfg.swiglu_hidden
    spec: list[tuple[str, tuple, str]] = []
    if cfg.text_abs_pos_embed:
        spec.append(("y_pos_embedding", (1, cfg.text_len, d), "p"))
    spec += _linear("s_embedder.proj", d, p * p * c, True)
    spec += _linear("t_embedder.mlp.0", d, 256, True)
    spec += _linear("t_embedder.mlp.2", d, d, True)
    if cfg.text_adapter == "linear":
        spec += _linear("y_embedder.proj", d, cfg.text_dim, True)
        spec += _norm("y_embedder.norm", d)
    else:  # the masked adapters (lap_blocks2, blocks2)
        from oracle.adapter import adapter_param_spec

        spec += [(f"y_embedder.{n}", s, k) for n, s, k in adapter_param_spec(cfg)]
    if cfg.modulation == "shared_bias":
        spec += _linear("modulation_cores.adaln_img", 6 * d, d, True)
        spec += _linear("modulation_cores.adaln_txt", 6 * d, d, True)
    elif cfg.modulation != "per_block":
        raise NotImplementedError(f"modulation {cfg.modulation}")
    mha = hkv == cfg.num_heads
    for i in range(cfg.depth):
        b = f"blocks.{i}"
        dual = i < cfg.dual_depth or cfg.block == "mmdit"
        if dual:
            spec += _norm(f"{b}.norm_x1", d) + _norm(f"{b}.norm_x2", d)
            spec += _norm(f"{b}.norm_y1", d) + _norm(f"{b}.norm_y2", d)
            if mha:
                spec += _linear(f"{b}.attn.qkv_x", 3 * d, d, cfg.qkv_bias)
                spec += _linear(f"{b}.attn.qkv_y", 3 * d, d, cfg.qkv_bias)
            else:
                for s in ("x", "y"):
                    spec += _linear(f"{b}.attn.q_proj_{s}", d, d, cfg.qkv_bias)
                    spec += _linear(f"{b}.attn.k_proj_{s}", hkv * hd, d, cfg.qkv_bias)
                    spec += _linear(f"{b}.attn.v_proj_{s}", hkv * hd, d, cfg.qkv_bias)
            if cfg.qk_norm:
                for n in ("q_norm_x", "k_norm_x", "q_norm_y", "k_norm_y"):
                    spec += _norm(f"{b}.attn.{n}", hd)
            spec += _linear(f"{b}.attn.proj_x", d, d, True)
            spec += _linear(f"{b}.attn.proj_y", d, d, True)
            if cfg.gated_attention:
                spec += _linear(f"{b}.attn_gate_x", d, d, False)
                spec += _linear(f"{b}.attn_gate_y", d, d, False)
            if cfg.sandwich_norm:
                spec += _norm(f"{b}.attn_post_norm_x", d) + _norm(f"{b}.attn_post_norm_y", d)
            for s in ("x", "y"):
                spec += _linear(f"{b}.mlp_{s}.w1", ffn, d, False)
                spec += _linear(f"{b}.mlp_{s}.w3", ffn, d, False)
                spec += _linear(f"{b}.mlp_{s}.w2", d, ffn, False)
            if cfg.sandwich_norm:
                spec += _norm(f"{b}.mlp_post_norm_x", d) + _norm(f"{b}.mlp_post_norm_y", d)
            if cfg.modulation == "shared_bias":
                spec += [(f"{b}.adaln_img.bias", (6 * d,), "b"), (f"{b}.adaln_txt.bias", (6 * d,), "b")]
            else:
                spec += _linear(f"{b}.adaln_img", 6 * d, d, True)
                spec += _linear(f"{b}.adaln_txt", 6 * d, d, True)
        else:
            spec += _norm(f"{b}.norm1", d) + _norm(f"{b}.norm2", d)
            if mha:
                spec += _linear(f"{b}.qkv", 3 * d, d, cfg.qkv_bias)
            else:
                spec += _linear(f"{b}.q_proj", d, d, cfg.qkv_bias)
                spec += _linear(f"{b}.k_proj", hkv * hd, d, cfg.qkv_bias)
                spec += _linear(f"{b}.v_proj", hkv * hd, d, cfg.qkv_bias)
            if cfg.qk_norm:
                spec += _norm(f"{b}.q_norm", hd) + _norm(f"{b}.k_norm", hd)
            if cfg.gated_attention:
                spec += _linear(f"{b}.attn_gate", d, d, False)
            spec += _linear(f"{b}.attn_proj", d, d, True)
            if cfg.sandwich_norm:
                spec += _norm(f"{b}.attn_post_norm", d)
            spec += _linear(f"{b}.mlp.w1", ffn, d, False)
            spec += _linear(f"{b}.mlp.w3", ffn, d, False)
            spec += _linear(f"{b}.mlp.w2", d, ffn, False)
            if cfg.sandwich_norm:
                spec += _norm(f"{b}.mlp_post_norm", d)
            if cfg.modulation == "shared_bias":
                spec += [(f"{b}.adaln.bias", (6 * d,), "b")]
            else:
                spec += _linear(f"{b}.adaln", 6 * d, d, True)
    pix = cfg.pixel
    if not pix.enabled:
        raise NotImplementedError("the oracle restates the pixel-stage model only")
    dp, pp, da = pix.hidden_size, p * p, pix.attn_hidden_size
    spec += _linear("pixel_embedder.proj", dp, c, True)
    n_mod = 6 if pix.modulation == "pre" else 4
    for i in range(pix.depth):
        b = f"pixel_blocks.{i}"
        spec += _norm(f"{b}.norm1", dp) + _norm(f"{b}.norm2", dp)
        spec += _linear(f"{b}.adaln", n_mod * dp * pp, d, True)
        spec += _linear(f"{b}.compress", da, pp * dp, True)
        spec += _linear(f"{b}.expand", pp * dp, da, True)
        spec += _linear(f"{b}.attn.qkv", 3 * da, da, False)
        if cfg.qk_norm:
            spec += _norm(f"{b}.attn.q_norm", da // pix.num_heads) + _norm(f"{b}.attn.k_norm", da // pix.num_heads)
        spec += _linear(f"{b}.attn.proj", da, da, True)
        hidden = int(dp * pix.mlp_ratio)
        spec += _linear(f"{b}.mlp.fc1", hidden, dp, True)
        spec += _linear(f"{b}.mlp.fc2", dp, hidden, True)
    spec += _norm("final_layer.norm", dp)
    spec += _linear("final_layer.linear", c, dp, True)
    return spec


def seeded_init(
    cfg: OracleConfig,
    seed: int = 0,
    device: torch.device | str = "cpu",
    dtype: torch.dtype = torch.float32,
) -> dict[str, torch.Tensor]:
    """The recipe above, drawn from one generator in ``named_parameters()`` order.

    On ``device="cpu"`` this is bit-identical to running the recipe over the
    reference's own ``IrisDiT`` with ``torch.manual_seed(seed)``. On a CUDA
    device the same recipe draws from a CUDA generator (a different stream),
    which is how the full-size configs get their weights on the GPU box.
    """
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    params = {}
    for name, shape, kind in param_spec(cfg):
        value = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * STD
        if kind == "g":
            value += 1.0
        params[name] = value.to(dtype)
    return params


def num_parameters(cfg: OracleConfig) -> int:
    total = 0
    for _, shape, _ in param_spec(cfg):
        n = 1
        for s in shape:
            n *= s
        total += n
    return total


def depth_task_params(cfg: OracleConfig, seed: int = 0, extra_seed: int = 7) -> dict[str, torch.Tensor]:
    """Weights of a depth fine-tune (``IrisDepth``, ``src/iris3b/downstream/depth.py:30-38``):
    the model of ``seeded_init(cfg, seed)`` with the patch and pixel embedders
    widened to one extra input channel, concatenated after RGB, and the 1x1
    ``depth_reducer`` (3 -> 1). The widened weights and the reducer are drawn
    afresh, ``N(0, 0.02)``, from a generator seeded with ``extra_seed`` in the
    order s_embedder, pixel_embedder, depth_reducer (weight then bias each).
    Keys of the denoiser keep their ``IrisDiT`` names; the reducer's are
    ``depth_reducer.weight`` / ``depth_reducer.bias``."""
    params = seeded_init(cfg, seed)
    gen = torch.Generator().manual_seed(extra_seed)
    d, p, c = cfg.hidden_size, cfg.patch_size, cfg.in_channels
    shapes = {
        "s_embedder.proj.weight": (d, p * p * (c + 1)),
        "s_embedder.proj.bias": (d,),
        "pixel_embedder.proj.weight": (cfg.pixel.hidden_size, c + 1),
        "pixel_embedder.proj.bias": (cfg.pixel.hidden_size,),
        "depth_reducer.weight": (1, c, 1, 1),
        "depth_reducer.bias": (1,),
    }
    for name, shape in shapes.items():
        params[name] = torch.randn(shape, generator=gen) * STD
    return params
