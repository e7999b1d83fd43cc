"""fp32 restatement of the masked text adapters (checker only).

``LayerwiseTextEmbedder`` ("lap_blocks2", ``src/iris3b/nn/embeddings.py:209-266``):
two pre-norm blocks over each token's encoder-layer states
(``LayerwiseAttentionBlock``, ``:111-142``: unmasked self-attention without QK
norm or RoPE, then a Linear-SiLU-Linear MLP), a ``Linear(layers -> 1)`` pool
over the layer axis, then the refiner. ``TransformerTextEmbedder`` ("blocks2",
``:144-207``) is the refiner on its own: Linear, two ``TextAdapterBlock``s
(``:79-108``: QK-normed self-attention with pad keys masked except on the
diagonal, SwiGLU), RMSNorm. Attention follows ``SelfAttention.forward``
(``src/iris3b/nn/attention.py:117-132``). Parameters are keyed by the
reference's ``named_parameters()`` names under the adapter module.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import ops


def adapter_param_spec(cfg) -> list[tuple[str, tuple, str]]:
    """``[(name, shape, kind)]`` of the adapter module ``y_embedder`` in the
    reference's registration order (kinds as ``oracle.params.param_spec``)."""
    d, dt = cfg.hidden_size, cfg.text_dim
    spec: list[tuple[str, tuple, str]] = []

    def linear(name, out_f, in_f, bias):
        spec.append((f"{name}.weight", (out_f, in_f), "w"))
        if bias:
            spec.append((f"{name}.bias", (out_f,), "b"))

    def norm(name, dim):
        spec.append((f"{name}.weight", (dim,), "g"))

    def refiner(prefix):
        linear(f"{prefix}proj", d, dt, True)
        hd = d // cfg.num_heads
        ffn = int(2 * int(d * cfg.mlp_ratio) / 3)
        for i in range(2):
            b = f"{prefix}blocks.{i}"
            norm(f"{b}.norm1", d)
            linear(f"{b}.attn.qkv", 3 * d, d, cfg.qkv_bias)
            if cfg.qk_norm:
                norm(f"{b}.attn.q_norm", hd)
                norm(f"{b}.attn.k_norm", hd)
            linear(f"{b}.attn.proj", d, d, True)
            norm(f"{b}.norm2", d)
            linear(f"{b}.mlp.w1", ffn, d, False)
            linear(f"{b}.mlp.w3", ffn, d, False)
            linear(f"{b}.mlp.w2", d, ffn, False)
        norm(f"{prefix}norm", d)

    if cfg.text_adapter == "blocks2":
        refiner("")
        return spec
    if cfg.text_adapter != "lap_blocks2":
        raise NotImplementedError(f"text adapter {cfg.text_adapter}")
    hidden = int(dt * cfg.text_lap_mlp_ratio)
    for i in range(2):
        b = f"layer_blocks.{i}"
        norm(f"{b}.norm1", dt)
        linear(f"{b}.attn.qkv", 3 * dt, dt, False)
        linear(f"{b}.attn.proj", dt, dt, True)
        norm(f"{b}.norm2", dt)
        linear(f"{b}.mlp.0", hidden, dt, True)
        linear(f"{b}.mlp.2", dt, hidden, True)
    linear("layer_pool", 1, cfg.text_lap_num_layers, True)
    refiner("refiner.")
    return spec


class AdapterOracle:
    """``y_embedder(y, mask)`` of a masked adapter; ``params`` keyed as
    :func:`adapter_param_spec` names."""

    def __init__(self, cfg, params: dict[str, torch.Tensor]):
        self.cfg = cfg
        self.p = params

    def _lin(self, x, name):
        return ops.linear(x, self.p[f"{name}.weight"], self.p.get(f"{name}.bias"))

    def _norm(self, x, name):
        return ops.rms_norm(x, self.p[f"{name}.weight"], self.cfg.norm_eps)

    def _attention(self, x, prefix, heads, qk_norm, mask):
        """``SelfAttention.forward`` without RoPE, ``attention.py:117-132``."""
        batch, n, dim = x.shape
        hd = dim // heads
        q, k, v = self._lin(x, f"{prefix}.qkv").reshape(batch, n, 3, heads, hd).unbind(2)
        if qk_norm:
            q, k = self._norm(q, f"{prefix}.q_norm"), self._norm(k, f"{prefix}.k_norm")
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
        out = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return self._lin(out.transpose(1, 2).reshape(batch, n, dim), f"{prefix}.proj")

    def refiner(self, y, mask, prefix=""):
        """``TransformerTextEmbedder.forward``, ``embeddings.py:199-207``."""
        cfg = self.cfg
        if mask.shape != y.shape[:2]:
            raise ValueError(f"text mask must be {tuple(y.shape[:2])}, got {tuple(mask.shape)}")
        keep = mask.bool()[:, None, None, :]
        eye = torch.eye(y.shape[1], dtype=torch.bool, device=y.device)
        attn_mask = keep | eye
        y = self._lin(y, f"{prefix}proj")
        for i in range(2):
            b = f"{prefix}blocks.{i}"
            y = y + self._attention(self._norm(y, f"{b}.norm1"), f"{b}.attn", cfg.num_heads, cfg.qk_norm, attn_mask)
            h = self._norm(y, f"{b}.norm2")
            mlp = self._lin(F.silu(self._lin(h, f"{b}.mlp.w1")) * self._lin(h, f"{b}.mlp.w3"), f"{b}.mlp.w2")
            y = y + mlp
        return self._norm(y, f"{prefix}norm")

    def forward(self, y: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        """``LayerwiseTextEmbedder.forward`` (``embeddings.py:254-266``): ``y``
        ``[B, T, layers, text_dim]`` -> ``[B, T, hidden]``; or the refiner alone
        on ``[B, T, text_dim]`` for "blocks2"."""
        cfg = self.cfg
        y = y.float()
        if cfg.text_adapter == "blocks2":
            return self.refiner(y, mask)
        batch, tokens, layers, dim = y.shape
        x = y.reshape(batch * tokens, layers, dim)
        for i in range(2):
            b = f"layer_blocks.{i}"
            x = x + self._attention(self._norm(x, f"{b}.norm1"), f"{b}.attn", cfg.text_lap_num_heads, False, None)
            x = x + self._lin(F.silu(self._lin(self._norm(x, f"{b}.norm2"), f"{b}.mlp.0")), f"{b}.mlp.2")
        pooled = self._lin(x.transpose(1, 2), "layer_pool").squeeze(-1)
        return self.refiner(pooled.reshape(batch, tokens, dim), mask, "refiner.")

    __call__ = forward
