"""fp32 restatement of ``IrisDiT.forward`` over a parameter dict (checker only).

Follows ``src/iris3b/models/dit.py:283-375``: patchify -> patch embed ->
timestep embedding -> hybrid trunk (``MMDiTBlock.forward``,
``src/iris3b/models/blocks/mmdit.py:84-128``; ``SingleStreamBlock.forward``,
``src/iris3b/models/blocks/single_stream.py:71-143``) -> timestep re-fuse ->
pixel stage (``PiTBlock.forward``, ``src/iris3b/models/blocks/pit.py:66-93``)
-> ``FinalLayer`` (``dit.py:53-62``) -> fold. Parameters are keyed by the
reference's ``state_dict`` names (``oracle.params.param_spec``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import ops
from oracle.config import OracleConfig


class OracleModel:
    def __init__(self, cfg: OracleConfig, params: dict[str, torch.Tensor]):
        self.cfg = cfg
        self.p = params

    # -- pieces ----------------------------------------------------------------
    def _lin(self, x, name, bias=True):
        return ops.linear(x, self.p[f"{name}.weight"], self.p.get(f"{name}.bias") if bias else None)

    def _norm(self, x, name):
        return ops.rms_norm(x, self.p[f"{name}.weight"], self.cfg.norm_eps)

    def t_embed(self, t: torch.Tensor) -> torch.Tensor:
        """``TimestepEmbedder.forward``, ``src/iris3b/nn/embeddings.py:47-52``."""
        emb = ops.timestep_embedding(t.reshape(-1), 256, self.cfg.timestep_max_period)
        h = F.silu(self._lin(emb, "t_embedder.mlp.0"))
        return self._lin(h, "t_embedder.mlp.2").reshape(t.shape[0], -1, self.cfg.hidden_size)

    def embed_text(self, y: torch.Tensor, mask: torch.Tensor | None = None) -> torch.Tensor:
        """``IrisDiT.embed_text``, ``dit.py:263-281``: the linear adapter
        (``TextEmbedder.forward``, ``src/iris3b/nn/embeddings.py:75-76``) or a
        masked one (``oracle.adapter``), which needs the encoder's ``[B, T]`` mask."""
        cfg = self.cfg
        y = y[:, : cfg.text_len]
        if cfg.text_adapter == "linear":
            y = self._norm(self._lin(y, "y_embedder.proj"), "y_embedder.norm")
        else:
            from oracle.adapter import AdapterOracle

            if mask is None:
                raise ValueError(f"the {cfg.text_adapter} text adapter needs the encoder's [B, T] mask")
            prefix = "y_embedder."
            params = {k[len(prefix) :]: v for k, v in self.p.items() if k.startswith(prefix)}
            y = AdapterOracle(cfg, params)(y, mask[:, : cfg.text_len])
        if cfg.text_abs_pos_embed:
            y = y + self.p["y_pos_embedding"][:, : y.shape[1]].to(y.dtype)
        return y

    def rope_tables(self, grid, n_text, device):
        cfg = self.cfg
        rope_img = ops.rope_2d(cfg.head_dim, grid[0], grid[1], cfg.rope_theta, cfg.rope_scale, cfg.rope_aspect)
        rope_txt = ops.rope_1d(cfg.head_dim, n_text, cfg.text_rope_theta) if cfg.text_rope else None
        pix_hd = cfg.pixel.attn_hidden_size // cfg.pixel.num_heads
        rope_pix = ops.rope_2d(pix_hd, grid[0], grid[1], cfg.rope_theta, cfg.rope_scale, cfg.rope_aspect)
        rope_txt = None if rope_txt is None else rope_txt.to(device)
        return rope_img.to(device), rope_txt, rope_pix.to(device)

    def _mods(self, block: str, stream: str, cond: torch.Tensor, shared: dict) -> torch.Tensor:
        """``SharedCoreBias.forward`` (``modulation.py:284-285``) or the per-block Linear."""
        if self.cfg.modulation == "shared_bias":
            core = "img" if stream in ("img", "shared") else "txt"
            return shared[core] + self.p[f"{block}.{'adaln' if stream == 'shared' else 'adaln_' + stream}.bias"]
        name = f"{block}.adaln" if stream == "shared" else f"{block}.adaln_{stream}"
        return self._lin(cond, name)

    def _project(self, h, prefix, suffix, device_layout):
        """q, k, v ``[B, N, H, hd]`` from a fused ``qkv`` or split projections
        (``attention.py:191-203``, ``single_stream.py:111-117``)."""
        cfg = self.cfg
        batch, n, _ = h.shape
        hd, hkv = cfg.head_dim, cfg.kv_heads
        fused = f"{prefix}.qkv{suffix}.weight" if device_layout == "joint" else f"{prefix}.qkv.weight"
        if fused in self.p:
            qkv = ops.linear(h, self.p[fused], self.p.get(fused.replace("weight", "bias")))
            return qkv.reshape(batch, n, 3, cfg.num_heads, hd).unbind(2)
        q = self._lin(h, f"{prefix}.q_proj{suffix}", cfg.qkv_bias).reshape(batch, n, cfg.num_heads, hd)
        k = self._lin(h, f"{prefix}.k_proj{suffix}", cfg.qkv_bias).reshape(batch, n, hkv, hd)
        v = self._lin(h, f"{prefix}.v_proj{suffix}", cfg.qkv_bias).reshape(batch, n, hkv, hd)
        return q, k, v

    def _post(self, residual, gate, name, branch):
        """``gated_norm_residual``, ``modulation.py:23-35``: ``residual + gate * norm(branch)``."""
        if self.cfg.sandwich_norm:
            branch = self._norm(branch, name)
        return residual + gate * branch

    def _swiglu(self, h, prefix):
        """``SwiGLU.forward``, ``src/iris3b/nn/mlp.py:38-40``."""
        w1 = self._lin(h, f"{prefix}.w1", False)
        w3 = self._lin(h, f"{prefix}.w3", False)
        return self._lin(F.silu(w1) * w3, f"{prefix}.w2", False)

    def dual_block(self, i, x, y, cond, rope_img, rope_txt, shared):
        """``MMDiTBlock.forward`` + ``JointAttention.forward`` (``attention.py:205-244``)."""
        cfg, b = self.cfg, f"blocks.{i}"
        batch, n_img, dim = x.shape
        n_txt = y.shape[1]
        xs1, xc1, xg1, xs2, xc2, xg2 = self._mods(b, "img", cond, shared).chunk(6, dim=-1)
        ys1, yc1, yg1, ys2, yc2, yg2 = self._mods(b, "txt", cond, shared).chunk(6, dim=-1)
        hx = ops.modulate(self._norm(x, f"{b}.norm_x1"), xs1, xc1)
        hy = ops.modulate(self._norm(y, f"{b}.norm_y1"), ys1, yc1)
        qx, kx, vx = self._project(hx, f"{b}.attn", "_x", "joint")
        qy, ky, vy = self._project(hy, f"{b}.attn", "_y", "joint")
        if cfg.qk_norm:
            qx, kx = self._norm(qx, f"{b}.attn.q_norm_x"), self._norm(kx, f"{b}.attn.k_norm_x")
            qy, ky = self._norm(qy, f"{b}.attn.q_norm_y"), self._norm(ky, f"{b}.attn.k_norm_y")
        qx, kx = ops.apply_rope(qx, rope_img), ops.apply_rope(kx, rope_img)
        if rope_txt is not None:
            qy, ky = ops.apply_rope(qy, rope_txt), ops.apply_rope(ky, rope_txt)
        q = torch.cat([qy, qx], dim=1).transpose(1, 2)
        k = torch.cat([ky, kx], dim=1).transpose(1, 2)
        v = torch.cat([vy, vx], dim=1).transpose(1, 2)
        out = ops.sdpa(q, k, v).transpose(1, 2).reshape(batch, n_txt + n_img, dim)
        out_x, out_y = out[:, n_txt:], out[:, :n_txt]
        if cfg.gated_attention:
            out_x = out_x * torch.sigmoid(self._lin(hx, f"{b}.attn_gate_x", False))
            out_y = out_y * torch.sigmoid(self._lin(hy, f"{b}.attn_gate_y", False))
        attn_x = self._lin(out_x, f"{b}.attn.proj_x")
        attn_y = self._lin(out_y, f"{b}.attn.proj_y")
        x = self._post(x, xg1, f"{b}.attn_post_norm_x", attn_x)
        mlp_x = self._swiglu(ops.modulate(self._norm(x, f"{b}.norm_x2"), xs2, xc2), f"{b}.mlp_x")
        x = self._post(x, xg2, f"{b}.mlp_post_norm_x", mlp_x)
        y = self._post(y, yg1, f"{b}.attn_post_norm_y", attn_y)
        mlp_y = self._swiglu(ops.modulate(self._norm(y, f"{b}.norm_y2"), ys2, yc2), f"{b}.mlp_y")
        y = self._post(y, yg2, f"{b}.mlp_post_norm_y", mlp_y)
        return x, y

    def single_block(self, i, x, y, cond, rope_img, rope_txt, shared):
        """``SingleStreamBlock.forward`` -> ``forward_joint``, ``single_stream.py:71-143``."""
        cfg, b = self.cfg, f"blocks.{i}"
        n_txt = y.shape[1]
        tokens = torch.cat([y, x], dim=1)
        batch, n_tokens, dim = tokens.shape
        s1, c1, g1, s2, c2, g2 = self._mods(b, "shared", cond, shared).chunk(6, dim=-1)
        h = ops.modulate(self._norm(tokens, f"{b}.norm1"), s1, c1)
        q, k, v = self._project(h, b, "", "single")
        if cfg.qk_norm:
            q, k = self._norm(q, f"{b}.q_norm"), self._norm(k, f"{b}.k_norm")
        cis = rope_img if rope_txt is None else torch.cat([rope_txt, rope_img])
        if rope_txt is None:
            q = torch.cat([q[:, :n_txt], ops.apply_rope(q[:, n_txt:], rope_img)], dim=1)
            k = torch.cat([k[:, :n_txt], ops.apply_rope(k[:, n_txt:], rope_img)], dim=1)
        else:
            q, k = ops.apply_rope(q, cis), ops.apply_rope(k, cis)
        attn = ops.sdpa(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        attn = attn.transpose(1, 2).reshape(batch, n_tokens, dim)
        if cfg.gated_attention:
            attn = attn * torch.sigmoid(self._lin(h, f"{b}.attn_gate", False))
        tokens = self._post(tokens, g1, f"{b}.attn_post_norm", self._lin(attn, f"{b}.attn_proj"))
        mlp = self._swiglu(ops.modulate(self._norm(tokens, f"{b}.norm2"), s2, c2), f"{b}.mlp")
        tokens = self._post(tokens, g2, f"{b}.mlp_post_norm", mlp)
        return tokens[:, n_txt:], tokens[:, :n_txt]

    def pixel_block(self, i, x, cond, rope_pix, grid):
        """``PiTBlock.forward`` / ``_global_attn``, ``src/iris3b/models/blocks/pit.py:66-93``."""
        cfg, b = self.cfg, f"pixel_blocks.{i}"
        pp = cfg.patch_size**2
        mods = self._lin(cond, f"{b}.adaln").reshape(x.shape[0], pp, -1)

        def global_attn(h):
            n_patches = grid[0] * grid[1]
            batch = h.shape[0] // n_patches
            compact = self._lin(h.reshape(batch * n_patches, -1), f"{b}.compress").reshape(batch, n_patches, -1)
            heads = cfg.pixel.num_heads
            hd = compact.shape[-1] // heads
            qkv = self._lin(compact, f"{b}.attn.qkv", False).reshape(batch, n_patches, 3, heads, hd)
            q, k, v = qkv.unbind(2)
            if cfg.qk_norm:
                q, k = self._norm(q, f"{b}.attn.q_norm"), self._norm(k, f"{b}.attn.k_norm")
            q, k = ops.apply_rope(q, rope_pix), ops.apply_rope(k, rope_pix)
            out = ops.sdpa(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
            out = self._lin(out.transpose(1, 2).reshape(batch, n_patches, -1), f"{b}.attn.proj")
            return self._lin(out.reshape(batch * n_patches, -1), f"{b}.expand").reshape_as(h)

        def mlp(h):
            return self._lin(F.gelu(self._lin(h, f"{b}.mlp.fc1")), f"{b}.mlp.fc2")

        if cfg.pixel.modulation == "pre":
            shift1, scale1, gate1, shift2, scale2, gate2 = mods.chunk(6, dim=-1)
            h = ops.modulate(self._norm(x, f"{b}.norm1"), shift1, scale1)
            x = x + gate1 * global_attn(h)
            x = x + gate2 * mlp(ops.modulate(self._norm(x, f"{b}.norm2"), shift2, scale2))
        else:
            scale1, shift1, scale2, shift2 = mods.chunk(4, dim=-1)
            attn = global_attn(self._norm(x, f"{b}.norm1"))
            x = x + ops.modulate(attn, shift1, scale1)
            x = x + ops.modulate(mlp(self._norm(x, f"{b}.norm2")), shift2, scale2)
        return x

    # -- forward -----------------------------------------------------------------
    def forward(self, x: torch.Tensor, t: torch.Tensor, text: torch.Tensor, capture: dict | None = None):
        """``x``: ``[B, C, H, W]``; ``t``: model time ``[B]``; ``text``: adapted text
        tokens ``[B, T, D]`` (the ``prepared_text`` of ``dit.py:291-331``)."""
        cfg = self.cfg
        p = cfg.patch_size
        batch, _, height, width = x.shape
        if height % p or width % p:
            raise ValueError(f"input {height}x{width} is not divisible by patch_size {p}")
        grid = (height // p, width // p)
        n_patches = grid[0] * grid[1]
        patches = ops.patchify(x, p)
        s = self._lin(patches, "s_embedder.proj")
        t_emb = self.t_embed(t)
        cond = F.silu(t_emb)
        y = text
        rope_img, rope_txt, rope_pix = self.rope_tables(grid, y.shape[1], x.device)
        shared = None
        if cfg.modulation == "shared_bias":
            shared = {
                "img": self._lin(cond, "modulation_cores.adaln_img"),
                "txt": self._lin(cond, "modulation_cores.adaln_txt"),
            }
        for i in range(cfg.depth):
            dual = i < cfg.dual_depth or cfg.block == "mmdit"
            block = self.dual_block if dual else self.single_block
            s, y = block(i, s, y, cond, rope_img, rope_txt, shared)
            if capture is not None:
                capture[f"block{i}"] = s
        s = F.silu(t_emb + s)
        s_cond = s.reshape(batch * n_patches, -1)
        tokens = self._lin(x.permute(0, 2, 3, 1), "pixel_embedder.proj")
        if cfg.pixel.abs_pos_embed:
            pos = ops.sincos_pos_embed_2d(cfg.pixel.hidden_size, height, width).reshape(height, width, -1)
            tokens = tokens + pos.to(device=tokens.device, dtype=tokens.dtype)
        pixels = ops.pixel_regroup(tokens, p)
        if capture is not None:
            capture["pixels_in"] = pixels
            capture["s_cond"] = s_cond
        for i in range(cfg.pixel.depth):
            pixels = self.pixel_block(i, pixels, s_cond, rope_pix, grid)
            if capture is not None:
                capture[f"pixel_block{i}"] = pixels
        out = self._lin(self._norm(pixels, "final_layer.norm"), "final_layer.linear")
        return ops.unpatchify_pixels(out, batch, height, width, p)

    __call__ = forward
