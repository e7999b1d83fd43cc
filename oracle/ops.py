"""fp32 restatements of the per-op math on the hot path (checker only).

Each function names the reference code it restates. The per-kernel references
mirror the CPU branches of ``src/iris_metal/kernels.py`` so kernel tests read
like ``tests/test_metal_engine.py:159-289``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# -- primitives ---------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``RMSNorm.forward``, ``src/iris3b/nn/norms.py:15-21``: statistics in fp32,
    gain applied after casting back to the input dtype."""
    x32 = x.float()
    normed = x32 * torch.rsqrt(x32.pow(2).mean(dim=-1, keepdim=True) + eps)
    return weight * normed.to(x.dtype)


def modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """``src/iris3b/nn/modulation.py:11-12``."""
    return x * (1 + scale) + shift


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    return F.linear(x, w, b)


def timestep_embedding(t: torch.Tensor, freq_dim: int = 256, max_period: float = 10.0) -> torch.Tensor:
    """``TimestepEmbedder.timestep_embedding``, ``src/iris3b/nn/embeddings.py:41-45``:
    ``[cos | sin]`` of ``t * exp(-ln(max_period) k / n)``."""
    n = freq_dim // 2
    k = torch.arange(n, dtype=torch.float32, device=t.device)
    phase = torch.outer(t.float(), torch.exp(-math.log(max_period) * k / n))
    return torch.cat([phase.cos(), phase.sin()], dim=-1)


def rope_2d(head_dim: int, height: int, width: int, theta: float, scale: float, aspect: str) -> torch.Tensor:
    """``rope_2d`` without frame pairs, ``src/iris3b/nn/rope.py:19-82``: complex64
    ``[H*W, head_dim/2]``, (x, y) frequency pairs interleaved, row-major tokens."""
    n_pairs = head_dim // 4
    freqs = 1.0 / theta ** (torch.arange(0, head_dim, 4)[:n_pairs].float() / head_dim)
    if aspect == "square":
        x_pos = torch.linspace(0, scale, width)
        y_pos = torch.linspace(0, scale, height)
    elif aspect == "isotropic":
        step = scale / max(max(height, width) - 1, 1)
        x_pos = torch.arange(width).float() * step
        y_pos = torch.arange(height).float() * step
    else:
        raise ValueError(aspect)
    x_cis = torch.polar(torch.ones(width, n_pairs), torch.outer(x_pos, freqs))
    y_cis = torch.polar(torch.ones(height, n_pairs), torch.outer(y_pos, freqs))
    x_grid = x_cis[None, :, :].expand(height, width, -1)
    y_grid = y_cis[:, None, :].expand(height, width, -1)
    return torch.stack([x_grid, y_grid], dim=-1).reshape(height * width, 2 * n_pairs)


def rope_1d(head_dim: int, length: int, theta: float) -> torch.Tensor:
    """``src/iris3b/nn/rope.py:85-89``."""
    freqs = 1.0 / theta ** (torch.arange(0, head_dim, 2)[: head_dim // 2].float() / head_dim)
    ang = torch.outer(torch.arange(length).float(), freqs)
    return torch.polar(torch.ones_like(ang), ang)


def apply_rope(x: torch.Tensor, cis: torch.Tensor) -> torch.Tensor:
    """One tensor of ``apply_rope``, ``src/iris3b/nn/rope.py:92-101``; ``x``: ``[B, N, H, D]``."""
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * cis[None, :, None, :]).flatten(3).to(x.dtype)


def sincos_pos_embed_2d(embed_dim: int, height: int, width: int) -> torch.Tensor:
    """``src/iris3b/nn/embeddings.py:269-288``: ``[H*W, dim]``; first half of the
    channels from the x (width) coordinate, second from y; each half is
    ``[sin | cos]`` at ``omega_i = 10000^(-i / (dim/4))``, computed in float64."""

    def one(dim: int, pos: torch.Tensor) -> torch.Tensor:
        omega = torch.arange(dim // 2, dtype=torch.float64) / (dim / 2.0)
        omega = 1.0 / 10000.0**omega
        out = torch.outer(pos.reshape(-1).double(), omega)
        return torch.cat([torch.sin(out), torch.cos(out)], dim=1)

    grid_h = torch.arange(height, dtype=torch.float32)
    grid_w = torch.arange(width, dtype=torch.float32)
    grid = torch.meshgrid(grid_w, grid_h, indexing="xy")
    grid = torch.stack(grid, dim=0).reshape(2, 1, height, width)
    return torch.cat([one(embed_dim // 2, grid[0]), one(embed_dim // 2, grid[1])], dim=1).float()


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """``scaled_dot_product`` (sdpa backend), ``src/iris3b/nn/attention.py:61-68``;
    ``[B, H, N, D]``, grouped K/V expanded explicitly."""
    if k.shape[1] != q.shape[1]:
        rep = q.shape[1] // k.shape[1]
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    # long sequences (2048^2: 16640 tokens) in query chunks, so that an fp32 score
    # matrix never has more than 2^31 entries; rows are independent, the math is unchanged
    rows = max(1, (1 << 31) // max(1, q.shape[0] * q.shape[1] * k.shape[2]))
    if q.shape[2] <= rows:
        return F.scaled_dot_product_attention(q, k, v)
    return torch.cat([F.scaled_dot_product_attention(c, k, v) for c in q.split(rows, dim=2)], dim=2)


# -- index maps (integer layouts, bit-exact) ------------------------------------
def patchify(x: torch.Tensor, p: int) -> torch.Tensor:
    """``F.unfold(x, p, stride=p).transpose(1, 2)``, ``src/iris3b/models/dit.py:326``:
    ``[B, C, H, W] -> [B, L, C*p*p]`` with features ordered (c, ky, kx)."""
    return F.unfold(x, kernel_size=p, stride=p).transpose(1, 2)


def unpatchify_pixels(out: torch.Tensor, batch: int, height: int, width: int, p: int) -> torch.Tensor:
    """Per-pixel head output ``[B*L, p*p, C]`` -> ``[B, C, H, W]``,
    ``src/iris3b/models/dit.py:367-374`` (``F.fold``)."""
    n_patches = (height // p) * (width // p)
    folded = out.reshape(batch, n_patches, p * p, -1).permute(0, 3, 2, 1).reshape(batch, -1, n_patches)
    return F.fold(folded, output_size=(height, width), kernel_size=p, stride=p)


def pixel_regroup(tokens: torch.Tensor, p: int) -> torch.Tensor:
    """``[B, H, W, d] -> [B*L, p*p, d]``, pixels row-major within a patch,
    ``src/iris3b/nn/embeddings.py:325-328``."""
    batch, height, width, dim = tokens.shape
    t = tokens.reshape(batch, height // p, p, width // p, p, dim).permute(0, 1, 3, 2, 4, 5)
    return t.reshape(batch * (height // p) * (width // p), p * p, dim)


# -- per-kernel references (iris_metal.kernels CPU branches) ---------------------
def qk_norm_rope_reference(x, weight, cos, sin, eps, out_dtype=None):
    """``src/iris_metal/kernels.py:314-331``: ``[B, N, H*128] -> [B, H, N, 128]``."""
    batch, tokens, width = x.shape
    hd = weight.numel()
    h = x.reshape(batch, tokens, width // hd, hd).float()
    normed = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    pairs = normed.reshape(*normed.shape[:-1], hd // 2, 2)
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    rotated = torch.stack((pairs[..., 0] * c - pairs[..., 1] * s, pairs[..., 0] * s + pairs[..., 1] * c), dim=-1)
    return rotated.flatten(-2).to(out_dtype or x.dtype).transpose(1, 2).contiguous()


def rms_norm_modulate_reference(x, weight, shift, scale, eps, out_dtype):
    """``src/iris_metal/kernels.py:424-426``."""
    width = x.shape[-1]
    normed = F.rms_norm(x.float(), (width,), weight, eps)
    return torch.addcmul(shift, normed, 1 + scale).to(out_dtype)


def gated_residual_rms_norm_reference(residual, branch, weight, gate, eps):
    """``src/iris_metal/kernels.py:460-462`` (returns a new tensor)."""
    width = residual.shape[-1]
    normed = F.rms_norm(branch.float(), (width,), weight, eps)
    return residual.float().addcmul(gate, normed)


def pixel_rms_norm_reference(pixels, weight, eps):
    """``src/iris_metal/kernels.py:488-489``."""
    return F.rms_norm(pixels.float(), pixels.shape[-1:], weight, eps).to(pixels.dtype)


def pixel_mlp_reference(pixels, branch, mods, norm_weight, fc1_w, fc1_b, fc2_w, fc2_b, next_norm_weight, eps):
    """``src/iris_metal/kernels.py:501-524``: returns ``(new_pixels, next_input)``;
    values the autocast path materializes are rounded to the pixel dtype."""
    dtype = pixels.dtype
    scale1, shift1, scale2, shift2 = mods.float().chunk(4, dim=-1)
    modulated = (branch.float() * (1 + scale1) + shift1).to(dtype)
    x = (pixels.float() + modulated.float()).to(dtype)
    h = F.rms_norm(x.float(), x.shape[-1:], norm_weight, eps).to(dtype)
    a = F.linear(h.float(), fc1_w.float(), fc1_b.float()).to(dtype)
    g = F.gelu(a.float()).to(dtype)
    mlp = F.linear(g.float(), fc2_w.float(), fc2_b.float()).to(dtype)
    modulated = (mlp.float() * (1 + scale2) + shift2).to(dtype)
    new_pixels = (x.float() + modulated.float()).to(dtype)
    nxt = F.rms_norm(new_pixels.float(), new_pixels.shape[-1:], next_norm_weight, eps).to(dtype)
    return new_pixels, nxt
