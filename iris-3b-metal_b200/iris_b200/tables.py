"""Position tables computed once per resolution on the host, then kept on the device.

They must match the reference bit for bit (the token-position mapping is an
integer layout), so they are evaluated with the same fp32 torch arithmetic:

* ``rope_2d`` / ``rope_1d``: ``src/iris3b/nn/rope.py:19-89``; cos/sin split as
  ``RopeTable.from_complex`` does (``src/iris_metal/model.py:55-65``);
* ``sincos_pos_embed_2d``: ``src/iris3b/nn/embeddings.py:269-288`` (float64,
  stored as float32).
"""

from __future__ import annotations

import torch


def rope_2d(head_dim: int, height: int, width: int, theta: float, scale: float, aspect: str) -> torch.Tensor:
    """Complex64 ``[height*width, head_dim/2]``: frequency pairs interleaved (x, y),
    tokens row-major."""
    n_pairs = head_dim // 4
    freqs = 1.0 / theta ** (torch.arange(0, head_dim, 4)[:n_pairs].float() / head_dim)
    if aspect == "square":
        xs, ys = torch.linspace(0, scale, width), torch.linspace(0, scale, height)
    elif aspect == "isotropic":
        step = scale / max(max(height, width) - 1, 1)
        xs, ys = torch.arange(width).float() * step, torch.arange(height).float() * step
    else:
        raise ValueError(f"unknown rope aspect mode '{aspect}'")
    xc = torch.polar(torch.ones(width, n_pairs), torch.outer(xs, freqs))
    yc = torch.polar(torch.ones(height, n_pairs), torch.outer(ys, freqs))
    grid = torch.stack([xc[None, :, :].expand(height, width, -1), yc[:, None, :].expand(height, width, -1)], dim=-1)
    return grid.reshape(height * width, 2 * n_pairs)


def rope_1d(head_dim: int, length: int, theta: float) -> torch.Tensor:
    freqs = 1.0 / theta ** (torch.arange(0, head_dim, 2)[: head_dim // 2].float() / head_dim)
    angles = torch.outer(torch.arange(length).float(), freqs)
    return torch.polar(torch.ones_like(angles), angles)


def cos_sin(*tables: torch.Tensor, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Concatenated complex tables -> contiguous FP32 (cos, sin) ``[N, head_dim/2]``."""
    cis = torch.view_as_real(torch.cat(tables))
    return cis[..., 0].contiguous().to(device), cis[..., 1].contiguous().to(device)


def sincos_pos_embed_2d(embed_dim: int, height: int, width: int) -> torch.Tensor:
    """``[H*W, dim]``: channels ``[sin | cos](x * w_i)`` then ``[sin | cos](y * w_i)``,
    ``w_i = 10000^(-i / (dim / 4))``, evaluated in float64."""
    quarter = embed_dim // 4
    omega = 1.0 / 10000.0 ** (torch.arange(quarter, dtype=torch.float64) / quarter)
    ys, xs = torch.meshgrid(torch.arange(height, dtype=torch.float64), torch.arange(width, dtype=torch.float64),
                            indexing="ij")  # fmt: skip
    ax = torch.outer(xs.reshape(-1), omega)
    ay = torch.outer(ys.reshape(-1), omega)
    return torch.cat([ax.sin(), ax.cos(), ay.sin(), ay.cos()], dim=1).float()
