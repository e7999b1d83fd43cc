"""Tiled one-step restoration (the restoration / 4x upscaling task) on the engine.

The reference's restorer (``Restorer`` / ``MetalRestorer``,
``src/iris3b/downstream/restoration.py:104-167``, ``src/iris_metal/tasks.py:106-150``)
runs one denoiser call per ``tile x tile`` crop at model time ``sigma * 1000``
with the empty prompt, restores ``x - sigma v`` and fuses overlapping tiles
(stride ``tile / 2``, the last one flush with the far edge) with a Gaussian
window (``tiled``, ``gaussian_window``, ``restoration.py:68-101``). Here:

* the crops are gathered on the device (``iris_tile_crop``) and several tiles
  go through one engine call (the engine is per-sample independent, so a batch
  of tiles gives the same per-tile result as the reference's one-tile calls);
* each restored tile is fused straight into the output with its window in
  one pass (``iris_tile_accumulate``: ``x - sigma v`` times the window), and the
  weighted average is one more pass (``iris_tile_normalize``);
* over a process group the tiles are split across ranks (independent units,
  no exchange until the end): every rank fuses its own tiles into a zeroed
  image, the window weights of all tiles are summed on every rank, and one sum
  all-reduce of the image assembles the result.

Image handling around the tiles (bicubic resizing, padding to the patch, the
wavelet colour fix, PIL I/O) stays with the caller, as in the reference's
``Restorer.__call__``.
"""

from __future__ import annotations

import torch

from iris_b200 import _lib
from iris_b200.kernels import stream_of
from iris_b200.model import require_finite


def tile_positions(size: int, tile: int, stride: int) -> list[int]:
    """Tile start offsets along one axis, the last tile flush with the far edge
    (``restoration.py:68-72``)."""
    if size <= tile:
        return [0]
    return [*range(0, size - tile, stride), size - tile]


def gaussian_window(tile: int) -> torch.Tensor:
    """The ``[tile, tile]`` fusion weights of ``restoration.py:75-84`` (FP32, on
    the CPU): variance 0.01 in tile-normalised coordinates, vertical centre
    ``tile / 2``, horizontal centre ``(tile - 1) / 2``."""
    index = torch.arange(tile, dtype=torch.float32)
    cols = torch.exp(-((index - (tile - 1) / 2) ** 2) / (tile * tile) / 0.02)
    rows = torch.exp(-((index - tile / 2) ** 2) / (tile * tile) / 0.02)
    return rows[:, None] * cols[None, :]


def tile_plan(height: int, width: int, tile: int, rank: int = 0, world: int = 1):
    """Every tile's ``(top, left)`` in the reference's order (rows of tiles top to
    bottom, each left to right, stride ``tile / 2``) and this rank's contiguous
    share of them (balanced to within one tile)."""
    from iris_b200.parallel import image_shard

    stride = tile // 2
    tiles = [(top, left) for top in tile_positions(height, tile, stride) for left in tile_positions(width, tile, stride)]
    lo, hi = image_shard(len(tiles), rank, world)
    return tiles, tiles[lo:hi]


def _balanced(items: list, calls: int) -> list[list]:
    base, extra = divmod(len(items), calls)
    out, start = [], 0
    for i in range(calls):
        n = base + (1 if i < extra else 0)
        out.append(items[start : start + n])
        start += n
    return [c for c in out if c]


class TiledRestorer:
    """``restore_tile`` and the tiled fusion of the restorer on a
    :class:`iris_b200.model.CudaIris` engine.

    ``text``: the adapted empty prompt ``[1, T, D]`` (``engine.encode_text`` of
    the export's prompt states); ``sigma`` and ``tile`` from the export's task
    settings. ``tiles_per_call`` tiles share one engine call. ``group``: a
    ``torch.distributed`` process group whose ranks split the tiles (None: all
    tiles on this GPU). ``on_tile``, when set, runs before every tile; raising
    from it stops the image between tiles, as in ``MetalRestorer``."""

    def __init__(self, engine, text: torch.Tensor, sigma: float = 0.5, tile: int = 1024,
                 num_train_timesteps: int = 1000, tiles_per_call: int = 8, group=None):  # fmt: skip
        if tiles_per_call < 1:
            raise ValueError("tiles_per_call must be at least 1")
        self.engine = engine
        self.text = text.to(engine.device, torch.float32)
        self.sigma = float(sigma)
        self.tile = int(tile)
        self.patch = engine.cfg.patch_size
        self.time = self.sigma * num_train_timesteps
        self.tiles_per_call = tiles_per_call
        self.group = group
        self.on_tile = None
        self._window: torch.Tensor | None = None

    def tile_count(self, size: tuple[int, int], scale: int = 4) -> int:
        """Tiles run for an input of ``size`` (width, height) upscaled by ``scale``:
        the work-area arithmetic of ``MetalRestorer.tile_count`` (``tasks.py:124-137``)."""
        out = [side * scale for side in reversed(size)]
        if min(out) <= self.tile:
            ratio = self.tile / min(out)
            out = [max(self.tile, round(side * ratio)) for side in out]
        height, width = (side + -side % self.patch for side in out)
        if height <= self.tile and width <= self.tile:
            return 1
        stride = self.tile // 2
        return len(tile_positions(height, self.tile, stride)) * len(tile_positions(width, self.tile, stride))

    def _restore(self, x: torch.Tensor) -> torch.Tensor:
        """``x - sigma v`` of a batch of tiles (no finiteness check)."""
        b = x.shape[0]
        t = torch.full((b,), self.time, device=x.device, dtype=torch.float32)
        v = self.engine(x, t, self.text.expand(b, -1, -1))
        out = torch.empty_like(x)
        # the flow step with sigma_next < 0 is the clean estimate x - sigma v
        _lib.call("iris_cfg_euler", v.data_ptr(), x.data_ptr(), out.data_ptr(), b, x[0].numel(), 1.0, self.sigma,
                  -1.0, 0, stream_of(x))  # fmt: skip
        return out

    @torch.no_grad()
    def restore_tile(self, x: torch.Tensor) -> torch.Tensor:
        """``[B, 3, tile, tile]`` in ``[-1, 1]`` -> restored, same range and size
        (``MetalRestorer.restore_tile``, ``tasks.py:143-150``)."""
        if self.on_tile is not None:
            self.on_tile()
        x = x.to(self.engine.device, torch.float32).contiguous()
        return require_finite(self._restore(x))

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """``tiled(restore_tile, x, tile, tile // 2)`` (``restoration.py:87-101``) for
        ``x``: ``[1, C, H, W]`` in ``[-1, 1]`` with H and W multiples of the patch."""
        if x.dim() != 4 or x.shape[0] != 1:
            raise ValueError("the restorer takes one image [1, C, H, W]")
        x = x.to(self.engine.device, torch.float32).contiguous()
        _, channels, height, width = x.shape
        tile = self.tile
        if height <= tile and width <= tile:
            return self.restore_tile(x)
        if height < tile or width < tile:
            raise ValueError(f"an image larger than one tile needs both sides >= {tile}, got {height}x{width}")
        if height % self.patch or width % self.patch:
            raise ValueError(f"input {height}x{width} is not divisible by patch_size {self.patch}")
        rank, world = 0, 1
        if self.group is not None:
            import torch.distributed as dist

            rank, world = dist.get_rank(self.group), dist.get_world_size(self.group)
        tiles, mine = tile_plan(height, width, tile, rank, world)
        dev = x.device
        st = stream_of(x)
        if self._window is None or self._window.device != dev:
            self._window = gaussian_window(tile).to(dev).contiguous()
        window = self._window
        out = torch.zeros_like(x)
        weight = torch.zeros(height, width, device=dev, dtype=torch.float32)
        for top, left in tiles:  # the weights of every tile, on every rank
            _lib.call("iris_tile_accumulate", None, channels, height, width, None, tile, window.data_ptr(), top, left,
                      0.0, None, weight.data_ptr(), st)  # fmt: skip
        calls = -(-len(mine) // self.tiles_per_call)
        for chunk in _balanced(mine, max(calls, 1)):
            batch = torch.empty(len(chunk), channels, tile, tile, device=dev, dtype=torch.float32)
            for i, (top, left) in enumerate(chunk):
                if self.on_tile is not None:
                    self.on_tile()
                _lib.call("iris_tile_crop", x.data_ptr(), channels, height, width, top, left, tile, batch[i].data_ptr(),
                          st)  # fmt: skip
            b = len(chunk)
            v = self.engine(batch, torch.full((b,), self.time, device=dev), self.text.expand(b, -1, -1))
            for i, (top, left) in enumerate(chunk):
                _lib.call("iris_tile_accumulate", x.data_ptr(), channels, height, width, v[i].data_ptr(), tile,
                          window.data_ptr(), top, left, self.sigma, out.data_ptr(), None, st)  # fmt: skip
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(out, group=self.group)
        _lib.call("iris_tile_normalize", out.data_ptr(), weight.data_ptr(), channels, height, width, st)
        return require_finite(out)
