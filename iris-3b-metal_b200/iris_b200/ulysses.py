"""Sequence parallelism (Ulysses) for one denoiser call spread over P GPUs.

The reference runs one image on one device; at 2048^2 (N = 256 + 16384 joint
tokens) this module splits a call across ranks instead of splitting the batch.
Rank r owns joint tokens ``[r n, (r + 1) n)`` of every sample's ``[text |
image]`` sequence, ``n = N / P``. Everything per token (norms, modulation,
every linear, the residual updates, the whole per-pixel stage) stays local;
the exchanges are:

* trunk attention: Q, K and V leave ``iris_qkv_heads`` head-major
  (``[H, B, n, 128]``), so the rows of the ``H / P`` heads that rank j will own
  form one contiguous chunk; an all-to-all turns them into every token of
  those heads, which ``iris_block_copy`` lays out as ``[B, H / P, N, 128]``.
  The attention output goes back the same way (pack, all-to-all, unpack into
  ``[B n, H 128]`` token rows), and the sigmoid gate is applied by the gate
  GEMM's epilogue (out = o * sigmoid(h W_g^T)) on the local rows;
* pixel-stage attention (10 heads, not divisible by every P): each rank keeps
  its own queries and all-gathers K and V of every patch token;
* the velocity image: each rank writes the pixels of its own patch tokens into
  a zeroed image and a sum all-reduce assembles it (every pixel has exactly one
  writer, so the sum is exact).

RoPE tables are indexed by global token position, the collectives go through
a small communicator (:class:`TorchComm` over ``torch.distributed`` / NCCL in
production), and every rank returns the full velocity.

With one process per GPU (a communicator with ``peer_capable``), the exchanges
are not collectives at all: the ranks map each other's exchange buffers with
CUDA IPC (:class:`PeerBuffers`) and the producing kernels store into the
consumer's buffer over NVLink -- the Q/K/V projection's epilogue writes every
head row to the full-sequence buffer of the rank that owns that head, the
attention epilogue writes every output row to the token rows of the rank that
owns that token, and the pixel-stage K/V projection writes its rows to every
rank. A bounded barrier kernel on flags in peer memory orders each producer
before its consumers.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol

import torch


class Communicator(Protocol):
    """The three collectives a sequence-parallel call uses (flat, equal-split)."""

    rank: int
    world: int

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor) -> None: ...

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None: ...

    def all_reduce_sum(self, t: torch.Tensor) -> None: ...


class TorchComm:
    """:class:`Communicator` over a ``torch.distributed`` process group (NCCL on
    GPUs: the collectives are enqueued after the current stream's work and the
    stream waits for them; the host is not synchronised)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self._dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        self._dist.all_to_all_single(out, inp, group=self.group)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        self._dist.all_gather_into_tensor(out, inp, group=self.group)

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        self._dist.all_reduce(t, group=self.group)

    # one process per GPU on one node: the ranks can map each other's buffers
    peer_capable = True

    def all_gather_object(self, obj) -> list:
        out = [None] * self.world
        self._dist.all_gather_object(out, obj, group=self.group)
        return out


class PeerBuffers:
    """This rank's exchange buffers and, for each, the device pointer of every
    rank's copy as mapped into this process (CUDA IPC; the rank's own entry is
    its local pointer). Buffers that share an allocation are mapped once."""

    def __init__(self, comm, tensors: dict[str, torch.Tensor]):
        from iris_b200 import kernels as K

        self._K = K
        self.tensors = tensors
        handles = {name: K.ipc_export(t) for name, t in tensors.items()}
        everyone = comm.all_gather_object(handles)
        self._bases: dict[bytes, int] = {}
        self.ptrs: dict[str, list[int]] = {name: [] for name in tensors}
        for j, theirs in enumerate(everyone):
            for name in tensors:
                handle, offset = theirs[name]
                if j == comm.rank:
                    self.ptrs[name].append(tensors[name].data_ptr())
                    continue
                base = self._bases.get(handle)
                if base is None:
                    base = self._bases[handle] = K.ipc_import(handle)
                self.ptrs[name].append(base + offset)

    def close(self) -> None:
        for base in self._bases.values():
            self._K.ipc_close(base)
        self._bases.clear()


@dataclass(frozen=True)
class SequenceShard:
    """Rank ``rank``'s share of a ``[text (T) | image (L)]`` sequence."""

    rank: int
    world: int
    T: int
    L: int

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"bad rank {self.rank} of {self.world}")
        if (self.T + self.L) % self.world:
            raise ValueError(
                f"sequence parallelism over {self.world} ranks needs T + L = {self.T + self.L} divisible by {self.world}"
            )
        for r in range(self.world):
            if self._split(r)[1] <= 0:
                raise ValueError(f"rank {r} of {self.world} would hold no image tokens")

    def _split(self, rank: int) -> tuple[int, int, int]:
        """(text tokens, image tokens, first image token) of ``rank``."""
        n = self.n
        start = rank * n
        text = min(max(self.T - start, 0), n)
        return text, n - text, max(start - self.T, 0)

    @property
    def N(self) -> int:
        return self.T + self.L

    @property
    def n(self) -> int:
        """Joint tokens per rank."""
        return (self.T + self.L) // self.world

    @property
    def start(self) -> int:
        """First global joint token of this rank (its RoPE table row)."""
        return self.rank * self.n

    @property
    def text(self) -> int:
        """Text tokens held (they come first in the rank's rows)."""
        return self._split(self.rank)[0]

    @property
    def text_start(self) -> int:
        """First text token held (meaningful when ``text > 0``)."""
        return min(self.start, self.T)

    @property
    def image(self) -> int:
        return self._split(self.rank)[1]

    @property
    def image_start(self) -> int:
        """First image (patch) token held, in image numbering."""
        return self._split(self.rank)[2]

    @property
    def image_max(self) -> int:
        """The largest image share over the ranks (all-gather padding)."""
        return max(self._split(r)[1] for r in range(self.world))

    def of(self, rank: int) -> "SequenceShard":
        return SequenceShard(rank, self.world, self.T, self.L)


# --------------------------------------------------------------------- layout plans
# Each plan is (dst byte offset, dst strides, src byte offset, src strides, counts,
# block bytes) for one iris_block_copy launch; element size 2 (bf16).


def heads_unpack_plan(world: int, heads_local: int, batch: int, n: int, head_dim: int = 128):
    """All-to-all receive ``[P(src), H/P, B, n, D]`` -> ``[B, H/P, P n, D]``:
    rank ``src``'s tokens land at ``src * n`` of every (b, h)."""
    row = head_dim * 2
    N = world * n
    src = (heads_local * batch * n * row, batch * n * row, n * row)
    dst = (n * row, N * row, heads_local * N * row)
    return [(0, dst, 0, src, (world, heads_local, batch), n * row)]


def output_pack_plan(world: int, batch: int, n: int, width: int):
    """Attention output ``[B, P n, C]`` (C = H/P * 128 columns) -> all-to-all
    send ``[P(dst), B, n, C]``: rank j gets its own tokens of these heads."""
    blk = n * width * 2
    src = (blk, world * blk, 0)
    dst = (batch * blk, blk, 0)
    return [(0, dst, 0, src, (world, batch, 1), blk)]


def output_unpack_plan(world: int, batch: int, n: int, width: int):
    """All-to-all receive ``[P(src head group), B, n, C]`` -> token rows
    ``[B n, P C]``: head group j fills columns ``[j C, (j + 1) C)``."""
    row = width * 2
    src = (batch * n * row, row, 0)
    dst = (row, world * row, 0)
    return [(0, dst, 0, src, (world, batch * n, 1), row)]


def gathered_kv_plan(shard: SequenceShard, batch: int, heads: int, head_dim: int = 128):
    """All-gather receive ``[P(src), B, H, image_max, D]`` (each rank's image
    tokens first, padded) -> ``[B, H, L, D]`` in image-token order. Ranks with
    equal shares whose image tokens follow one another share one launch."""
    row = head_dim * 2
    pad = shard.image_max
    L = shard.L
    src_strides = (batch * heads * pad * row, heads * pad * row, pad * row)
    plans = []
    r = 0
    while r < shard.world:
        s = shard.of(r)
        run = 1
        while r + run < shard.world:
            nxt = shard.of(r + run)
            if nxt.image != s.image or nxt.image_start != s.image_start + run * s.image:
                break
            run += 1
        dst_strides = (s.image * row, heads * L * row, L * row)
        plans.append((s.image_start * row, dst_strides, r * src_strides[0], src_strides, (run, batch, heads),
                      s.image * row))  # fmt: skip
        r += run
    return plans


def run_plan(copy, dst: torch.Tensor, src: torch.Tensor, plans) -> None:
    """Issue every launch of a plan through ``copy`` (``kernels.block_copy``)."""
    for dst_off, dst_strides, src_off, src_strides, counts, block in plans:
        copy(dst, dst_strides, src, src_strides, counts, block, dst_offset=dst_off, src_offset=src_off)


# --------------------------------------------------------------------- exchanges
# The engine's three exchange steps; ``copy`` is ``kernels.block_copy``.


def scatter_heads(comm, copy, local: torch.Tensor, recv: torch.Tensor, full: torch.Tensor, heads_local: int,
                  batch: int, n: int, head_dim: int = 128) -> None:  # fmt: skip
    """Head-major local rows ``[H, B, n, D]`` -> this rank's ``H / P`` heads over
    every token, ``full`` = ``[B, H / P, P n, D]``."""
    comm.all_to_all(recv, local.view(-1))
    run_plan(copy, full, recv, heads_unpack_plan(comm.world, heads_local, batch, n, head_dim))


def gather_tokens(comm, copy, out: torch.Tensor, send: torch.Tensor, recv: torch.Tensor, rows: torch.Tensor,
                  batch: int, n: int, width: int) -> None:  # fmt: skip
    """Attention output of this rank's heads ``out`` = ``[B, P n, C]`` -> every
    head of this rank's tokens, ``rows`` = ``[B n, P C]``."""
    run_plan(copy, send, out, output_pack_plan(comm.world, batch, n, width))
    comm.all_to_all(recv, send)
    run_plan(copy, rows, recv, output_unpack_plan(comm.world, batch, n, width))


def gather_image_tokens(comm, copy, shard: SequenceShard, local: torch.Tensor, gathered: torch.Tensor,
                        full: torch.Tensor, batch: int, heads: int, head_dim: int = 128) -> None:  # fmt: skip
    """This rank's image tokens ``local`` = ``[B, H, image_max, D]`` (padded) ->
    every image token, ``full`` = ``[B, H, L, D]``."""
    comm.all_gather(gathered, local.view(-1))
    run_plan(copy, full, gathered, gathered_kv_plan(shard, batch, heads, head_dim))
