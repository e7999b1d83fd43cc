"""Test infrastructure: P ranks as threads of one process.

``ThreadComm`` implements the three collectives of
``iris_b200.ulysses.Communicator`` with a barrier and plain tensor copies, so
a sequence-parallel call can run with every rank on one device (or on the
CPU). Each collective synchronises the device before publishing its input
and again before the closing barrier, so no rank overwrites a buffer another
rank is still reading. ``emulated_block_copy`` restates iris_block_copy on
CPU tensors for the host-logic tests.
"""

from __future__ import annotations

import threading

import torch


def _sync(t: torch.Tensor) -> None:
    if t.is_cuda:
        torch.cuda.synchronize(t.device)


class ThreadGroup:
    def __init__(self, world: int, timeout: float = 120.0):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=timeout)
        self.slots: list = [None] * world

    def comm(self, rank: int) -> "ThreadComm":
        return ThreadComm(self, rank)


class ThreadComm:
    def __init__(self, group: ThreadGroup, rank: int):
        self.group, self.rank, self.world = group, rank, group.world

    def _publish(self, t: torch.Tensor) -> list:
        _sync(t)
        self.group.slots[self.rank] = t
        self.group.barrier.wait()
        return list(self.group.slots)

    def _done(self, t: torch.Tensor) -> None:
        _sync(t)
        self.group.barrier.wait()

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        slots = self._publish(inp.view(-1))
        chunk = inp.numel() // self.world
        flat = out.view(-1)
        for src, t in enumerate(slots):
            flat[src * chunk : (src + 1) * chunk].copy_(t[self.rank * chunk : (self.rank + 1) * chunk])
        self._done(out)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        slots = self._publish(inp.view(-1))
        chunk = inp.numel()
        flat = out.view(-1)
        for src, t in enumerate(slots):
            flat[src * chunk : (src + 1) * chunk].copy_(t)
        self._done(out)

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        slots = self._publish(t)
        total = slots[0].clone()
        for other in slots[1:]:
            total += other
        _sync(total)
        self.group.barrier.wait()  # every rank has read every input
        t.copy_(total)
        _sync(t)


def run_ranks(world: int, fn):
    """Run ``fn(rank, comm)`` on ``world`` threads; returns the results in rank
    order and re-raises the first exception (the barrier is aborted so the
    other ranks do not wait for it)."""
    group = ThreadGroup(world)
    results: list = [None] * world
    errors: list = []

    def body(rank):
        try:
            results[rank] = fn(rank, group.comm(rank))
        except BaseException as exc:  # noqa: BLE001 - reported below
            errors.append(exc)
            group.barrier.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    if errors:
        raise errors[0]
    return results


def emulated_block_copy(dst, dst_strides, src, src_strides, counts, block_bytes, dst_offset=0, src_offset=0):
    """iris_block_copy semantics on contiguous CPU tensors (byte offsets)."""
    d = dst.reshape(-1).view(torch.uint8)
    s = src.reshape(-1).view(torch.uint8)
    for i0 in range(counts[0]):
        for i1 in range(counts[1]):
            for i2 in range(counts[2]):
                so = src_offset + i0 * src_strides[0] + i1 * src_strides[1] + i2 * src_strides[2]
                do = dst_offset + i0 * dst_strides[0] + i1 * dst_strides[1] + i2 * dst_strides[2]
                d[do : do + block_bytes] = s[so : so + block_bytes]
