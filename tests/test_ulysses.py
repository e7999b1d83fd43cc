"""Sequence-parallel (Ulysses) host logic on the CPU: the shard geometry, the
pack / unpack plans and the engine's exchange steps (ranks as threads, and 2
processes over real gloo collectives). iris_block_copy is emulated by a byte
copy here; the engine itself only ever calls the kernel."""

import os

import pytest
import torch
import torch.multiprocessing as mp

from thread_comm import emulated_block_copy, run_ranks

from iris_b200.ulysses import SequenceShard, gather_image_tokens, gather_tokens, scatter_heads

D = 8  # head width in these tests (the engine uses 128; the plans take it as a parameter)


def test_shard_geometry_covers_the_sequence_once():
    for T, L, P in [(256, 16384, 1), (256, 16384, 2), (256, 16384, 4), (256, 16384, 8), (16, 36, 2), (5, 91, 4)]:
        shards = [SequenceShard(r, P, T, L) for r in range(P)]
        assert sum(s.n for s in shards) == T + L
        assert sum(s.text for s in shards) == T and sum(s.image for s in shards) == L
        starts = [s.image_start for s in shards]
        assert starts == sorted(starts) and all(
            a.image_start + a.image == b.image_start for a, b in zip(shards, shards[1:])
        )
        assert [s.start for s in shards] == [r * (T + L) // P for r in range(P)]
        assert shards[0].image_max == max(s.image for s in shards)


def test_shard_geometry_rejects_unshardable_sequences():
    with pytest.raises(ValueError, match="divisible"):
        SequenceShard(0, 3, 16, 36)
    with pytest.raises(ValueError, match="no image tokens"):
        SequenceShard(0, 4, 16, 16)
    with pytest.raises(ValueError, match="bad rank"):
        SequenceShard(2, 2, 16, 36)


def _exchange_case(rank, comm, T, L, B, H, Hp, seed=0):
    """One rank's side of the three exchanges; returns what it received and
    what it should have received (from the full tensors every rank can build)."""
    P = comm.world
    shard = SequenceShard(rank, P, T, L)
    N, n, hl = T + L, shard.n, H // P
    gen = torch.Generator().manual_seed(seed)
    q_full = torch.randn(B, H, N, D, generator=gen).to(torch.bfloat16)
    o_full = torch.randn(B, N, H * D, generator=gen).to(torch.bfloat16)
    k_full = torch.randn(B, Hp, L, D, generator=gen).to(torch.bfloat16)
    # 1. Q of this rank's tokens, head-major [H, B, n, D] -> heads over all tokens
    local = q_full[:, :, shard.start : shard.start + n].permute(1, 0, 2, 3).contiguous()
    recv = torch.empty(P * hl * B * n * D, dtype=torch.bfloat16)
    full = torch.empty(B, hl, N, D, dtype=torch.bfloat16)
    scatter_heads(comm, emulated_block_copy, local, recv, full, hl, B, n, D)
    # 2. attention output of this rank's heads over all tokens -> all heads of its tokens
    out = o_full.view(B, N, H, D)[:, :, rank * hl : (rank + 1) * hl].reshape(B, N, hl * D).contiguous()
    send, back = torch.empty(B * n * H * D, dtype=torch.bfloat16), torch.empty(B * n * H * D, dtype=torch.bfloat16)
    rows = torch.empty(B * n, H * D, dtype=torch.bfloat16)
    gather_tokens(comm, emulated_block_copy, out, send, back, rows, B, n, hl * D)
    # 3. image-token K of this rank (padded) -> every image token
    pad = shard.image_max
    k_local = torch.zeros(B, Hp, pad, D, dtype=torch.bfloat16)
    k_local[:, :, : shard.image] = k_full[:, :, shard.image_start : shard.image_start + shard.image]
    gathered = torch.empty(P * B * Hp * pad * D, dtype=torch.bfloat16)
    k_all = torch.empty(B, Hp, L, D, dtype=torch.bfloat16)
    gather_image_tokens(comm, emulated_block_copy, shard, k_local, gathered, k_all, B, Hp, D)
    return (
        (full, q_full[:, rank * hl : (rank + 1) * hl]),
        (rows, o_full[:, shard.start : shard.start + n].reshape(B * n, H * D)),
        (k_all, k_full),
    )


@pytest.mark.parametrize("T,L,P,H", [(16, 36, 2, 2), (4, 44, 4, 8), (3, 33, 3, 6)])
def test_exchanges_deliver_the_ulysses_layouts(T, L, P, H):
    results = run_ranks(P, lambda rank, comm: _exchange_case(rank, comm, T, L, B=2, H=H, Hp=3))
    for per_rank in results:
        for got, want in per_rank:
            assert torch.equal(got, want)


def _gloo_worker(rank, world, port, queue):
    import torch.distributed as dist

    from iris_b200.ulysses import TorchComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ok = all(torch.equal(g, w) for g, w in _exchange_case(rank, TorchComm(), 16, 36, B=2, H=2, Hp=3))
        queue.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_exchanges_over_gloo_two_processes():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs)
    results = dict(queue.get(timeout=10) for _ in procs)
    assert results == {0: True, 1: True}


def test_peer_buffers_map_each_peer_allocation_once(monkeypatch):
    """PeerBuffers' host logic with the IPC calls replaced by fakes: this rank's
    entries are its own pointers, every peer buffer is the mapped base of its
    allocation plus the exported offset, an allocation holding several buffers
    is mapped once, and close() unmaps each mapping once."""
    from iris_b200 import kernels as K
    from iris_b200.ulysses import PeerBuffers

    class Buf:  # stands in for a device tensor: only data_ptr() is read
        def __init__(self, ptr):
            self.ptr = ptr

        def data_ptr(self):
            return self.ptr

    world, rank = 3, 1
    names = ("qf", "flags", "o_loc")
    # rank r: "qf" and "flags" share allocation A_r, "o_loc" lives in allocation B_r
    layout = {r: {"qf": (f"A{r}", 0), "flags": (f"A{r}", 4096), "o_loc": (f"B{r}", 256)} for r in range(world)}

    class Comm:
        def __init__(self):
            self.rank, self.world = rank, world

        def all_gather_object(self, obj):
            return [{n: (layout[r][n][0].encode(), layout[r][n][1]) for n in names} if r != rank else obj
                    for r in range(world)]  # fmt: skip

    exported, imported, closed = [], [], []
    monkeypatch.setattr(K, "ipc_export", lambda t: exported.append(t) or (b"mine", 0))
    bases = {f"{a}{r}".encode(): 0x10000 * (r + 1) + (0x1000 if a == "B" else 0) for r in range(world) for a in "AB"}
    monkeypatch.setattr(K, "ipc_import", lambda h: imported.append(h) or bases[h])
    monkeypatch.setattr(K, "ipc_close", lambda base: closed.append(base))
    local = {n: Buf(0x900000 + i * 0x100) for i, n in enumerate(names)}
    pb = PeerBuffers(Comm(), local)
    assert len(exported) == len(names)
    for n in names:
        assert pb.ptrs[n][rank] == local[n].data_ptr()
        for r in range(world):
            if r != rank:
                alloc, off = layout[r][n]
                assert pb.ptrs[n][r] == bases[alloc.encode()] + off
    assert sorted(imported) == sorted({f"{a}{r}".encode() for r in range(world) if r != rank for a in "AB"})
    pb.close()
    assert sorted(closed) == sorted(bases[h] for h in imported)
    pb.close()  # a second close unmaps nothing more
    assert len(closed) == len(imported)
