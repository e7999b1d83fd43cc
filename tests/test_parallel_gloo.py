"""The N > 1 path on CPU: two gloo ranks sample their image shards with the
oracle model (standing in for the device engine) and gather; the result equals
the single-process batch bit for bit. A rank that never joins makes the other
fail with a timeout error rather than hang."""

import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sample_all(images: int):
    from oracle.config import released_topology
    from oracle.model import OracleModel
    from oracle.params import seeded_init
    from oracle.sampler import euler_cfg

    cfg = released_topology(num_kv_heads=None, depth=2)
    model = OracleModel(cfg, seeded_init(cfg, seed=0))
    gen = torch.Generator().manual_seed(3)
    noise = torch.randn(images, 3, 16, 16, generator=gen)
    cond = torch.randn(images, cfg.text_len, cfg.hidden_size, generator=gen)
    uncond = torch.randn(1, cfg.text_len, cfg.hidden_size, generator=gen)
    return model, noise, cond, uncond, euler_cfg


def _rank_main(rank, world, port, images, queue):
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "iris-3b-metal_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    torch.set_num_threads(1)
    from iris_b200.parallel import gather_images, image_shard, init_process_group

    init_process_group("gloo", timeout_s=60)
    import torch.distributed as dist

    model, noise, cond, uncond, euler_cfg = _sample_all(images)
    lo, hi = image_shard(images, rank, world)
    with torch.no_grad():
        local = euler_cfg(model, noise[lo:hi], cond[lo:hi], uncond, 3.0)
    full = gather_images(local, images)
    if rank == 0:
        queue.put(full)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_data_parallel_equals_single_process():
    images, world = 3, 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, images, queue)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = queue.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    model, noise, cond, uncond, euler_cfg = _sample_all(images)
    threads = torch.get_num_threads()
    torch.set_num_threads(1)  # the ranks ran single-threaded: same summation order
    from iris_b200.parallel import image_shard

    try:
        with torch.no_grad():
            # the same slices in one process, so each matmul sees the same shapes
            shards = [image_shard(images, r, world) for r in range(world)]
            single = torch.cat([euler_cfg(model, noise[lo:hi], cond[lo:hi], uncond, 3.0) for lo, hi in shards])
    finally:
        torch.set_num_threads(threads)
    assert torch.equal(gathered, single)


def _lonely_rank(port, queue):
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "iris-3b-metal_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0", WORLD_SIZE="2")
    from iris_b200.parallel import init_process_group

    try:
        init_process_group("gloo", timeout_s=3)
        queue.put("joined")
    except Exception as exc:  # the missing rank surfaces as an error, not a hang
        queue.put(type(exc).__name__)


def test_missing_rank_times_out_instead_of_hanging():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(_free_port(), queue))
    p.start()
    outcome = queue.get(timeout=120)
    p.join(timeout=60)
    if p.is_alive():
        p.kill()
        pytest.fail("rank hung")
    assert outcome != "joined"
