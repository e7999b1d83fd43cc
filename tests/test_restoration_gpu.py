"""The tiled restorer on the B200 against the reference's ``tiled`` with
``restore_tile`` (src/iris3b/downstream/restoration.py:87-101,
src/iris_metal/tasks.py:143-150) on the toy model (tests/golden/restoration.pt),
the tile kernels against torch, and the tiles split over two GPUs."""

import math
import os

import pytest
import torch

from conftest import golden, requires_gpu
from oracle.config import OracleConfig, PixelConfig
from oracle.params import seeded_init

pytestmark = requires_gpu

REL_TOL = 2e-2
PSNR_MIN = 40.0


def _config(d):
    d = dict(d)
    return OracleConfig(**{**d, "pixel": PixelConfig(**d["pixel"])})


def rel_err(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max())


def psnr(a, ref):
    a, ref = a.double().cpu(), ref.double().cpu()
    mse = float(((a - ref) ** 2).mean())
    return 10 * math.log10(float(ref.max() - ref.min()) ** 2 / mse) if mse > 0 else math.inf


@pytest.fixture(scope="module")
def restorer():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import iris_b200
    from iris_b200.restoration import TiledRestorer

    fx = golden("released_mha")
    cfg = _config(fx["config"])
    engine = iris_b200.CudaIris(iris_b200.IrisWeights(cfg, {k: v.cuda() for k, v in seeded_init(cfg, 0).items()}))
    r = golden("restoration")
    return TiledRestorer(engine, r["text"].cuda(), sigma=r["sigma"], tile=r["tile"], tiles_per_call=4), r


def test_tiled_restoration_matches_reference(restorer):
    tr, r = restorer
    out = tr(r["x"].cuda())
    err, value = rel_err(out, r["fused"]), psnr(out, r["fused"])
    print(f"tiled restoration (6 tiles): max rel err {err:.2e}, psnr {value:.1f} dB")
    assert out.shape == r["fused"].shape
    assert err < REL_TOL and value > PSNR_MIN
    single = tr(r["x"][..., :32, :32].cuda())  # one tile: restore_tile, no window
    assert rel_err(single, r["single"]) < REL_TOL
    tr.tiles_per_call = 1  # one tile per engine call, as the reference runs them
    one = tr(r["x"].cuda())
    tr.tiles_per_call = 4
    assert rel_err(one, out) < 1e-3


def test_on_tile_runs_before_every_tile_and_stops_the_image(restorer):
    tr, r = restorer
    seen = []
    tr.on_tile = lambda: seen.append(1)
    try:
        tr(r["x"].cuda())
        assert len(seen) == 6

        def stop():
            raise InterruptedError

        tr.on_tile = stop
        with pytest.raises(InterruptedError):
            tr(r["x"].cuda())
    finally:
        tr.on_tile = None
    with pytest.raises(ValueError, match="both sides"):
        tr(torch.zeros(1, 3, 24, 64, device="cuda"))


def test_tile_kernels_match_torch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from iris_b200 import _lib
    from iris_b200.restoration import gaussian_window

    st = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(3, 80, 96, device="cuda", generator=gen)
    crop = torch.empty(3, 32, 32, device="cuda")
    _lib.call("iris_tile_crop", x.data_ptr(), 3, 80, 96, 48, 64, 32, crop.data_ptr(), st)
    assert torch.equal(crop, x[:, 48:80, 64:96])
    v = torch.randn(3, 32, 32, device="cuda", generator=gen)
    w = gaussian_window(32).cuda()
    out, weight = torch.randn(3, 80, 96, device="cuda", generator=gen), torch.rand(80, 96, device="cuda", generator=gen)
    want_out, want_w = out.clone(), weight.clone()
    want_out[:, 48:80, 64:96] += (x[:, 48:80, 64:96] - 0.5 * v) * w
    want_w[48:80, 64:96] += w
    _lib.call("iris_tile_accumulate", x.data_ptr(), 3, 80, 96, v.data_ptr(), 32, w.data_ptr(), 48, 64, 0.5,
              out.data_ptr(), weight.data_ptr(), st)  # fmt: skip
    torch.testing.assert_close(out, want_out, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(weight, want_w, rtol=0, atol=0)
    _lib.call("iris_tile_normalize", out.data_ptr(), weight.data_ptr(), 3, 80, 96, st)
    torch.testing.assert_close(out, want_out / want_w, rtol=1e-6, atol=1e-6)
    with pytest.raises(ValueError, match="inside the image"):
        _lib.call("iris_tile_crop", x.data_ptr(), 3, 80, 96, 60, 64, 32, crop.data_ptr(), st)


def _dp_worker(rank, world, port, queue):
    import torch.distributed as dist

    import iris_b200
    from iris_b200.restoration import TiledRestorer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        fx = golden("released_mha")
        cfg = _config(fx["config"])
        engine = iris_b200.CudaIris(iris_b200.IrisWeights(cfg, {k: v.cuda() for k, v in seeded_init(cfg, 0).items()}))
        r = golden("restoration")
        seen = []
        tr = TiledRestorer(engine, r["text"].cuda(), sigma=r["sigma"], tile=r["tile"], group=dist.group.WORLD)
        tr.on_tile = lambda: seen.append(1)
        out = tr(r["x"].cuda())
        alone = TiledRestorer(engine, r["text"].cuda(), sigma=r["sigma"], tile=r["tile"])(r["x"].cuda())
        torch.cuda.synchronize()
        queue.put((rank, len(seen), rel_err(out, alone), rel_err(out, r["fused"])))
    finally:
        dist.destroy_process_group()


def test_tiles_split_over_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    results = [queue.get(timeout=10) for _ in procs]
    print("tiles over 2 GPUs (rank, tiles, err vs one GPU, err vs reference):", results)
    assert sorted(n for _, n, _, _ in results) == [3, 3]
    assert all(e1 < 1e-3 and e2 < REL_TOL for _, _, e1, e2 in results)
