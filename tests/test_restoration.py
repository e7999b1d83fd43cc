"""Host side of the tiled restorer against the reference's own tiling
(tests/golden/restoration.pt, made by running src/iris3b/downstream/restoration.py
and src/iris_metal/tasks.py): tile positions, the Gaussian window (bit-exact),
tile counts, and the split of the tiles over ranks."""

from types import SimpleNamespace

import torch

from conftest import golden


def _restorer(tile=1024, patch=16):
    from iris_b200.restoration import TiledRestorer

    engine = SimpleNamespace(device=torch.device("cpu"), cfg=SimpleNamespace(patch_size=patch))
    return TiledRestorer(engine, torch.zeros(1, 4, 8), tile=tile)


def test_tile_positions_and_window_match_reference():
    from iris_b200.restoration import gaussian_window, tile_positions

    fx = golden("restoration")
    for size, want in fx["positions_1024"].items():
        assert tile_positions(size, 1024, 512) == want
    assert torch.equal(gaussian_window(32), fx["window_32"])
    assert torch.equal(gaussian_window(1024)[::37, ::37], fx["window_1024_every_37"])


def test_tile_count_matches_reference():
    fx = golden("restoration")
    restorer = _restorer()
    for size, want in fx["tile_counts"].items():
        assert restorer.tile_count(size) == want, size


def test_tile_plan_splits_every_tile_once_in_order():
    from iris_b200.restoration import tile_plan

    for height, width in ((2048, 4096), (2048, 2048), (1040, 1024)):
        tiles, _ = tile_plan(height, width, 1024)
        for world in (1, 2, 3, 4, 8):
            shares = [tile_plan(height, width, 1024, r, world)[1] for r in range(world)]
            assert [t for share in shares for t in share] == tiles
            assert max(map(len, shares)) - min(map(len, shares)) <= 1
    assert len(tile_plan(2048, 4096, 1024)[0]) == 21  # 4x of 512 x 1024: the budget's largest image
