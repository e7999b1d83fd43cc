"""Host-side logic of iris_b200 on the CPU: position tables (bit-exact against
the reference), topology checks, weight packing, samplers, configs."""

import dataclasses

import pytest
import torch

from conftest import golden
from oracle.config import baseline_step_config as oracle_baseline
from oracle.config import released_topology


def test_tables_are_bit_exact_with_reference():
    from iris_b200 import tables

    r = golden("ops")["rope"]
    assert torch.equal(torch.view_as_real(tables.rope_2d(128, 64, 64, 1e4, 16.0, "isotropic"))[::16], r["img_64_every16"])
    assert torch.equal(torch.view_as_real(tables.rope_2d(128, 6, 4, 1e4, 16.0, "isotropic")), r["img_6x4"])
    assert torch.equal(torch.view_as_real(tables.rope_2d(64, 8, 8, 1e4, 16.0, "square")), r["img_sq"])
    assert torch.equal(torch.view_as_real(tables.rope_1d(128, 256, 1e4)), r["txt_256"])
    s = golden("ops")["sincos"]
    assert torch.equal(tables.sincos_pos_embed_2d(16, 16, 24), s["t_16x24"])
    assert torch.equal(tables.sincos_pos_embed_2d(16, 64, 64), s["t_64"])


def test_trunk_table_puts_text_rows_first():
    from iris_b200 import tables

    text, image = tables.rope_1d(128, 5, 1e4), tables.rope_2d(128, 2, 3, 1e4, 16.0, "isotropic")
    cos, sin = tables.cos_sin(text, image, device="cpu")
    assert cos.shape == (11, 64) and cos.is_contiguous()
    assert torch.equal(cos[:5], text.real) and torch.equal(sin[5:], image.imag)


def test_config_round_trip_from_oracle_fields():
    from iris_b200.config import baseline_step_config, from_any

    ours = from_any(oracle_baseline())
    assert ours.hidden_size == 3072 and ours.num_heads == 24 and ours.kv_heads == 24
    assert ours.swiglu_hidden == 8192 and ours.text_len == 256
    assert dataclasses.asdict(baseline_step_config())["pixel"] == dataclasses.asdict(ours.pixel)


@pytest.mark.parametrize(
    "change,missing",
    [
        ({"modulation": "per_block"}, "shared_bias"),
        ({"sandwich_norm": False}, "sandwich"),
        ({"num_heads": 4}, "128-wide"),
        ({"block": "mmdit"}, "single-stream tail"),
    ],
)
def test_check_supported_rejects_other_topologies(change, missing):
    from iris_b200.config import from_any
    from iris_b200.model import check_supported

    cfg = dataclasses.replace(from_any(released_topology()), **change)
    state = {"s_embedder.proj.weight": 0, "t_embedder.mlp.0.weight": 0, "final_layer.linear.weight": 0}
    with pytest.raises(ValueError, match=missing):
        check_supported(cfg, state)
    check_supported(from_any(released_topology()), state)


def test_pack_swiglu_layout():
    from iris_b200.model import pack_swiglu

    ffn, d = 300, 8
    w1 = torch.arange(ffn * d, dtype=torch.float32).reshape(ffn, d)
    w3 = -w1
    w2 = torch.ones(d, ffn)
    w13, w2p = pack_swiglu(w1, w3, w2)
    assert w13.shape == (2 * 384, d) and w2p.shape == (d, 384)
    for tile in range(3):
        rows = slice(tile * 128, min(ffn, (tile + 1) * 128))
        n = rows.stop - rows.start
        assert torch.equal(w13[tile * 256 : tile * 256 + n], w1[rows])
        assert torch.equal(w13[tile * 256 + 128 : tile * 256 + 128 + n], w3[rows])
    assert torch.all(w13[2 * 256 + 44 : 2 * 256 + 128] == 0) and torch.all(w2p[:, ffn:] == 0)


def test_dpm_coefficients_match_oracle_updates():
    """The fused DPM-Solver++ step computes x_next = a x + b x0 + c (x0 - x0_prev);
    its host-side (a, b, c) reproduce the oracle's first- and second-order
    updates (solver.py:84-109) on every step of the golden grids."""
    from iris_b200.sampling import FlowDPMSolver

    from oracle.sampler import FlowDPMSolverOracle

    fx = golden("samplers")
    g = torch.Generator().manual_seed(0)
    x, x0, x0p = (torch.randn(64, generator=g, dtype=torch.float64) for _ in range(3))
    for key, case in fx.items():
        if not key.startswith("dpm_"):
            continue
        grid = FlowDPMSolver.time_grid(case["steps"], case["shift"])
        assert grid == case["grid"]
        steps, order = case["steps"], case["order"]
        for i in range(1, steps + 1):
            s, t = grid[i - 1], grid[i]
            second = min(i, order, steps + 1 - i) == 2
            a, b, c = FlowDPMSolver.coefficients(s, t, grid[i - 2] if second else None)
            fused = a * x + b * x0 + c * (x0 - x0p)
            if second:
                expect = FlowDPMSolverOracle.second_order(x, (grid[i - 2], x0p), (s, x0), t)
            else:
                expect = FlowDPMSolverOracle.first_order(x, s, t, x0)
            torch.testing.assert_close(fused, expect, rtol=1e-12, atol=1e-12)


def test_dp_shards_cover_every_image_once():
    from iris_b200.parallel import image_shard

    for images in (1, 5, 8, 13):
        for world in (1, 2, 4, 8):
            seen = []
            for rank in range(world):
                lo, hi = image_shard(images, rank, world)
                seen.extend(range(lo, hi))
            assert seen == list(range(images))


def _write_checkpoint(root, fx):
    """A released-style checkpoint directory: config.yaml (a training config with
    sections and keys the loader must drop) and model.safetensors (fp32)."""
    import yaml
    from safetensors.torch import save_file

    from oracle.config import OracleConfig, PixelConfig
    from oracle.params import seeded_init

    d = dict(fx["config"])
    cfg = OracleConfig(**{**d, "pixel": PixelConfig(**d["pixel"])})
    params = seeded_init(cfg, seed=0)
    model = {**d, "pixel": {**d["pixel"], "legacy_field": 1}, "unknown_model_key": "x"}
    (root / "config.yaml").write_text(yaml.safe_dump({"model": model, "train": {"lr": 1e-4}, "flow": {}}))
    save_file({k: v.contiguous() for k, v in params.items()}, str(root / "model.safetensors"))
    return d, params


def test_checkpoint_directory_loads_config_and_weights(tmp_path):
    from iris_b200 import IrisWeights

    fx = golden("released_mha")
    d, params = _write_checkpoint(tmp_path, fx)
    w = IrisWeights.from_checkpoint(tmp_path, device="cpu")
    for key, value in d.items():
        if key != "pixel":
            assert getattr(w.cfg, key) == value, key
    for key, value in d["pixel"].items():
        assert getattr(w.cfg.pixel, key) == value, key
    state = w.state_dict()
    assert set(state) == set(params)
    for key, value in params.items():
        assert torch.equal(state[key], value), key


def test_score_bound_covers_aligned_rms_normed_rows():
    """kernels.score_bound bounds |q . k| * scale for RMS-normed rows times their
    gains, also for the worst case: q and k both along the largest gains."""
    from iris_b200 import kernels as K

    gen = torch.Generator().manual_seed(3)
    for gain in (0.5, 1.0, 4.0):
        gq = gain * (1 + 0.3 * torch.rand(128, generator=gen))
        gk = gain * (1 + 0.3 * torch.rand(128, generator=gen))
        bound = K.score_bound([gq], [gk])

        def normed(x, g):
            return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * g

        worst = torch.zeros(128)
        worst[int(gq.argmax())] = 1.0  # all mass on one dimension: norm sqrt(128) there
        q = normed(torch.cat([torch.randn(64, 128, generator=gen), worst[None]]), gq).to(torch.bfloat16).float()
        k = normed(torch.cat([torch.randn(64, 128, generator=gen), worst[None] * -1]), gk).to(torch.bfloat16).float()
        scores = (q @ k.T) * 128**-0.5
        assert float(scores.abs().max()) <= bound
        assert float(scores.abs().max()) > 0.5 * bound  # and the bound is not loose by more than 2x
    # several streams share one bound: the largest gains of each side
    assert K.score_bound([torch.ones(128), 2 * torch.ones(128)], [torch.ones(128)]) == K.score_bound(
        [2 * torch.ones(128)], [torch.ones(128)])
