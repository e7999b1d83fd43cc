"""Pin the CPU oracle against the reference's own outputs (tests/golden/*.pt)."""

import math

import pytest
import torch

from conftest import golden
from oracle import ops
from oracle.config import OracleConfig, PixelConfig, baseline_step_config, released_topology, tiny_cpu_config
from oracle.model import OracleModel
from oracle.params import num_parameters, param_spec, seeded_init
from oracle.sampler import FlowDPMSolverOracle, euler_cfg


def _config(d: dict) -> OracleConfig:
    d = dict(d)
    return OracleConfig(**{**d, "pixel": PixelConfig(**d["pixel"])})


@pytest.mark.parametrize("name", ["released_mha", "released_gqa", "tiny_cpu"])
def test_oracle_forward_matches_reference(name):
    fx = golden(name)
    cfg = _config(fx["config"])
    params = seeded_init(cfg, seed=0)
    for pname, (s, s2) in fx["param_checksums"].items():
        p = params[pname].double()
        assert math.isclose(float(p.sum()), s, rel_tol=1e-9, abs_tol=1e-9), pname
        assert math.isclose(float(p.pow(2).sum()), s2, rel_tol=1e-9), pname
    model = OracleModel(cfg, params)
    with torch.no_grad():
        text = model.embed_text(fx["y"])
        # fp32 sums over 2560 features: the thread count changes the last bits
        torch.testing.assert_close(text, fx["prepared_text"], rtol=1e-4, atol=1e-5)
        capture = {}
        v = model(fx["x"], fx["t"], text, capture=capture)
    torch.testing.assert_close(v, fx["v"], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(capture["block0"], fx["features"][1], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(capture[f"block{cfg.depth - 1}"], fx["features"][cfg.depth], rtol=1e-4, atol=1e-5)


def test_oracle_euler_cfg_matches_reference():
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    model = OracleModel(cfg, seeded_init(cfg, seed=0))
    s = fx["euler_cfg"]
    with torch.no_grad():
        sample = euler_cfg(model, s["noise"], s["cond"], s["uncond"], s["cfg_scale"])
    torch.testing.assert_close(sample, s["sample"], rtol=1e-4, atol=1e-5)


def test_oracle_dpm_sample_of_the_model_matches_reference():
    """The reference's FlowDPMSolver.sample (10 steps, 2nd order, shift 3, CFG 3)
    driving IrisDiT, restated: the oracle solver driving the oracle model."""
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    model = OracleModel(cfg, seeded_init(cfg, seed=0))
    d = fx["dpm"]
    solver = FlowDPMSolverOracle(model, cfg_scale=d["cfg_scale"], cfg_interval=d["cfg_interval"])
    with torch.no_grad():
        sample = solver.sample(d["noise"], d["cond"], d["uncond"], steps=d["steps"], order=d["order"], shift=d["shift"])
    torch.testing.assert_close(sample, d["sample"], rtol=1e-4, atol=1e-4)


def turbo_params(cfg, linear):
    """Seeded weights with every Linear weight and bias rounded to BF16: the
    values a Turbo checkpoint stores (src/iris_metal/loading.py:20-38)."""
    params = seeded_init(cfg, seed=0)
    return {n: (p.to(torch.bfloat16).float() if n in linear else p) for n, p in params.items()}


def test_oracle_turbo_recipe_matches_reference():
    """The FP32 forward on Turbo-rounded weights reproduces the reference's FP32
    run of the Turbo loop, per step and for the sample; the reference's own
    autocast run stays within 1e-2 of it (its BF16 rounding)."""
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    tb = fx["turbo"]
    model = OracleModel(cfg, turbo_params(cfg, set(tb["linear"])))
    with torch.no_grad():
        for step in tb["steps"]:
            v = model(step["x"], step["t"], tb["cond"])
            torch.testing.assert_close(v, step["v_fp32"], rtol=1e-4, atol=1e-5)
            rel = float((step["v_autocast"] - v).abs().max() / v.abs().max())
            assert 0 < rel < 1e-2
        sample = euler_cfg(model, tb["noise"], tb["cond"], None)
    torch.testing.assert_close(sample, tb["fp32"], rtol=1e-4, atol=1e-5)


def depth_engine_inputs(fx):
    """The depth task's denoiser input (src/iris_metal/tasks.py:92-95): RGB plus a
    zero channel at the final timestep."""
    d = fx["depth"]
    rgb = d["rgb"]
    x = torch.cat([rgb, rgb.new_zeros(rgb.shape[0], 1, *rgb.shape[2:])], dim=1)
    return x, torch.full((rgb.shape[0],), d["time"]), d["prepared_text"]


def test_oracle_depth_task_matches_reference():
    """The widened (4-channel) denoiser of a depth fine-tune and the depth
    prediction (1x1 reducer over the velocity) against IrisDepth itself."""
    from oracle.params import depth_task_params

    fx = golden("released_mha")
    cfg = _config(fx["config"])
    params = depth_task_params(cfg)
    reducer = params.pop("depth_reducer.weight"), params.pop("depth_reducer.bias")
    model = OracleModel(cfg, params)
    d = fx["depth"]
    with torch.no_grad():
        v4 = model(d["x4"], d["t4"], d["prepared_text"].expand(2, -1, -1))
        depth = torch.nn.functional.conv2d(model(*depth_engine_inputs(fx)), *reducer)
    torch.testing.assert_close(v4, d["v4"], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(depth, d["depth"], rtol=1e-4, atol=1e-5)


def test_oracle_dpm_solver_matches_reference():
    fx = golden("samplers")
    z, cond, uncond = fx["inputs"]["z"], fx["inputs"]["cond"], fx["inputs"]["uncond"]

    def model_fn(x, t, text):
        return 0.3 * x + 0.05 * text + 1e-4 * t[:, None, None, None]

    for key, case in fx.items():
        if not key.startswith("dpm_"):
            continue
        solver = FlowDPMSolverOracle(model_fn, cfg_scale=case["cfg_scale"])
        assert solver.time_grid(case["steps"], case["shift"]) == case["grid"]
        out = solver.sample(z, cond, uncond, steps=case["steps"], order=case["order"], shift=case["shift"])
        torch.testing.assert_close(out, case["sample"], rtol=1e-6, atol=1e-6)


def test_oracle_op_references_match_reference():
    fx = golden("ops")
    q = fx["qk_norm_rope"]
    ref = ops.qk_norm_rope_reference(q["x"][..., q["col_offset"] :], q["weight"], q["cos"][5:], q["sin"][5:], 1e-6)
    assert torch.equal(ref, q["ref"])
    assert torch.equal(q["out"][:, :, 5:], q["ref"])
    r = fx["rms_norm_modulate"]
    assert torch.equal(
        ops.rms_norm_modulate_reference(r["x"], r["weight"], r["shift"], r["scale"], 1e-6, torch.float32), r["out_f32"]
    )
    g = fx["gated_residual"]
    assert torch.equal(ops.gated_residual_rms_norm_reference(g["residual"], g["branch"], g["weight"], g["gate"], 1e-6), g["out"])
    m = fx["pixel_mlp"]
    new_pixels, nxt = ops.pixel_mlp_reference(
        m["pixels"], m["branch"], m["mods"], m["norm_weight"], m["fc1_w"], m["fc1_b"], m["fc2_w"], m["fc2_b"],
        m["next_norm_weight"], 1e-6,
    )
    assert torch.equal(new_pixels, m["new_pixels"]) and torch.equal(nxt, m["next_input"])
    assert torch.equal(ops.pixel_rms_norm_reference(m["pixels"], m["norm_weight"], 1e-6), m["rms"])


def test_oracle_tables_are_bit_exact():
    fx = golden("ops")
    r = fx["rope"]
    assert torch.equal(torch.view_as_real(ops.rope_2d(128, 64, 64, 1e4, 16.0, "isotropic"))[::16], r["img_64_every16"])
    assert torch.equal(torch.view_as_real(ops.rope_2d(128, 6, 4, 1e4, 16.0, "isotropic")), r["img_6x4"])
    assert torch.equal(torch.view_as_real(ops.rope_2d(64, 8, 8, 1e4, 16.0, "square")), r["img_sq"])
    assert torch.equal(torch.view_as_real(ops.rope_1d(128, 256, 1e4)), r["txt_256"])
    a = fx["apply_rope"]
    cis = ops.rope_2d(128, 3, 3, 1e4, 16.0, "isotropic")
    assert torch.equal(ops.apply_rope(a["q"], cis), a["q_out"]) and torch.equal(ops.apply_rope(a["k"], cis), a["k_out"])
    s = fx["sincos"]
    assert torch.equal(ops.sincos_pos_embed_2d(16, 16, 24), s["t_16x24"])
    assert torch.equal(ops.sincos_pos_embed_2d(16, 64, 64), s["t_64"])
    t = fx["timestep"]
    assert torch.equal(ops.timestep_embedding(t["t"], 256, 10.0), t["feats"])


def test_oracle_inventories_match_full_size_reference():
    fx = golden("inventories")
    for name, cfg in (("baseline_step", baseline_step_config()), ("released_preset", OracleConfig()),
                      ("released_preset_lap", OracleConfig(text_adapter="lap_blocks2"))):  # fmt: skip
        assert [n for n, _, _ in param_spec(cfg)] == fx[name]["names"]
        assert num_parameters(cfg) == fx[name]["numel"]
    # the released preset's parameter count, tests/test_model.py:13-25 of the reference
    assert fx["released_preset_lap"]["numel"] == 2_987_511_888


@pytest.mark.parametrize("adapter", ["lap_blocks2", "blocks2"])
def test_oracle_masked_adapter_matches_reference(adapter):
    """The masked text adapters restated (oracle.adapter) against the reference's
    embed_text on a right-padded prompt, scattered real tokens and an all-pad
    prompt; the seeded weights reproduce the reference's parameter checksums."""
    fx = golden("adapters")[adapter]
    cfg = _config(fx["config"])
    params = seeded_init(cfg, seed=0)
    for name, (total, squares) in fx["param_checksums"].items():
        p = params[name].double()
        assert abs(float(p.sum()) - total) < 1e-6 * max(1.0, abs(total)) and abs(float(p.pow(2).sum()) - squares) < 1e-6
    model = OracleModel(cfg, params)
    with torch.no_grad():
        text = model.embed_text(fx["y"], fx["mask"])
    torch.testing.assert_close(text, fx["prepared_text"], rtol=1e-4, atol=1e-5)
    with pytest.raises(ValueError, match="mask"):
        model.embed_text(fx["y"])


def test_index_maps_round_trip():
    """patchify / pixel regroup / unpatchify are index permutations (integer layout)."""
    x = torch.arange(2 * 3 * 32 * 48, dtype=torch.float64).reshape(2, 3, 32, 48)
    patches = ops.patchify(x, 16)
    assert patches.shape == (2, 6, 768)
    # patch 4 of a 2 x 3 grid sits at (row 1, col 1); features are (c, ky, kx)
    assert patches[1, 4, 0] == x[1, 0, 16, 16] and patches[1, 4, 256 + 17] == x[1, 1, 17, 17]
    px = ops.pixel_regroup(x.permute(0, 2, 3, 1), 16)
    back = ops.unpatchify_pixels(px, 2, 32, 48, 16)
    assert torch.equal(back, x)


def test_tiny_config_shapes():
    cfg = tiny_cpu_config()
    assert cfg.swiglu_hidden == 682
    assert released_topology().kv_heads == 1
