"""Generate the golden fixtures by running the REFERENCE's own code.

Run in a container where the reference sources are available:

    python tests/golden/make_golden.py --reference <path to iris-3b-metal checkout>

It imports ``iris3b`` / ``iris_metal`` from ``<reference>/src`` (with a stub for
``omegaconf``, which only the config loader needs), builds ``IrisDiT`` for the
small configs, applies the seeded init recipe to the reference model itself,
and stores inputs and outputs as ``tests/golden/*.pt``. Nothing under
``tests/`` reads the reference at run time; the tests read these files.
"""

from __future__ import annotations

import argparse
import dataclasses
import math
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import config as ocfg  # noqa: E402
from oracle.params import STD, param_spec  # noqa: E402


def _import_reference(root: Path):
    stub = types.ModuleType("omegaconf")
    stub.OmegaConf = type("OmegaConf", (), {})
    sys.modules.setdefault("omegaconf", stub)
    sys.path.insert(0, str(root / "src"))
    from iris3b.config import ModelConfig, PixelStageConfig
    from iris3b.models.dit import IrisDiT

    return ModelConfig, PixelStageConfig, IrisDiT


def _reference_config(cfg: ocfg.OracleConfig, ModelConfig, PixelStageConfig):
    fields = {f.name for f in dataclasses.fields(ModelConfig)}
    values = {k: v for k, v in dataclasses.asdict(cfg).items() if k in fields and k != "pixel"}
    pixel = PixelStageConfig(**dataclasses.asdict(cfg.pixel))
    return ModelConfig(**values, pixel=pixel)


def _seed_reference(model, seed: int) -> None:
    """The recipe of ``oracle.params.seeded_init`` applied to the reference model."""
    from iris3b.nn.norms import RMSNorm

    gains = {id(m.weight) for m in model.modules() if isinstance(m, RMSNorm)}
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for _, p in model.named_parameters():
            value = torch.randn(p.shape, generator=gen) * STD
            if id(p) in gains:
                value += 1.0
            p.copy_(value)


def _model_fixture(name, cfg, ModelConfig, PixelStageConfig, IrisDiT, batch, height, width, times):
    rcfg = _reference_config(cfg, ModelConfig, PixelStageConfig)
    model = IrisDiT(rcfg).eval()
    ref_spec = [(n, tuple(p.shape)) for n, p in model.named_parameters()]
    ours = [(n, tuple(s)) for n, s, _ in param_spec(cfg)]
    assert ref_spec == ours, f"{name}: parameter inventory differs from the reference"
    _seed_reference(model, seed=0)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(batch, 3, height, width, generator=gen)
    y = torch.randn(batch, cfg.text_len, cfg.text_dim, generator=gen)
    t = torch.tensor(times, dtype=torch.float32)
    with torch.no_grad():
        prepared = model.embed_text(y)
        out = model(x, t, y, capture=(1, cfg.depth)).x
        features = model(x, t, y, capture=(1, cfg.depth)).features
    checksums = {n: (float(p.detach().double().sum()), float(p.detach().double().pow(2).sum()))
                 for n, p in model.named_parameters()}
    return {
        "config": dataclasses.asdict(cfg),
        "x": x,
        "t": t,
        "y": y,
        "prepared_text": prepared,
        "v": out,
        "features": {k: v.clone() for k, v in features.items()},
        "param_checksums": checksums,
    }, model


def _sample_fixture(model, fixture, cfg_scale=3.0, cfg_interval=(0.0, 1.5)):
    """4-step Turbo Euler with CFG, using the reference's own ``generate_few_step``
    and ``FlowDPMSolver._model_out`` (CFG on ``[uncond; cond]``). The interval
    ``(0, 1.5)`` keeps CFG on at sigma = 1 too (the reference's default ``(0, 1)``
    gates it off there), which is the all-steps-guided workload of the benchmark."""
    from iris3b.flow.solver import FlowDPMSolver
    from iris3b.sampling import generate_few_step
    from iris_metal.turbo import TURBO_SIGMAS

    prepared = fixture["prepared_text"]
    cond, uncond = prepared[1:], prepared[:1]
    noise = torch.randn(1, 3, fixture["x"].shape[2], fixture["x"].shape[3], generator=torch.Generator().manual_seed(5))

    def velocity(x, t_model, text):
        # the reference forward on adapted text (prepared_text), fp32
        return model(x, t_model, text, prepared_text=text, precompute_modulation=True).x

    solver = FlowDPMSolver(velocity, cfg_scale=cfg_scale, cfg_interval=cfg_interval)

    class CfgModel:
        cfg = model.cfg

        def parameters(self):
            return model.parameters()

        def __call__(self, x, t, y, y_mask):
            return SimpleNamespace(x=solver._model_out(x, float(t[0]) / 1000.0, cond, uncond))

    class Encoder:
        def encode(self, prompts):
            return SimpleNamespace(embeddings=torch.zeros(1), mask=torch.ones(1))

    seen = []
    with torch.no_grad():
        generate_few_step(
            CfgModel(), Encoder(), ["p"], noise.shape[2], noise.shape[3], list(TURBO_SIGMAS),
            noise=noise, device="cpu", check=seen.append,
        )  # fmt: skip
    return {"noise": noise, "cond": cond, "uncond": uncond, "cfg_scale": cfg_scale, "cfg_interval": cfg_interval,
            "sample": seen[0]}


def _dpm_fixture(model, fixture, steps=10, order=2, shift=3.0, cfg_scale=3.0):
    """The Original model's loop: the reference's ``FlowDPMSolver.sample``
    (``src/iris3b/flow/solver.py:112-141``; 2nd-order multistep, CFG on
    ``[uncond; cond]`` inside its default interval) driving the FP32 forward on
    adapted text."""
    from iris3b.flow.solver import FlowDPMSolver

    prepared = fixture["prepared_text"]
    cond, uncond = prepared[1:], prepared[:1]
    noise = torch.randn(1, 3, fixture["x"].shape[2], fixture["x"].shape[3], generator=torch.Generator().manual_seed(7))

    def velocity(x, t_model, text):
        return model(x, t_model, text, prepared_text=text, precompute_modulation=True).x

    solver = FlowDPMSolver(velocity, cfg_scale=cfg_scale)
    with torch.no_grad():
        sample = solver.sample(noise, cond, uncond, steps=steps, order=order, shift=shift)
    return {"noise": noise, "cond": cond, "uncond": uncond, "steps": steps, "order": order, "shift": shift,
            "cfg_scale": cfg_scale, "cfg_interval": solver.cfg_interval, "sample": sample}


def _turbo_fixture(model, fixture):
    """The Turbo recipe (``IrisPipeline._turbo``, ``src/iris_metal/pipeline.py:372-428``)
    on the toy model: every Linear weight and bias stored in BF16
    (``linear_dtypes`` with a BF16 trunk, ``src/iris_metal/loading.py:20-38``), every
    other parameter FP32, the forward under BF16 autocast with prepared text and
    the shared_bias cores evaluated once per forward; the reference's own
    ``generate_few_step`` (B = 1, no CFG, TURBO_SIGMAS). The same loop is also run
    in FP32 on the same BF16-valued weights: the exact arithmetic that both the
    autocast forward and the CUDA engine approximate. Each autocast step's input is
    also kept, with its velocity under autocast and in FP32."""
    import copy

    from iris3b.sampling import generate_few_step
    from iris_metal.loading import linear_dtypes
    from iris_metal.turbo import TURBO_SIGMAS

    turbo = copy.deepcopy(model)
    linear = linear_dtypes(turbo, torch.bfloat16)
    with torch.no_grad():
        for name, p in turbo.named_parameters():
            if name in linear:
                p.data = p.data.to(linear[name])
    exact = copy.deepcopy(turbo).float()
    cond = fixture["prepared_text"][1:]
    noise = torch.randn(1, 3, fixture["x"].shape[2], fixture["x"].shape[3], generator=torch.Generator().manual_seed(6))

    def run(net, autocast, calls=None):
        class Model:
            cfg = net.cfg

            def parameters(self):
                return net.parameters()

            def __call__(self, x, t, y, y_mask):
                out = net(x, t, y, y_mask=y_mask, prepared_text=cond, precompute_modulation=True)
                if calls is not None:
                    calls.append((x.clone(), t.clone(), out.x.float()))
                return out

        class Encoder:
            def encode(self, prompts):
                return SimpleNamespace(embeddings=cond, mask=torch.ones(1, cond.shape[1]))

        seen = []
        with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16, enabled=autocast):
            generate_few_step(Model(), Encoder(), ["p"], noise.shape[2], noise.shape[3], list(TURBO_SIGMAS),
                              noise=noise, device="cpu", check=seen.append)  # fmt: skip
        return seen[0].float()

    calls = []
    sample = run(turbo, True, calls)
    steps = []
    with torch.no_grad():
        for x, t, v in calls:  # each step's input, also through the FP32 forward
            exact_v = exact(x, t, cond, prepared_text=cond, precompute_modulation=True).x
            steps.append({"x": x, "t": t, "v_autocast": v, "v_fp32": exact_v})
    return {"noise": noise, "cond": cond, "linear": sorted(linear), "autocast": sample, "fp32": run(exact, False),
            "steps": steps}


def _depth_fixture(cfg, fixture, ModelConfig, PixelStageConfig):
    """The depth fine-tune (``IrisDepth``, ``src/iris3b/downstream/depth.py:30-49``) on
    the toy topology, weights from ``oracle.params.depth_task_params``: its own
    ``forward`` (RGB plus a zero channel at the final timestep, then the 1x1
    reducer), and the widened denoiser on a 4-channel input whose extra channel is
    not zero (the general case of an engine built on ``model.pixel``)."""
    from iris3b.downstream.depth import IrisDepth

    from oracle.params import depth_task_params

    model = IrisDepth(_reference_config(cfg, ModelConfig, PixelStageConfig)).eval()
    params = depth_task_params(cfg)
    state = {("" if k.startswith("depth_reducer") else "pixel.") + k: v for k, v in params.items()}
    model.load_state_dict(state, strict=True)
    gen = torch.Generator().manual_seed(8)
    rgb = torch.rand(1, 3, fixture["x"].shape[2], fixture["x"].shape[3], generator=gen) * 2 - 1
    x4 = torch.randn(2, 4, rgb.shape[2], rgb.shape[3], generator=gen)
    y = fixture["y"][1:]
    t = torch.tensor([1000.0, 431.0])
    with torch.no_grad():
        depth = model(rgb, y, torch.ones(1, y.shape[1], dtype=torch.bool))
        text = model.pixel.embed_text(y)
        v4 = model.pixel(x4, t, y.expand(2, -1, -1), prepared_text=text.expand(2, -1, -1)).x
    return {"rgb": rgb, "y": y, "prepared_text": text, "depth": depth, "x4": x4, "t4": t, "v4": v4,
            "time": float(model.num_train_timesteps)}


def _restoration_fixture(model, fixture):
    """The restorer's tiling (``tiled`` / ``gaussian_window`` / ``tile_positions``,
    ``src/iris3b/downstream/restoration.py:68-101``) with ``restore_tile``'s
    ``x - sigma v`` at model time 500 (``src/iris_metal/tasks.py:143-150``) on the
    toy model and adapted text standing in for the export's empty prompt: a
    48 x 64 image in 32-pixel tiles (stride 16, six tiles, as the reference's
    tests/test_metal_tasks.py uses tile 32), and a 32 x 32 image (one tile, no
    window). Also the tile positions and windows at the release's tile of 1024,
    and ``MetalRestorer.tile_count`` for several input sizes."""
    from iris3b.downstream.restoration import gaussian_window, tile_positions, tiled
    from iris_metal.tasks import MetalRestorer

    text = fixture["prepared_text"][1:]
    sigma, tile = 0.5, 32

    def restore(crop):
        b = crop.shape[0]
        t = torch.full((b,), sigma * 1000.0)
        y = text.expand(b, -1, -1)
        return crop - sigma * model(crop, t, y, prepared_text=y, precompute_modulation=True).x

    gen = torch.Generator().manual_seed(21)
    x = torch.rand(1, 3, 48, 64, generator=gen) * 2 - 1
    with torch.no_grad():
        fused = tiled(restore, x, tile, tile // 2)
        single = tiled(restore, x[..., :tile, :tile], tile, tile // 2)
    positions = {size: tile_positions(size, 1024, 512) for size in (1024, 1040, 1536, 2048, 2064, 4096)}
    counter = SimpleNamespace(tile=1024, patch=16)
    sizes = ((256, 256), (512, 512), (512, 1024), (1024, 512), (300, 200), (257, 1023), (64, 256))
    return {"x": x, "text": text, "sigma": sigma, "tile": tile, "fused": fused, "single": single,
            "window_32": gaussian_window(tile, torch.device("cpu"))[0, 0],
            "window_1024_every_37": gaussian_window(1024, torch.device("cpu"))[0, 0, ::37, ::37].clone(),
            "positions_1024": positions,
            "tile_counts": {size: MetalRestorer.tile_count(counter, size) for size in sizes}}  # fmt: skip


def _adapter_fixtures(ModelConfig, PixelStageConfig, IrisDiT):
    """The masked text adapters through the reference's own ``IrisDiT.embed_text``
    (``src/iris3b/models/dit.py:263-281``): ``lap_blocks2`` (``LayerwiseTextEmbedder``,
    ``src/iris3b/nn/embeddings.py:209-266``) and ``blocks2``
    (``TransformerTextEmbedder``, ``:144-207``) on the toy topology with text
    states of width 640 (8 layer-attention heads of 80, as 2560 / 32 in the
    release) and 3 encoder layers; seeded init recipe over the whole model. The
    masks cover a right-padded prompt, real tokens at scattered positions and a
    prompt of padding only (identity attention on the diagonal); the states run
    4 tokens past ``text_len`` (truncated by embed_text)."""
    out = {}
    mask = torch.zeros(3, 20, dtype=torch.bool)
    mask[0, :13] = True
    mask[1, ::3] = True
    mask[1, 7] = True
    for adapter in ("lap_blocks2", "blocks2"):
        cfg = ocfg.released_topology(num_kv_heads=None, text_adapter=adapter, text_dim=640, text_lap_num_layers=3,
                                     text_lap_num_heads=8)  # fmt: skip
        model = IrisDiT(_reference_config(cfg, ModelConfig, PixelStageConfig)).eval()
        ref_spec = [(n, tuple(p.shape)) for n, p in model.named_parameters()]
        assert ref_spec == [(n, tuple(s)) for n, s, _ in param_spec(cfg)], f"{adapter}: inventory differs"
        _seed_reference(model, seed=0)
        gen = torch.Generator().manual_seed(12)
        shape = (3, 20, 3, 640) if adapter == "lap_blocks2" else (3, 20, 640)
        y = torch.randn(shape, generator=gen)
        with torch.no_grad():
            text = model.embed_text(y, mask)
            bare = model.y_embedder(y[:, : cfg.text_len], mask[:, : cfg.text_len])
        checksums = {n: (float(p.detach().double().sum()), float(p.detach().double().pow(2).sum()))
                     for n, p in model.named_parameters() if n.startswith("y_embedder.")}  # fmt: skip
        out[adapter] = {"config": dataclasses.asdict(cfg), "y": y, "mask": mask, "prepared_text": text,
                        "adapter_out": bare, "param_checksums": checksums}  # fmt: skip
        print(adapter, "adapter", tuple(text.shape), float(text.abs().max()))
    return out


def _op_fixtures():
    from iris3b.nn.embeddings import TimestepEmbedder, sincos_pos_embed_2d
    from iris3b.nn.rope import apply_rope, rope_1d, rope_2d
    from iris_metal.kernels import (
        gated_residual_rms_norm_,
        pixel_mlp_,
        pixel_rms_norm,
        qk_norm_rope,
        qk_norm_rope_reference,
        rms_norm_modulate,
    )

    gen = torch.Generator().manual_seed(0)
    out = {}
    # qk_norm_rope at the shapes of tests/test_metal_engine.py:159-176 (CPU branch)
    batch, tokens, heads = 2, 37, 3
    fused = torch.randn(batch, tokens, 2 * heads * 128, generator=gen)
    weight = torch.rand(128, generator=gen) + 0.5
    angles = torch.rand(tokens + 5, 64, generator=gen) * 6.0
    cos, sin = angles.cos(), angles.sin()
    dst = torch.zeros(batch, heads, tokens + 5, 128)
    qk_norm_rope(fused, weight, cos, sin, 1e-6, heads, col_offset=heads * 128, out=dst, offset=5)
    out["qk_norm_rope"] = dict(x=fused, weight=weight, cos=cos, sin=sin, heads=heads, col_offset=heads * 128,
                               offset=5, out=dst,
                               ref=qk_norm_rope_reference(fused[..., heads * 128:], weight, cos[5:], sin[5:], 1e-6))
    # row kernels at tests/test_metal_engine.py:191-207
    x = torch.randn(2, 7, 384, generator=gen)
    branch = torch.randn(2, 7, 384, generator=gen)
    w = torch.rand(384, generator=gen) + 0.5
    shift, scale, gate = (torch.randn(2, 1, 384, generator=gen) for _ in range(3))
    out["rms_norm_modulate"] = dict(x=x, weight=w, shift=shift, scale=scale,
                                    out_f32=rms_norm_modulate(x, w, shift, scale, 1e-6, torch.float32),
                                    out_bf16=rms_norm_modulate(x, w, shift, scale, 1e-6, torch.bfloat16))
    out["gated_residual"] = dict(residual=x, branch=branch, weight=w, gate=gate,
                                 out=gated_residual_rms_norm_(x.clone(), branch, w, gate, 1e-6))
    # pixel kernels at tests/test_metal_engine.py:258-289
    bf16 = torch.bfloat16
    pixels = torch.randn(5, 256, 16, generator=gen).to(bf16)
    pbranch = torch.randn(5, 256, 16, generator=gen).to(bf16)
    mods = (torch.randn(5, 256, 64, generator=gen) * 0.3).to(bf16)
    nw, nxt = (torch.rand(16, generator=gen) + 0.5 for _ in range(2))
    torch.manual_seed(0)
    fc1, fc2 = torch.nn.Linear(16, 64).to(bf16), torch.nn.Linear(64, 16).to(bf16)
    new_pixels = pixels.clone()
    nxt_in = pixel_mlp_(new_pixels, pbranch, mods, nw, fc1, fc2, nxt, 1e-6)
    out["pixel_mlp"] = dict(pixels=pixels, branch=pbranch, mods=mods, norm_weight=nw, next_norm_weight=nxt,
                            fc1_w=fc1.weight.detach(), fc1_b=fc1.bias.detach(), fc2_w=fc2.weight.detach(),
                            fc2_b=fc2.bias.detach(), new_pixels=new_pixels, next_input=nxt_in,
                            rms=pixel_rms_norm(pixels, nw, 1e-6))
    # tables
    out["rope"] = dict(img_64_every16=torch.view_as_real(rope_2d(128, 64, 64, 1e4, 16.0, "isotropic"))[::16].clone(),
                       img_6x4=torch.view_as_real(rope_2d(128, 6, 4, 1e4, 16.0, "isotropic")),
                       img_sq=torch.view_as_real(rope_2d(64, 8, 8, 1e4, 16.0, "square")),
                       txt_256=torch.view_as_real(rope_1d(128, 256, 1e4)))
    q = torch.randn(2, 9, 3, 128, generator=gen)
    k = torch.randn(2, 9, 3, 128, generator=gen)
    cis = rope_2d(128, 3, 3, 1e4, 16.0, "isotropic")
    qr, kr = apply_rope(q, k, cis)
    out["apply_rope"] = dict(q=q, k=k, q_out=qr, k_out=kr)
    out["sincos"] = dict(t_16x24=sincos_pos_embed_2d(16, 16, 24), t_64=sincos_pos_embed_2d(16, 64, 64))
    emb = TimestepEmbedder(64, max_period=10.0)
    tt = torch.tensor([0.0, 125.0, 625.0, 938.0, 1000.0])
    out["timestep"] = dict(t=tt, feats=emb.timestep_embedding(tt))
    return out


def _sampler_fixtures():
    """Known answers of the samplers with toy models (``tests/test_metal_turbo.py:24-73``,
    ``tests/test_flow.py``)."""
    from iris3b.flow.solver import FlowDPMSolver

    out = {}
    gen = torch.Generator().manual_seed(17)
    z = torch.randn(2, 3, 8, 8, generator=gen)
    cond = torch.randn(2, 3, 8, 8, generator=gen)
    uncond = torch.randn(2, 3, 8, 8, generator=gen)

    def model_fn(x, t, text):
        return 0.3 * x + 0.05 * text + 1e-4 * t[:, None, None, None]

    for steps, order, shift, scale in ((4, 1, 1.0, 3.0), (10, 2, 4.0, 3.0), (7, 2, 3.0, 1.0)):
        solver = FlowDPMSolver(model_fn, cfg_scale=scale, cfg_interval=(0.0, 1.0))
        out[f"dpm_{steps}_{order}_{shift}_{scale}"] = dict(
            steps=steps, order=order, shift=shift, cfg_scale=scale,
            grid=FlowDPMSolver.time_grid(steps, shift),
            sample=solver.sample(z, cond, uncond, steps=steps, order=order, shift=shift))
    out["inputs"] = dict(z=z, cond=cond, uncond=uncond)
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, type=Path)
    parser.add_argument("--only", choices=["adapters"], help="regenerate one fixture file only")
    args = parser.parse_args()
    torch.set_num_threads(8)
    ModelConfig, PixelStageConfig, IrisDiT = _import_reference(args.reference)
    if args.only != "adapters":
        _model_fixtures(ModelConfig, PixelStageConfig, IrisDiT)
    torch.save(_adapter_fixtures(ModelConfig, PixelStageConfig, IrisDiT), HERE / "adapters.pt")


def _model_fixtures(ModelConfig, PixelStageConfig, IrisDiT):
    fixtures = {
        "released_mha": (ocfg.released_topology(num_kv_heads=None), 2, 24, 24, [125.0, 850.0]),
        "released_gqa": (ocfg.released_topology(), 2, 24, 16, [125.0, 850.0]),
        "tiny_cpu": (ocfg.tiny_cpu_config(), 1, 128, 128, [431.0]),
    }
    for name, (cfg, batch, h, w, times) in fixtures.items():
        fixture, model = _model_fixture(name, cfg, ModelConfig, PixelStageConfig, IrisDiT, batch, h, w, times)
        if name == "released_mha":
            fixture["euler_cfg"] = _sample_fixture(model, fixture)
            fixture["turbo"] = _turbo_fixture(model, fixture)
            fixture["dpm"] = _dpm_fixture(model, fixture)
            fixture["depth"] = _depth_fixture(cfg, fixture, ModelConfig, PixelStageConfig)
            torch.save(_restoration_fixture(model, fixture), HERE / "restoration.pt")
        torch.save(fixture, HERE / f"{name}.pt")
        print(name, "saved", tuple(fixture["v"].shape), float(fixture["v"].abs().max()))
    torch.save(_op_fixtures(), HERE / "ops.pt")
    torch.save(_sampler_fixtures(), HERE / "samplers.pt")
    # the full-size inventories, built on the meta device (no memory)
    inventories = {}
    for name, cfg in (("baseline_step", ocfg.baseline_step_config()),
                      ("released_preset", ocfg.OracleConfig(text_adapter="linear")),
                      ("released_preset_lap", ocfg.OracleConfig(text_adapter="lap_blocks2"))):
        with torch.device("meta"):
            model = IrisDiT(_reference_config(cfg, ModelConfig, PixelStageConfig))
        spec = [(n, tuple(p.shape)) for n, p in model.named_parameters()]
        assert spec == [(n, tuple(s)) for n, s, _ in param_spec(cfg)], name
        inventories[name] = {"names": [n for n, _ in spec], "numel": sum(math.prod(s) for _, s in spec)}
        print(name, "parameters:", inventories[name]["numel"])
    torch.save(inventories, HERE / "inventories.pt")


if __name__ == "__main__":
    main()
