"""Whole-forward parity of CudaIris on the B200 against the reference.

* toy released topology (MHA and GQA): the reference's own fp32 outputs stored
  in tests/golden (tests/test_metal_engine.py:73-91 is the reference's version);
* the 4-step guided Euler sample: PSNR >= 40 dB against the reference's sample;
* the BASELINE config-3 model at 1024^2: against the fp32 oracle run on the
  same GPU with TF32 off (per-op metric max|a-b|/max|b| and PSNR).
"""

import math

import pytest
import torch

from conftest import golden, requires_gpu
from oracle.config import OracleConfig, PixelConfig, baseline_step_config
from oracle.model import OracleModel
from oracle.params import seeded_init
from oracle.sampler import euler_cfg as oracle_euler

pytestmark = requires_gpu

REL_TOL = 2e-2  # per-op max relative error in BF16 (max|a-b| / max|b|)
PSNR_MIN = 40.0


def _config(d):
    d = dict(d)
    return OracleConfig(**{**d, "pixel": PixelConfig(**d["pixel"])})


def rel_err(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max())


def psnr(a, ref, peak_to_peak=None):
    a, ref = a.double().cpu(), ref.double().cpu()
    mse = float(((a - ref) ** 2).mean())
    ptp = float(ref.max() - ref.min()) if peak_to_peak is None else peak_to_peak
    return 10 * math.log10(ptp**2 / mse) if mse > 0 else math.inf


@pytest.fixture(scope="module")
def iris():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import iris_b200

    return iris_b200


def _engine(iris, cfg, params):
    state = {k: v.cuda() for k, v in params.items()}
    return iris.CudaIris(iris.IrisWeights(cfg, state))


@pytest.mark.parametrize("name", ["released_mha", "released_gqa"])
def test_forward_matches_reference(iris, name):
    fx = golden(name)
    cfg = _config(fx["config"])
    engine = _engine(iris, cfg, seeded_init(cfg, seed=0))
    text = fx["prepared_text"].cuda()
    text_before = text.clone()
    v = engine(fx["x"].cuda(), fx["t"].cuda(), text)
    assert torch.equal(text, text_before), "the engine must not write its text input"
    err = rel_err(v, fx["v"])
    print(f"{name}: max rel err {err:.3e}, psnr {psnr(v, fx['v']):.1f} dB")
    assert err < REL_TOL
    assert psnr(v, fx["v"]) > PSNR_MIN


def test_graph_mode_matches_eager(iris):
    """CudaIris(graphs=True) replays one captured CUDA graph per input geometry:
    bit-identical velocities to the eager engine across alternating geometries
    (batch 2, batch 1, a non-square grid), a fresh output tensor per call, the
    text input never written, and the library's launch count advancing by the
    graph's kernels on each replay."""
    from iris_b200 import _lib

    fx = golden("released_mha")
    cfg = _config(fx["config"])
    weights = iris.IrisWeights(cfg, {k: v.cuda() for k, v in seeded_init(cfg, seed=0).items()})
    eager, graphed = iris.CudaIris(weights), iris.CudaIris(weights, graphs=True)
    x, t, text = fx["x"].cuda(), fx["t"].cuda(), fx["prepared_text"].cuda()
    cases = [(x, t, text), (x[:1], t[:1], text[:1]), (x[..., :16], t, text), (x, t, text), (x[:1], t[:1], text[:1])]
    outs = []
    for xi, ti, yi in cases:
        before = yi.clone()
        got = graphed(xi, ti, yi)
        assert torch.equal(yi, before), "the engine must not write its text input"
        assert torch.equal(got, eager(xi, ti, yi))
        outs.append(got)
    assert outs[0].data_ptr() != outs[3].data_ptr(), "every call returns a fresh tensor"
    assert torch.equal(outs[0], outs[3])
    n0 = _lib.launch_count()
    graphed(x, t, text)
    assert _lib.launch_count() - n0 == graphed._graphs[(tuple(x.shape), tuple(text.shape))]["kernels"] > 20
    # GEMM timing through a capture: the graph's event nodes time every GEMM of the
    # latest replay, and replays after timing stops still run
    from iris_b200 import kernels as K

    timed = iris.CudaIris(weights, graphs=True)
    K.profile_gemms(True)
    timed(x, t, text)
    timed(x, t, text)
    flops, ms, launches, _ = K.profile_gemms(False)
    assert launches > 0 and flops > 0 and ms > 0
    assert torch.equal(timed(x, t, text), outs[0])
    sample_g = iris.euler_cfg(graphed, fx["euler_cfg"]["noise"].cuda(), fx["euler_cfg"]["cond"].cuda(),
                              fx["euler_cfg"]["uncond"].cuda())  # fmt: skip
    sample_e = iris.euler_cfg(eager, fx["euler_cfg"]["noise"].cuda(), fx["euler_cfg"]["cond"].cuda(),
                              fx["euler_cfg"]["uncond"].cuda())  # fmt: skip
    assert torch.equal(sample_g, sample_e)


def test_checkpoint_directory_forward_matches_reference(iris, tmp_path):
    """config.yaml + model.safetensors loaded by IrisWeights.from_checkpoint
    (the directory layout of load_config / load_dit) give the reference output."""
    from test_host import _write_checkpoint

    fx = golden("released_mha")
    _write_checkpoint(tmp_path, fx)
    engine = iris.CudaIris(iris.IrisWeights.from_checkpoint(tmp_path, device="cuda"))
    v = engine(fx["x"].cuda(), fx["t"].cuda(), fx["prepared_text"].cuda())
    assert rel_err(v, fx["v"]) < REL_TOL


def test_encode_text_matches_reference(iris):
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    engine = _engine(iris, cfg, seeded_init(cfg, seed=0))
    text = engine.encode_text(fx["y"].cuda())
    assert rel_err(text, fx["prepared_text"]) < REL_TOL


def test_euler_cfg_sample_matches_reference(iris):
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    engine = _engine(iris, cfg, seeded_init(cfg, seed=0))
    s = fx["euler_cfg"]
    sample = iris.euler_cfg(engine, s["noise"].cuda(), s["cond"].cuda(), s["uncond"].cuda(), cfg_scale=s["cfg_scale"],
                            cfg_interval=s["cfg_interval"])  # fmt: skip
    value = psnr(sample, s["sample"])
    print(f"euler cfg sample: psnr {value:.1f} dB (ptp-2: {psnr(sample, s['sample'], 2.0):.1f} dB)")
    assert value >= PSNR_MIN


def test_dpm_solver_sample_matches_reference(iris):
    """The Original model's loop: iris_b200.FlowDPMSolver (fused CFG + DPM-Solver++
    step per kernel) driving the engine, against the reference's FlowDPMSolver
    driving IrisDiT (src/iris3b/flow/solver.py:112-141; 10 steps, 2nd order,
    shift 3, CFG 3 inside the default interval)."""
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    engine = _engine(iris, cfg, seeded_init(cfg, seed=0))
    d = fx["dpm"]
    solver = iris.FlowDPMSolver(engine, cfg_scale=d["cfg_scale"], cfg_interval=d["cfg_interval"])
    sample = solver.sample(d["noise"].cuda(), d["cond"].cuda(), d["uncond"].cuda(), steps=d["steps"], order=d["order"],
                           shift=d["shift"])  # fmt: skip
    value = psnr(sample, d["sample"])
    print(f"dpm-solver++ 10-step sample: psnr {value:.1f} dB, max rel err {rel_err(sample, d['sample']):.2e}")
    assert value > PSNR_MIN
    assert rel_err(sample, d["sample"]) < REL_TOL


def test_pipeline_runs_the_original_dpm_loop(iris):
    """DenoisePipeline with ``steps``: host noise and adapted text in, the
    DPM-Solver++ loop on the device, the clamped sample out into host memory."""
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    engine = _engine(iris, cfg, seeded_init(cfg, seed=0))
    d = fx["dpm"]
    pipe = iris.DenoisePipeline(engine, cfg_scale=d["cfg_scale"], cfg_interval=d["cfg_interval"], steps=d["steps"],
                                order=d["order"], shift=d["shift"])  # fmt: skip
    out = torch.empty_like(d["noise"]).pin_memory()
    got = pipe(d["noise"], d["cond"], d["uncond"], adapted=True, out=out)
    torch.cuda.synchronize()
    assert got is out
    assert psnr(out, d["sample"].clamp(-1, 1)) > PSNR_MIN


@pytest.mark.parametrize("steps", [None, 10])
def test_pipeline_expands_one_unconditional_row(iris, steps):
    """Two images with one shared unconditional row (and one with a one-row
    prompt) through both loops, as the reference pipeline expands them
    (src/iris_metal/pipeline.py:297-298): image 0 reproduces the reference's
    sample; image 1 matches a one-image call on its own noise. The caller's
    noise is left untouched."""
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    engine = _engine(iris, cfg, seeded_init(cfg, seed=0))
    d = fx["dpm"] if steps else fx["euler_cfg"]
    kw = {"steps": d["steps"], "order": d["order"], "shift": d["shift"]} if steps else {}
    pipe = iris.DenoisePipeline(engine, cfg_scale=d["cfg_scale"], cfg_interval=d["cfg_interval"], **kw)
    other = torch.randn(d["noise"].shape, generator=torch.Generator().manual_seed(11))
    noise = torch.cat([d["noise"], other]).cuda()
    before = noise.clone()
    both = pipe(noise, d["cond"], d["uncond"], adapted=True)
    assert torch.equal(noise, before), "the pipeline must not write the caller's noise"
    alone = pipe(other.cuda(), d["cond"], d["uncond"], adapted=True)
    assert psnr(both[:1], d["sample"].clamp(-1, 1)) > PSNR_MIN
    assert psnr(both[1:], alone) > PSNR_MIN
    with pytest.raises(ValueError, match="rows for 2 images"):
        pipe(noise, torch.cat([d["cond"]] * 3), d["uncond"], adapted=True)


def test_turbo_four_step_sample_without_cfg(iris):
    """The Turbo loop (generate_few_step, src/iris3b/sampling.py:98-138: four
    deterministic Euler steps at TURBO_SIGMAS, no CFG) on the engine against
    the fp32 oracle model run through the oracle's loop on the CPU."""
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    params = seeded_init(cfg, seed=0)
    engine = _engine(iris, cfg, params)
    s = fx["euler_cfg"]
    noise, cond = s["noise"], s["cond"]
    sample = iris.euler_cfg(engine, noise.cuda(), cond.cuda(), None)
    oracle = OracleModel(cfg, params)
    with torch.no_grad():
        want = oracle_euler(lambda x, t, y: oracle.forward(x, t, y), noise, cond, None)
    value = psnr(sample, want)
    print(f"turbo (no CFG) 4-step sample: psnr {value:.1f} dB")
    assert value > PSNR_MIN


def test_turbo_recipe_matches_reference_autocast(iris):
    """Turbo (src/iris_metal/pipeline.py:372-428): BF16-stored Linear weights,
    the upstream forward under BF16 autocast. The engine keeps FP32 residuals and
    accumulators instead of autocast's BF16 activations, so it is re-validated
    rather than bit-matched: at every step's input its velocity must be within
    the per-op tolerance of the reference's autocast velocity and at most a
    quarter as far from the FP32 forward on the same weights as autocast itself
    is (on B200: 3.1e-4 to 3.5e-4 against autocast's 5.6e-3 to 6.3e-3); the
    4-step sample above PSNR_MIN against the autocast sample (88.5 dB)."""
    from test_oracle import turbo_params

    fx = golden("released_mha")
    cfg = _config(fx["config"])
    tb = fx["turbo"]
    engine = _engine(iris, cfg, turbo_params(cfg, set(tb["linear"])))
    cond = tb["cond"].cuda()
    for step in tb["steps"]:
        v = engine(step["x"].cuda(), step["t"].cuda(), cond)
        to_autocast, to_fp32 = rel_err(v, step["v_autocast"]), rel_err(v, step["v_fp32"])
        autocast_to_fp32 = rel_err(step["v_autocast"], step["v_fp32"])
        print(f"t={float(step['t'][0]):.0f}: engine-autocast {to_autocast:.2e}, engine-fp32 {to_fp32:.2e}, "
              f"autocast-fp32 {autocast_to_fp32:.2e}")  # fmt: skip
        assert to_autocast < REL_TOL
        assert to_fp32 < 0.25 * autocast_to_fp32
    sample = iris.euler_cfg(engine, tb["noise"].cuda(), cond, None)
    value = psnr(sample, tb["autocast"])
    print(f"turbo sample: psnr {value:.1f} dB against autocast")
    assert value > PSNR_MIN


def test_depth_task_four_channel_input_matches_reference(iris):
    """A depth fine-tune's widened denoiser (src/iris3b/downstream/depth.py:30-38),
    which the reference engine accepts (src/iris_metal/model.py:181-217): 4 input
    channels, 3 output. The engine built on it as MetalDepth builds its engine
    (src/iris_metal/tasks.py:79-97) against IrisDepth's own outputs: a 4-channel
    input whose extra channel is not zero, and the depth prediction (RGB plus a
    zero channel at t = 1000, then the 1x1 reducer)."""
    from oracle.params import depth_task_params
    from test_oracle import depth_engine_inputs

    fx = golden("released_mha")
    cfg = _config(fx["config"])
    d = fx["depth"]
    params = depth_task_params(cfg)
    reducer = [params.pop(k).cuda() for k in ("depth_reducer.weight", "depth_reducer.bias")]
    engine = _engine(iris, cfg, params)
    assert engine.in_channels == 4
    # the text as tasks.py passes it: one prompt expanded over the batch (a stride-0 view)
    v4 = engine(d["x4"].cuda(), d["t4"].cuda(), d["prepared_text"].cuda().expand(2, -1, -1))
    print(f"depth model, 4-channel input: max rel err {rel_err(v4, d['v4']):.3e}, psnr {psnr(v4, d['v4']):.1f} dB")
    assert v4.shape == d["v4"].shape
    assert rel_err(v4, d["v4"]) < REL_TOL
    assert psnr(v4, d["v4"]) > PSNR_MIN
    x, t, text = depth_engine_inputs(fx)
    depth = torch.nn.functional.conv2d(engine(x.cuda(), t.cuda(), text.cuda()), *reducer)
    assert rel_err(depth, d["depth"]) < REL_TOL
    with pytest.raises(ValueError, match="input channels"):
        engine(d["rgb"].cuda(), t.cuda(), text.cuda())


def test_non_square_grid_and_odd_batch(iris):
    fx = golden("released_gqa")  # 24 x 16 input: a 6 x 4 patch grid
    cfg = _config(fx["config"])
    params = seeded_init(cfg, seed=0)
    engine = _engine(iris, cfg, params)
    oracle = OracleModel(cfg, params)
    x, t, text = fx["x"][:1], fx["t"][:1], fx["prepared_text"][:1]
    with torch.no_grad():
        expected = oracle(x, t, text)
    v = engine(x.cuda(), t.cuda(), text.cuda())
    assert rel_err(v, expected) < REL_TOL


@pytest.fixture(scope="module")
def full_size(iris):
    """BASELINE config 3 (d = 3072, 24 blocks, 24 MHA heads x 128) with seeded
    random weights drawn on the GPU, shared by the oracle (fp32) and the engine."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    cfg = baseline_step_config()
    params = seeded_init(cfg, seed=0, device="cuda")
    engine = iris.CudaIris(iris.IrisWeights(cfg, params))
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1, 3, 1024, 1024, generator=gen).repeat(2, 1, 1, 1)
    y = torch.randn(2, 256, cfg.text_dim, generator=gen)
    oracle = OracleModel(cfg, params)
    with torch.no_grad():
        text = oracle.embed_text(y.cuda())
    return cfg, params, engine, oracle, x.cuda(), text


def test_full_size_step_matches_fp32_oracle(full_size):
    cfg, params, engine, oracle, x, text = full_size
    t = torch.full((2,), 625.0, device="cuda")
    with torch.no_grad():
        expected = oracle(x, t, text)
    v = engine(x, t, text)
    err, value = rel_err(v, expected), psnr(v, expected)
    print(f"1024^2 step: max rel err {err:.3e}, psnr {value:.1f} dB")
    assert err < REL_TOL
    assert value > PSNR_MIN


def test_full_size_euler_cfg_psnr(full_size, iris):
    cfg, params, engine, oracle, x, text = full_size
    noise = torch.randn(1, 3, 1024, 1024, generator=torch.Generator().manual_seed(0)).cuda()
    cond, uncond = text[1:], text[:1]
    with torch.no_grad():
        expected = oracle_euler(oracle, noise, cond, uncond, 3.0)
    sample = iris.euler_cfg(engine, noise, cond, uncond, cfg_scale=3.0)
    value = psnr(sample, expected)
    print(f"1024^2 4-step Euler CFG 3: psnr {value:.1f} dB (ptp-2: {psnr(sample, expected, 2.0):.1f} dB)")
    assert value >= PSNR_MIN
