"""Parity at the shapes the benchmark times, against the fp32 oracle on the
same GPU (TF32 off), with the benchmark's own weights and seeded inputs.

* config 4 as benched (``bench.py`` default workload): one denoiser call of
  16 rows (8 images x [uncond; cond]) and the 4-step guided Euler loop over all
  8 images (src/iris3b/sampling.py:98-138, src/iris3b/flow/solver.py:58-74);
* config 5 on one GPU: one B = 2 call at 2048^2 (16384 + 256 tokens);
* config 2 through the reference-named kernel API: ``qk_norm_rope`` on Q and K
  [2, 4352, 3072] with the 64 x 64 + 256 rotary table and ``rms_norm_modulate``
  on [2, 4096, 3072] BF16 (src/iris_metal/kernels.py:314-331,413-452).

Tolerances (BASELINE): per-op max relative error max|a-b| / max|b| <= 2e-2
in BF16; pre-clamp sample PSNR >= 40 dB per image.
"""

import math

import pytest
import torch

import bench
from conftest import requires_gpu
from oracle import ops
from oracle.config import baseline_step_config as oracle_config
from oracle.model import OracleModel
from oracle.sampler import euler_cfg as oracle_euler

pytestmark = requires_gpu

REL_TOL = 2e-2
PSNR_MIN = 40.0


def rel_err(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max())


def psnr(a, ref):
    a, ref = a.double(), ref.double()
    mse = float(((a - ref) ** 2).mean())
    return 10 * math.log10(float(ref.max() - ref.min()) ** 2 / mse) if mse > 0 else math.inf


@pytest.fixture(scope="module")
def bench_model():
    """The benchmark's model: BASELINE config 3 with ``synthetic_state`` seed 0
    (BF16 matrices); the oracle runs the same values in FP32."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import iris_b200

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    cfg = iris_b200.baseline_step_config()
    state = iris_b200.synthetic_state(cfg, torch.device("cuda"), seed=0)
    engine = iris_b200.CudaIris(iris_b200.IrisWeights(cfg, state))
    oracle = OracleModel(oracle_config(), {k: v.float() for k, v in state.items()})
    yield iris_b200, engine, oracle
    del engine, oracle, state
    torch.cuda.empty_cache()


def _bench_text(engine, oracle):
    noise, cond_states, uncond_states = bench.make_inputs()
    with torch.no_grad():
        text = {
            "engine": (engine.encode_text(cond_states.cuda()), engine.encode_text(uncond_states.cuda())),
            "oracle": (oracle.embed_text(cond_states.cuda()), oracle.embed_text(uncond_states.cuda())),
        }
    return noise.cuda(), text


def test_config4_sixteen_row_call_matches_oracle(bench_model):
    """The first denoiser call of a benchmark step: x = [noise; noise] of all 8
    images, t = 1000 (sigma 1), text = [uncond x 8; cond]."""
    iris, engine, oracle = bench_model
    noise, text = _bench_text(engine, oracle)
    images = noise.shape[0]
    x = torch.cat([noise, noise])
    t = torch.full((2 * images,), 1000.0, device="cuda")
    cond, uncond = text["oracle"]
    with torch.no_grad():
        expected = oracle(x, t, torch.cat([uncond.expand(images, -1, -1), cond]))
    v = engine(x, t, torch.cat([uncond.expand(images, -1, -1), cond]).contiguous())
    err = rel_err(v, expected)
    rows = [rel_err(v[i], expected[i]) for i in range(2 * images)]
    print(f"16-row call: max rel err {err:.3e} (worst row {max(rows):.3e}), psnr {psnr(v, expected):.1f} dB")
    assert err < REL_TOL
    assert max(rows) < REL_TOL


def test_config4_loop_over_eight_images_matches_oracle(bench_model):
    """The whole benchmark step: the 4-step guided Euler loop (CFG 3) over the 8
    images, each path with its own text adapter, pre-clamp PSNR per image."""
    iris, engine, oracle = bench_model
    noise, text = _bench_text(engine, oracle)
    cond, uncond = text["engine"]
    sample = iris.euler_cfg(engine, noise, cond, uncond, cfg_scale=bench.CFG_SCALE, sigmas=bench.SIGMAS)
    ocond, ouncond = text["oracle"]
    with torch.no_grad():
        expected = oracle_euler(oracle, noise, ocond, ouncond, bench.CFG_SCALE, bench.SIGMAS)
    values = [psnr(sample[i], expected[i]) for i in range(noise.shape[0])]
    print("per-image pre-clamp psnr (dB):", ", ".join(f"{v:.1f}" for v in values))
    assert min(values) >= PSNR_MIN


def test_config5_2048_call_matches_oracle(bench_model):
    """One B = 2 CFG call at 2048^2 on one GPU (bench.py --workload step2048 at
    N = 1): 16640 joint tokens, 16384 pixel-stage patch tokens."""
    iris, engine, oracle = bench_model
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1, 3, 2048, 2048, generator=gen).repeat(2, 1, 1, 1).cuda()
    states = torch.randn(2, bench.TEXT_LEN, bench.TEXT_DIM, generator=torch.Generator().manual_seed(4)).cuda()
    t = torch.full((2,), 625.0, device="cuda")
    with torch.no_grad():
        text = oracle.embed_text(states)
        expected = oracle(x, t, text)
    v = engine(x, t, text)
    err, value = rel_err(v, expected), psnr(v, expected)
    print(f"2048^2 call: max rel err {err:.3e}, psnr {value:.1f} dB")
    assert err < REL_TOL
    assert value > PSNR_MIN


def test_config2_fused_ops_match_oracle():
    """The two config-2 microbenchmark calls of ``bench.py --workload ops`` with
    the same seeds, checked against the kernel references."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from iris_b200 import kernels as K
    from iris_b200.tables import cos_sin, rope_1d, rope_2d

    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 4096, 3072, generator=g).to("cuda", torch.bfloat16)
    w = (1 + 0.02 * torch.randn(3072, generator=g)).cuda()
    shift, scale = (0.1 * torch.randn(2, 1, 3072, generator=g)).cuda(), (0.1 * torch.randn(2, 1, 3072, generator=g)).cuda()
    out = K.rms_norm_modulate(x, w, shift, scale, 1e-6, torch.bfloat16)
    want = ops.rms_norm_modulate_reference(x, w, shift, scale, 1e-6, torch.bfloat16)
    print(f"rms_norm_modulate [2,4096,3072]: max rel err {rel_err(out, want):.3e}")
    assert rel_err(out, want) < REL_TOL
    torch.testing.assert_close(out.float(), want.float(), rtol=8e-3, atol=1e-5)

    g3 = torch.Generator().manual_seed(3)
    q, k = (torch.randn(2, 4352, 3072, generator=g3).to("cuda", torch.bfloat16) for _ in range(2))
    qw, kw = (1 + 0.02 * torch.randn(128, generator=g3)).cuda(), (1 + 0.02 * torch.randn(128, generator=g3)).cuda()
    cos, sin = cos_sin(rope_1d(128, 256, 1e4), rope_2d(128, 64, 64, 1e4, 16.0, "isotropic"), device="cuda")
    for name, proj, gain in (("q", q, qw), ("k", k, kw)):
        got = K.qk_norm_rope(proj, gain, cos, sin, 1e-6, 24)
        want = ops.qk_norm_rope_reference(proj, gain, cos, sin, 1e-6)
        print(f"qk_norm_rope {name} [2,4352,24,128]: max rel err {rel_err(got, want):.3e}")
        assert got.shape == (2, 24, 4352, 128)
        assert rel_err(got, want) < REL_TOL
        torch.testing.assert_close(got.float(), want.float(), rtol=8e-3, atol=1e-5)
