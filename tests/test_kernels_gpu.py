"""Kernel parity on the B200: each entry point of libiris_b200.so against the
reference's own outputs (tests/golden/ops.pt) or the fp32 oracle, mirroring
tests/test_metal_engine.py:159-289 of the reference."""

import pytest
import torch
import torch.nn.functional as F

from conftest import golden, requires_gpu
from oracle import ops

pytestmark = requires_gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from iris_b200 import kernels

    return kernels


def rel_err(a, b):
    """max |a - b| / max |b| (the per-op tolerance metric)."""
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("out_dtype", DTYPES)
def test_qk_norm_rope_matches_reference(K, dtype, out_dtype):
    fx = golden("ops")["qk_norm_rope"]
    x = fx["x"].to("cuda", dtype)
    out = torch.zeros(2, fx["heads"], 42, 128, device="cuda", dtype=out_dtype)
    K.qk_norm_rope(x, fx["weight"].cuda(), fx["cos"].cuda(), fx["sin"].cuda(), 1e-6, fx["heads"],
                   col_offset=fx["col_offset"], out=out, offset=fx["offset"])  # fmt: skip
    expected = ops.qk_norm_rope_reference(x[..., fx["col_offset"] :].float().cpu(), fx["weight"], fx["cos"][5:],
                                          fx["sin"][5:], 1e-6)  # fmt: skip
    tol = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 8e-3}[out_dtype]
    torch.testing.assert_close(out[:, :, 5:].float().cpu(), expected, rtol=tol, atol=1e-5)
    assert torch.all(out[:, :, :5] == 0)
    if dtype == torch.float32 and out_dtype == torch.float32:
        torch.testing.assert_close(out.cpu(), fx["out"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("branch_dtype", [torch.float32, torch.bfloat16])
def test_row_kernels_match_reference(K, branch_dtype):
    fx = golden("ops")
    r = fx["rms_norm_modulate"]
    args = [t.cuda() for t in (r["x"], r["weight"], r["shift"], r["scale"])]
    out = K.rms_norm_modulate(*args, 1e-6, torch.bfloat16)
    torch.testing.assert_close(out.float().cpu(), r["out_bf16"].float(), rtol=8e-3, atol=1e-5)
    out = K.rms_norm_modulate(*args, 1e-6, torch.float32)
    torch.testing.assert_close(out.cpu(), r["out_f32"], rtol=1e-5, atol=1e-5)
    g = fx["gated_residual"]
    branch = g["branch"].to(branch_dtype)
    expected = ops.gated_residual_rms_norm_reference(g["residual"], branch, g["weight"], g["gate"], 1e-6)
    actual = K.gated_residual_rms_norm_(g["residual"].cuda(), branch.cuda(), g["weight"].cuda(), g["gate"].cuda(), 1e-6)
    torch.testing.assert_close(actual.cpu(), expected, rtol=1e-5, atol=1e-5)
    if branch_dtype == torch.float32:
        torch.testing.assert_close(actual.cpu(), g["out"], rtol=1e-5, atol=1e-5)


def _modulation_layouts(batch, width, gen):
    mods = torch.randn(batch, 1, 6 * width, generator=gen).cuda()
    chunks = list(mods.chunk(6, dim=-1)[:3])
    one = torch.randn(1, 1, 3 * width, generator=gen).cuda()
    padded = torch.randn(batch * 3 * width + 1, generator=gen).cuda()
    misaligned = [padded[1 + i * batch * width :][: batch * width].view(batch, 1, width) for i in range(3)]
    return {
        "contiguous": [c.contiguous() for c in chunks],
        "chunks": chunks,
        "expanded": [c.expand(batch, 1, width) for c in one.chunk(3, dim=-1)],
        "misaligned": misaligned,
    }


@pytest.mark.parametrize("batch", [1, 2, 3])
def test_row_kernels_read_strided_modulation_exactly(K, batch):
    """tests/test_metal_engine.py:226-246: every modulation layout gives bit-identical rows."""
    gen = torch.Generator().manual_seed(batch)
    width = 384
    x = torch.randn(batch, 5, width, generator=gen).cuda()
    branch = torch.randn(batch, 5, width, generator=gen).to("cuda", torch.bfloat16)
    weight = (torch.rand(width, generator=gen) + 0.5).cuda()
    for name, (shift, scale, gate) in _modulation_layouts(batch, width, gen).items():
        dense = [t.contiguous() for t in (shift, scale, gate)]
        expected = K.rms_norm_modulate(x, weight, dense[0], dense[1], 1e-6, torch.float16)
        actual = K.rms_norm_modulate(x, weight, shift, scale, 1e-6, torch.float16)
        assert actual.view(torch.int16).equal(expected.view(torch.int16)), name
        expected = K.gated_residual_rms_norm_(x.clone(), branch, weight, dense[2], 1e-6)
        actual = K.gated_residual_rms_norm_(x.clone(), branch, weight, gate, 1e-6)
        assert actual.view(torch.int32).equal(expected.view(torch.int32)), name
        rows, _ = K._per_batch(gate, batch, width)
        in_place = rows.untyped_storage().data_ptr() == gate.untyped_storage().data_ptr()
        assert in_place == (name != "misaligned"), name


def test_kernels_reject_non_fp32_gains(K):
    x = torch.randn(1, 4, 128, device="cuda")
    gain = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    zeros = torch.zeros(1, 1, 128, device="cuda")
    with pytest.raises(ValueError, match="FP32"):
        K.rms_norm_modulate(x, gain, zeros, zeros, 1e-6, torch.bfloat16)


@pytest.mark.parametrize("pixel_dtype", [torch.bfloat16, torch.float32])
def test_pixel_kernels_match_reference(K, pixel_dtype):
    m = golden("ops")["pixel_mlp"]

    class Lin:
        def __init__(self, w, b):
            self.weight, self.bias = w.cuda(), b.cuda()

    pixels = m["pixels"].to("cuda", pixel_dtype)
    nxt = K.pixel_mlp_(pixels, m["branch"].cuda(), m["mods"].cuda(), m["norm_weight"].cuda(),
                       Lin(m["fc1_w"], m["fc1_b"]), Lin(m["fc2_w"], m["fc2_b"]), m["next_norm_weight"].cuda(), 1e-6)  # fmt: skip
    # one BF16 ulp where rounding order differs (tests/test_metal_engine.py:281-289)
    tol = 1e-2 if pixel_dtype == torch.bfloat16 else 2e-2
    torch.testing.assert_close(pixels.float().cpu(), m["new_pixels"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(nxt.float().cpu(), m["next_input"].float(), rtol=tol, atol=tol)
    rms = K.pixel_rms_norm(m["pixels"].cuda(), m["norm_weight"].cuda(), 1e-6)
    torch.testing.assert_close(rms.float().cpu(), m["rms"].float(), rtol=1e-2, atol=1e-2)


def test_pixel_mlp_gelu_matches_cuda_erf(K):
    """The pixel tail's GELU takes erf from Abramowitz & Stegun 7.1.26 (error
    <= 1.5e-7) instead of CUDA's erff. Against the same tail in torch on the GPU
    (its exact GELU is erff's), with the kernel's roundings (bf16 MMA inputs,
    fp32 sums): almost every output agrees to fp32 summation order, and the rest
    differ by a bf16 rounding of a GELU value at a tie (2.1 M pixels)."""
    gen = torch.Generator(device="cuda").manual_seed(29)
    n = 2 * 4096 * 256
    pixels = torch.randn(n, 16, device="cuda", generator=gen)
    branch = torch.randn(n, 16, device="cuda", generator=gen).to(torch.bfloat16)
    mods = (0.3 * torch.randn(n, 64, device="cuda", generator=gen)).to(torch.bfloat16)
    gain = torch.rand(16, device="cuda", generator=gen) + 0.5
    gain_next = torch.rand(16, device="cuda", generator=gen) + 0.5

    class Lin:
        def __init__(self, o, i):
            self.weight = (0.3 * torch.randn(o, i, device="cuda", generator=gen)).to(torch.bfloat16)
            self.bias = (0.1 * torch.randn(o, device="cuda", generator=gen)).to(torch.bfloat16)

    fc1, fc2 = Lin(64, 16), Lin(16, 64)
    eps = 1e-6
    # the tail in torch, rounding where the kernel does
    bf = lambda t: t.to(torch.bfloat16).float()  # noqa: E731
    s1, t1, s2, t2 = mods.float().view(n, 4, 16).unbind(1)
    x = pixels + (branch.float() * (1 + s1) + t1)
    h = bf(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * gain)
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        a = h @ fc1.weight.float().T + fc1.bias.float()
        g = bf(F.gelu(a))
        out = g @ fc2.weight.float().T + fc2.bias.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    want = x + (out * (1 + s2) + t2)
    got = pixels.clone()
    K.pixel_mlp_(got, branch, mods, gain, fc1, fc2, gain_next, eps)
    diff = (got - want).abs()
    close = diff <= 1e-4 * want.abs().clamp_min(1.0)
    print(f"pixel GELU vs erff: {int((~close).sum())} of {diff.numel()} beyond fp32 order, max diff {diff.max():.3e}")
    assert close.float().mean() > 0.999
    # a flipped bf16 rounding of one GELU value moves an output by at most 2^-8 |g| |w2| (1 + |s2|)
    bound = 2.0**-8 * g.abs().amax() * fc2.weight.float().abs().amax() * (1 + s2.abs().amax()) * 4
    assert float(diff.max()) <= float(bound)


def test_pixel_kernels_reject_short_parameter_buffers(K):
    pixels = torch.zeros(1, 1, 16, device="cuda", dtype=torch.bfloat16)
    gain = torch.ones(16, device="cuda")
    with pytest.raises(ValueError, match="gain width"):
        K.pixel_rms_norm(pixels, gain[:1], 1e-6)
    mods = torch.zeros(1, 1, 64, device="cuda", dtype=torch.bfloat16)
    fc1 = torch.nn.Linear(16, 64, device="cuda", dtype=torch.bfloat16)
    fc2 = torch.nn.Linear(64, 16, device="cuda", dtype=torch.bfloat16)
    fc1.bias = torch.nn.Parameter(fc1.bias[:1])
    with pytest.raises(ValueError, match="pixel-stage widths"):
        K.pixel_mlp_(pixels, pixels.clone(), mods, gain, fc1, fc2, gain, 1e-6)


# ------------------------------------------------------------------------- GEMM
# M >= 256 runs the CTA-pair kernel (256-row tiles); (4096, 2560, 512) gives
# every SM pair several tiles, so both TMEM accumulators and the ring wrap.
GEMM_SHAPES = [
    (128, 256, 64),
    (200, 96, 48),
    (1000, 544, 312),
    (8704 // 8, 9216 // 8, 3072 // 4),
    (64, 1280, 1280),
    (4096, 2560, 512),
]


@pytest.mark.parametrize("M,N,K_", GEMM_SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_matches_fp32_reference(K, M, N, K_, out_dtype):
    gen = torch.Generator(device="cuda").manual_seed(M + N + K_)
    a = torch.randn(M, K_, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(N, K_, device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=gen)
    out = torch.empty(M, N, device="cuda", dtype=out_dtype)
    K.gemm(a, w, out, bias=bias)
    expected = a.float() @ w.float().T + bias
    assert rel_err(out, expected) < (1e-2 if out_dtype == torch.bfloat16 else 1e-4)


def test_gemm_row_map_writes_only_mapped_rows(K):
    """Image rows into a joint [text | image] buffer: rows (b, T + i)."""
    T, L, B, N, D = 7, 45, 2, 52, 256
    gen = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(B * L, 64, device="cuda", generator=gen).to(torch.bfloat16)
    w = torch.randn(D, 64, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.full((B * N, D), -7.0, device="cuda")
    K.gemm(a, w, out, out_rows=(L, N, T))
    expected = (a.float() @ w.float().T).view(B, L, D)
    got = out.view(B, N, D)
    assert rel_err(got[:, T:], expected) < 1e-4
    assert torch.all(got[:, :T] == -7.0)


def test_gemm_swiglu_epilogue(K):
    from iris_b200._lib import EPI_SWIGLU
    from iris_b200.model import pack_swiglu

    M, D, F_ = 300, 256, 682
    gen = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(M, D, device="cuda", generator=gen).to(torch.bfloat16)
    w1, w3 = ((torch.randn(F_, D, device="cuda", generator=gen) * 0.05).to(torch.bfloat16) for _ in range(2))
    w2 = (torch.randn(D, F_, device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    w13, w2p = pack_swiglu(w1, w3, w2)
    act = torch.empty(M, w2p.shape[1], device="cuda", dtype=torch.bfloat16)
    K.gemm(a, w13, act, epilogue=EPI_SWIGLU)
    out = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    K.gemm(act, w2p, out)
    h = F.silu(a.float() @ w1.float().T) * (a.float() @ w3.float().T)
    assert rel_err(act[:, :F_], h) < 1e-2
    assert torch.all(act[:, F_:] == 0)
    assert rel_err(out, h @ w2.float().T) < 2e-2


def test_gemm_gate_epilogue_with_aux_rows(K):
    from iris_b200._lib import EPI_GATE

    T, L, B, D = 16, 36, 2, 256
    N = T + L
    gen = torch.Generator(device="cuda").manual_seed(9)
    h = torch.randn(B * L, D, device="cuda", generator=gen).to(torch.bfloat16)
    wg = (torch.randn(D, D, device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    attn = torch.randn(B * N, D, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.empty(B * L, D, device="cuda", dtype=torch.bfloat16)
    K.gemm(h, wg, out, epilogue=EPI_GATE, aux=attn, aux_rows=(L, N, T))
    expected = attn.view(B, N, D)[:, T:].reshape(B * L, D).float() * torch.sigmoid(h.float() @ wg.float().T)
    assert rel_err(out, expected) < 1e-2


def test_gemm_grouped_runs_independent_problems(K):
    """Text and image problems of a dual block in one launch, each with its own
    weights, bias and epilogue, match separate reference products."""
    from iris_b200._lib import EPI_SWIGLU
    from iris_b200.model import pack_swiglu

    gen = torch.Generator(device="cuda").manual_seed(21)
    shapes = [(1000, 768, 256), (72, 512, 256), (300, 256, 384)]
    a = [torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16) for m, _, k in shapes]
    w = [(torch.randn(n, k, device="cuda", generator=gen) * 0.05).to(torch.bfloat16) for _, n, k in shapes]
    bias = torch.randn(768, device="cuda", generator=gen)
    outs = [torch.empty(m, n, device="cuda", dtype=torch.bfloat16) for m, n, _ in shapes]
    w13, _ = pack_swiglu(w[2][:128], w[2][128:], torch.zeros(8, 128, device="cuda", dtype=torch.bfloat16))
    act = torch.empty(300, 128, device="cuda", dtype=torch.bfloat16)
    problems = [
        K.gemm_problem(a[0], w[0], outs[0], bias=bias),
        K.gemm_problem(a[1], w[1], outs[1]),
        K.gemm_problem(a[2], w13, act, epilogue=EPI_SWIGLU),
    ]
    K.gemm_grouped(problems, torch.cuda.current_stream().cuda_stream)
    assert rel_err(outs[0], a[0].float() @ w[0].float().T + bias) < 1e-2
    assert rel_err(outs[1], a[1].float() @ w[1].float().T) < 1e-2
    ref = F.silu(a[2].float() @ w[2][:128].float().T) * (a[2].float() @ w[2][128:].float().T)
    assert rel_err(act, ref) < 1e-2


def test_gemm_pair_kernel_epilogues_and_row_maps(K):
    """All problems with M >= 256 take the CTA-pair kernel: bias + row map, gate
    with aux rows and SwiGLU in one launch, ragged last pair tiles included."""
    from iris_b200._lib import EPI_GATE, EPI_SWIGLU
    from iris_b200.model import pack_swiglu

    gen = torch.Generator(device="cuda").manual_seed(33)
    T, L, B, D = 40, 300, 2, 512
    N = T + L
    a0 = torch.randn(B * L, 256, device="cuda", generator=gen).to(torch.bfloat16)
    w0 = (torch.randn(D, 256, device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    bias = torch.randn(D, device="cuda", generator=gen)
    joint = torch.full((B * N, D), -7.0, device="cuda")
    wg = (torch.randn(D, 256, device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    attn = torch.randn(B * N, D, device="cuda", generator=gen).to(torch.bfloat16)
    gated = torch.empty(B * L, D, device="cuda", dtype=torch.bfloat16)
    M2, F_ = 260, 384
    a2 = torch.randn(M2, 256, device="cuda", generator=gen).to(torch.bfloat16)
    w1, w3 = ((torch.randn(F_, 256, device="cuda", generator=gen) * 0.05).to(torch.bfloat16) for _ in range(2))
    w13, _ = pack_swiglu(w1, w3, torch.zeros(8, F_, device="cuda", dtype=torch.bfloat16))
    act = torch.empty(M2, w13.shape[0] // 2, device="cuda", dtype=torch.bfloat16)
    problems = [
        K.gemm_problem(a0, w0, joint, bias=bias, out_rows=(L, N, T)),
        K.gemm_problem(a0, wg, gated, epilogue=EPI_GATE, aux=attn, aux_rows=(L, N, T)),
        K.gemm_problem(a2, w13, act, epilogue=EPI_SWIGLU),
    ]
    K.gemm_grouped(problems, torch.cuda.current_stream().cuda_stream)
    got = joint.view(B, N, D)
    assert rel_err(got[:, T:], (a0.float() @ w0.float().T + bias).view(B, L, D)) < 1e-4
    assert torch.all(got[:, :T] == -7.0)
    gate_ref = attn.view(B, N, D)[:, T:].reshape(B * L, D).float() * torch.sigmoid(a0.float() @ wg.float().T)
    assert rel_err(gated, gate_ref) < 1e-2
    h = F.silu(a2.float() @ w1.float().T) * (a2.float() @ w3.float().T)
    assert rel_err(act[:, :F_], h) < 1e-2
    assert torch.all(act[:, F_:] == 0)


@pytest.mark.parametrize("M,hq,hkv,head_major", [(90, 2, 1, False), (300, 3, 1, False), (600, 4, 2, True)])
def test_gemm_heads_epilogue_matches_projection_then_qk_norm_rope(K, M, hq, hkv, head_major):
    """EPI_HEADS (one-SM and CTA-pair kernels; odd slot counts; a row map that
    puts the rows after T text positions) against the fp32 projection followed
    by the oracle's qk_norm_rope and the V copy."""
    T, B = 5, 2
    L = M // B
    tokens = T + L
    Kd = 256
    gen = torch.Generator(device="cuda").manual_seed(M + hq)
    a = torch.randn(M, Kd, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn((hq + 2 * hkv) * 128, Kd, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    qw, kw = (torch.rand(128, device="cuda", generator=gen) + 0.5 for _ in range(2))
    cos, sin = (torch.randn(tokens, 64, device="cuda", generator=gen) for _ in range(2))
    shape_q = (hq, B, tokens, 128) if head_major else (B, hq, tokens, 128)
    shape_kv = (hkv, B, tokens, 128) if head_major else (B, hkv, tokens, 128)
    q = torch.zeros(*shape_q, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.zeros(*shape_kv, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    heads = K.HeadsOut(q, k, v, qw, kw, cos, sin, 1e-6, hq, hkv, tokens, B, tokens, tokens, head_major=head_major)
    K.gemm_grouped([K.gemm_problem(a, w, None, out_rows=(L, tokens, T), heads=heads)],
                   torch.cuda.current_stream().cuda_stream)  # fmt: skip
    proj = (a.float() @ w.float().T).view(B, L, hq + 2 * hkv, 128).cpu()
    c, s_ = cos[T:].cpu(), sin[T:].cpu()
    if head_major:
        q, k, v = (t.transpose(0, 1) for t in (q, k, v))
    got_q, got_k, got_v = (t[:, :, T:].float().cpu() for t in (q, k, v))
    for h in range(hq):
        ref = ops.qk_norm_rope_reference(proj[:, :, h].reshape(B, L, 128), qw.cpu(), c, s_, 1e-6)[:, 0]
        assert rel_err(got_q[:, h], ref) < 1e-2
    for h in range(hkv):
        ref = ops.qk_norm_rope_reference(proj[:, :, hq + h].reshape(B, L, 128), kw.cpu(), c, s_, 1e-6)[:, 0]
        assert rel_err(got_k[:, h], ref) < 1e-2
        assert rel_err(got_v[:, h], proj[:, :, hq + hkv + h]) < 1e-2
    assert torch.all(q[:, :, :T] == 0) and torch.all(k[:, :, :T] == 0)


# -------------------------------------------------------------------- attention
def test_flash_attention_split_gate_writes_each_stream_densely(K):
    B, H, T, N = 2, 2, 16, 52
    L = N - T
    gen = torch.Generator(device="cuda").manual_seed(13)
    q, k, v = (torch.randn(B, H, N, 128, device="cuda", generator=gen).to(torch.bfloat16) for _ in range(3))
    gate = torch.randn(B * N, H * 128, device="cuda", generator=gen).to(torch.bfloat16)  # [text rows | image rows]
    out = torch.full((B * N, H * 128), 7.0, device="cuda", dtype=torch.bfloat16)
    K.flash_attention_split(q, k, v, T, out[: B * T], out[B * T :], gate[: B * T], gate[B * T :])
    attn = ops.sdpa(q.float(), k.float(), v.float()).transpose(1, 2)  # [B, N, H, 128]
    text = attn[:, :T].reshape(B * T, -1) * torch.sigmoid(gate[: B * T].float())
    image = attn[:, T:].reshape(B * L, -1) * torch.sigmoid(gate[B * T :].float())
    assert rel_err(out[: B * T], text) < 2e-2
    assert rel_err(out[B * T :], image) < 2e-2



@pytest.mark.parametrize("B,H,Hkv,N", [(1, 1, 1, 128), (2, 2, 1, 52), (2, 3, 3, 300), (1, 2, 2, 4352)])
def test_flash_attention_matches_fp32_sdpa(K, B, H, Hkv, N):
    gen = torch.Generator(device="cuda").manual_seed(B * 100 + N)
    q = torch.randn(B, H, N, 128, device="cuda", generator=gen).to(torch.bfloat16)
    k = torch.randn(B, Hkv, N, 128, device="cuda", generator=gen).to(torch.bfloat16)
    v = torch.randn(B, Hkv, N, 128, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.empty(B, N, H * 128, device="cuda", dtype=torch.bfloat16)
    K.flash_attention(q, k, v, out)
    expected = ops.sdpa(q.float(), k.float(), v.float()).transpose(1, 2).reshape(B, N, H * 128)
    assert rel_err(out, expected) < 2e-2
    assert K.device_error() == 0


def test_flash_attention_sharp_softmax(K):
    """Large logits exercise the lazy rescale path (row max growing by > 2^8)."""
    B, H, N = 1, 1, 640
    gen = torch.Generator(device="cuda").manual_seed(11)
    q = (torch.randn(B, H, N, 128, device="cuda", generator=gen) * 4).to(torch.bfloat16)
    k = (torch.randn(B, H, N, 128, device="cuda", generator=gen) * 4).to(torch.bfloat16)
    k[:, :, 400:] *= 3  # later key blocks carry larger scores
    v = torch.randn(B, H, N, 128, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.empty(B, N, H * 128, device="cuda", dtype=torch.bfloat16)
    K.flash_attention(q, k, v, out)
    expected = ops.sdpa(q.float(), k.float(), v.float()).transpose(1, 2).reshape(B, N, H * 128)
    assert rel_err(out, expected) < 2e-2


@pytest.mark.parametrize("gain,sharp_tail", [(1.0, False), (1.0, True), (3.0, True)])
def test_flash_attention_with_score_bound(K, gain, sharp_tail):
    """QK-normed q and k with the engine's score bound. Gain 1: every row
    settles after the first key block (bound - max < 64 log2 units) and skips
    the row-max pass; with the sharp tail the later keys lie along the queries,
    so the true scores climb towards the bound after the rows settled. Gain 3:
    the bound (~118 log2 units) is too far above the scores to settle, so the
    row-max pass and the lazy rescale keep running with a bound given."""
    B, H, N = 1, 2, 640
    gen = torch.Generator(device="cuda").manual_seed(17)

    def normed(x, g):
        return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * g).to(torch.bfloat16)

    gq = gain * (1 + 0.05 * torch.randn(128, device="cuda", generator=gen))
    gk = gain * (1 + 0.05 * torch.randn(128, device="cuda", generator=gen))
    qr = torch.randn(B, H, N, 128, device="cuda", generator=gen)
    kr = torch.randn(B, H, N, 128, device="cuda", generator=gen)
    if sharp_tail:  # keys 400.. point along query 0's direction: large late scores
        kr[:, :, 400:] = qr[:, :, :1] + 0.1 * kr[:, :, 400:]
    q, k = normed(qr, gq), normed(kr, gk)
    v = torch.randn(B, H, N, 128, device="cuda", generator=gen).to(torch.bfloat16)
    bound = K.score_bound([gq], [gk])
    scores = (q.float() @ k.float().transpose(-1, -2)) * 128**-0.5
    assert float(scores.abs().max()) <= bound
    out = torch.empty(B, N, H * 128, device="cuda", dtype=torch.bfloat16)
    K.flash_attention(q, k, v, out, bound=bound)
    expected = ops.sdpa(q.float(), k.float(), v.float()).transpose(1, 2).reshape(B, N, H * 128)
    assert torch.isfinite(out).all()
    assert rel_err(out, expected) < 2e-2
    assert K.device_error() == 0


# ---------------------------------------------------------- heads, layout, small
@pytest.mark.parametrize("channels", [3, 4])
@pytest.mark.parametrize("pixel_dtype", [torch.float32, torch.bfloat16])
def test_pixel_embed_matches_reference(K, channels, pixel_dtype):
    """iris_pixel_embed through the C ABI (PixelEmbedder.forward,
    src/iris3b/nn/embeddings.py:319-328, plus the first block's pixel RMSNorm)
    for RGB and for the depth export's widened 4-channel embedder
    (src/iris3b/downstream/depth.py:30-38), against the fp32 restatement."""
    from iris_b200 import _lib

    B, H, W, p = 2, 32, 48, 16
    L = (H // p) * (W // p)
    gen = torch.Generator(device="cuda").manual_seed(21 + channels)
    x = torch.randn(B, channels, H, W, device="cuda", generator=gen)
    w = 0.5 * torch.randn(16, channels, device="cuda", generator=gen)
    b = 0.1 * torch.randn(16, device="cuda", generator=gen)
    pos = torch.randn(H * W, 16, device="cuda", generator=gen)
    gain = torch.rand(16, device="cuda", generator=gen) + 0.5
    pix = torch.empty(B * L * p * p, 16, device="cuda", dtype=pixel_dtype)
    nrm = torch.empty(B * L, p * p * 16, device="cuda", dtype=torch.bfloat16)
    code = _lib.F32 if pixel_dtype == torch.float32 else _lib.BF16
    _lib.call("iris_pixel_embed", x.data_ptr(), w.data_ptr(), b.data_ptr(), pos.data_ptr(), pix.data_ptr(), code,
              nrm.data_ptr(), gain.data_ptr(), 1e-6, B, channels, H, W, p, 0, L,
              torch.cuda.current_stream().cuda_stream)  # fmt: skip
    want = ops.pixel_regroup(ops.linear(x.permute(0, 2, 3, 1), w, b) + pos.view(H, W, 16), p)
    got = pix.view(B * L, p * p, 16)
    assert rel_err(got, want) < (1e-5 if pixel_dtype == torch.float32 else 1e-2)
    want_norm = F.rms_norm(want.to(pixel_dtype).float(), (16,), gain, 1e-6)
    assert rel_err(nrm.view(B * L, p * p, 16), want_norm) < 2e-2
    with pytest.raises(ValueError, match="channels"):  # more than 4 input channels: rejected before any launch
        _lib.call("iris_pixel_embed", x.data_ptr(), w.data_ptr(), b.data_ptr(), pos.data_ptr(), pix.data_ptr(), code,
                  nrm.data_ptr(), gain.data_ptr(), 1e-6, B, 5, H, W, p, 0, L,
                  torch.cuda.current_stream().cuda_stream)  # fmt: skip


def test_qkv_heads_matches_oracle(K):
    from iris_b200 import _lib

    B, N, T, hq, hkv = 2, 40, 9, 3, 1
    gen = torch.Generator().manual_seed(2)
    qkv = torch.randn(B, N, (hq + 2 * hkv) * 128, generator=gen).to(torch.bfloat16)
    qw, kw = torch.rand(128, generator=gen) + 0.5, torch.rand(128, generator=gen) + 0.5
    cis = ops.rope_2d(128, 4, 10, 1e4, 16.0, "isotropic")
    cis = torch.cat([ops.rope_1d(128, T, 1e4), cis])
    cos, sin = torch.view_as_real(cis)[..., 0].contiguous(), torch.view_as_real(cis)[..., 1].contiguous()
    q = torch.zeros(B, hq, T + N, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(B, hkv, T + N, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.zeros(B, hkv, T + N, 128, device="cuda", dtype=torch.bfloat16)
    # device copies held in variables: the launch is asynchronous
    g, qw_d, kw_d, cos_d, sin_d = (t.cuda() for t in (qkv, qw, kw, cos, sin))
    _lib.call("iris_qkv_heads", g.data_ptr(), B, N, g.shape[-1], hq, hkv, qw_d.data_ptr(), kw_d.data_ptr(),
              cos_d.data_ptr(), sin_d.data_ptr(), 1e-6, q.data_ptr(), k.data_ptr(), v.data_ptr(), T + N, T + N, T, 0,
              torch.cuda.current_stream().cuda_stream)  # fmt: skip
    torch.cuda.synchronize()
    c, s = cos[T:], sin[T:]
    eq = ops.qk_norm_rope_reference(qkv[..., : hq * 128].float(), qw, c, s, 1e-6)
    ek = ops.qk_norm_rope_reference(qkv[..., hq * 128 : (hq + hkv) * 128].float(), kw, c, s, 1e-6)
    ev = qkv[..., (hq + hkv) * 128 :].reshape(B, N, hkv, 128).transpose(1, 2)
    torch.testing.assert_close(q[:, :, T:].float().cpu(), eq, rtol=8e-3, atol=1e-2)
    torch.testing.assert_close(k[:, :, T:].float().cpu(), ek, rtol=8e-3, atol=1e-2)
    assert torch.equal(v[:, :, T:].cpu(), ev)
    assert torch.all(q[:, :, :T] == 0)


def test_patchify_and_unpatchify_are_bit_exact(K):
    from iris_b200 import _lib

    st = torch.cuda.current_stream().cuda_stream
    for (B, H, W, p) in ((2, 32, 48, 16), (1, 24, 16, 4)):
        x = (torch.arange(B * 3 * H * W, dtype=torch.float32) % 251).reshape(B, 3, H, W)
        out = torch.empty(B * (H // p) * (W // p), 3 * p * p, device="cuda", dtype=torch.bfloat16)
        xc = x.cuda()
        _lib.call("iris_patchify", xc.data_ptr(), out.data_ptr(), B, 3, H, W, p, 0, (H // p) * (W // p), st)
        assert torch.equal(out.float().cpu(), ops.patchify(x, p).reshape(-1, 3 * p * p))
        pix = torch.randn(B * (H // p) * (W // p), p * p, 3)
        v = torch.empty(B, 3, H, W, device="cuda")
        pc = pix.cuda()
        _lib.call("iris_unpatchify", pc.data_ptr(), v.data_ptr(), B, 3, H, W, p, st)
        assert torch.equal(v.cpu(), ops.unpatchify_pixels(pix, B, H, W, p))


def test_timestep_gemv_and_cfg_euler(K):
    from iris_b200 import _lib

    st = torch.cuda.current_stream().cuda_stream
    t = torch.tensor([0.0, 125.0, 625.0, 938.0, 1000.0])
    feats = torch.empty(5, 256, device="cuda")
    tc = t.cuda()
    _lib.call("iris_timestep_embedding", tc.data_ptr(), feats.data_ptr(), 5, 256, 10.0, st)
    # phases reach 1000 rad, whose fp32 ulp is 6.1e-5: allow 2.5 ulp of phase
    torch.testing.assert_close(feats.cpu(), ops.timestep_embedding(t, 256, 10.0), rtol=1e-5, atol=1.5e-4)
    gen = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(5, 512, device="cuda", generator=gen)
    w = torch.randn(384, 512, device="cuda", generator=gen) * 0.05
    b = torch.randn(384, device="cuda", generator=gen)
    out = torch.empty(5, 384, device="cuda")
    _lib.call("iris_gemv", x.data_ptr(), 5, 512, w.data_ptr(), _lib.F32, b.data_ptr(), out.data_ptr(), 384, 1, 1, st)
    torch.testing.assert_close(out, F.silu(F.silu(x) @ w.T + b), rtol=1e-4, atol=1e-5)
    v = torch.randn(4, 3, 8, 8, device="cuda", generator=gen)
    xs = torch.randn(2, 3, 8, 8, device="cuda", generator=gen)
    nxt = torch.empty_like(xs)
    _lib.call("iris_cfg_euler", v.data_ptr(), xs.data_ptr(), nxt.data_ptr(), 2, 192, 3.0, 0.938, 0.833, 1, st)
    vg = v[:2] + 3.0 * (v[2:] - v[:2])
    clean = xs - 0.938 * vg
    expected = (1 - 0.833) * clean + 0.833 * (xs - (1 - 0.938) * clean) / 0.938
    torch.testing.assert_close(nxt, expected, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("M,N,Kd", [(2, 18432, 3072), (16, 18432, 3072), (20, 3072, 3072), (1, 3072, 256),
                                     (3, 100, 200)])  # fmt: skip
@pytest.mark.parametrize("w_dtype", [torch.bfloat16, torch.float32])
def test_gemv_matches_fp32_reference(K, M, N, Kd, w_dtype):
    """The conditioning GEMV at the shared adaLN core (18432 x 3072) and
    timestep-MLP shapes, B = 2 and the 16 rows of the benchmark's calls (one
    pass over the weights), more rows than one pass, ragged K and N."""
    from iris_b200 import _lib

    gen = torch.Generator(device="cuda").manual_seed(M + N)
    x = torch.randn(M, Kd, device="cuda", generator=gen)
    w = (torch.randn(N, Kd, device="cuda", generator=gen) * 0.02).to(w_dtype)
    b = torch.randn(N, device="cuda", generator=gen)
    out = torch.empty(M, N, device="cuda")
    _lib.call("iris_gemv", x.data_ptr(), M, Kd, w.data_ptr(), _lib.BF16 if w_dtype == torch.bfloat16 else _lib.F32,
              b.data_ptr(), out.data_ptr(), N, 1, 0, torch.cuda.current_stream().cuda_stream)  # fmt: skip
    want = F.silu(x) @ w.float().T + b
    torch.testing.assert_close(out, want, rtol=1e-4, atol=1e-4)


def test_grouped_residual_matches_separate_launches(K):
    """A dual block's text and image residual updates in one launch
    (iris_gated_residual_rms_norm_grouped) give bit-identical rows to one launch
    per stream, each stream with its own gains, modulation rows and row maps."""
    from iris_b200 import _lib

    gen = torch.Generator(device="cuda").manual_seed(13)
    B, T, L, D = 2, 48, 200, 3072
    N = T + L
    tokens = torch.randn(B * N, D, device="cuda", generator=gen)
    branch = torch.randn(B * N, D, device="cuda", generator=gen).to(torch.bfloat16)
    mods = [torch.randn(B, 6 * D, device="cuda", generator=gen) * 0.1 for _ in range(2)]
    gains = [torch.rand(D, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    st = torch.cuda.current_stream().cuda_stream

    def problems(res, nxt):
        out = []
        for i, (rows, rpb, tmap, off) in enumerate(((B * T, T, (T, N, 0), 0), (B * L, L, (L, N, T), B * T))):
            m = mods[i]
            out.append(_lib.ResidualProblem(
                res.data_ptr(), *tmap, branch[off:].data_ptr(), rows, 0, 0, gains[i].data_ptr(),
                m.data_ptr() + 2 * D * 4, 6 * D, rows, rpb, _lib.NEXT_NORM_MODULATE, gains[2 + i].data_ptr(),
                m.data_ptr() + 3 * D * 4, m.data_ptr() + 4 * D * 4, 6 * D, nxt[off:].data_ptr(), rows, 0, 0,
            ))  # fmt: skip
        return out

    res_a, res_b = tokens.clone(), tokens.clone()
    nxt_a, nxt_b = (torch.zeros(B * N, D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    probs = problems(res_a, nxt_a)
    _lib.call("iris_gated_residual_rms_norm_grouped", (_lib.ResidualProblem * 2)(*probs), 2, _lib.BF16, _lib.BF16, D,
              1e-6, st)  # fmt: skip
    for q in problems(res_b, nxt_b):
        _lib.call("iris_gated_residual_rms_norm_grouped", (_lib.ResidualProblem * 1)(q), 1, _lib.BF16, _lib.BF16, D,
                  1e-6, st)  # fmt: skip
    torch.cuda.synchronize()
    assert torch.equal(res_a, res_b) and torch.equal(nxt_a, nxt_b)
    assert not torch.equal(res_a, tokens)


def test_require_finite_on_device(K):
    from iris_b200.model import require_finite

    ok = torch.zeros(2, 3, device="cuda")
    assert require_finite(ok) is ok
    for bad in (float("inf"), float("nan")):
        with pytest.raises(FloatingPointError):
            require_finite(torch.tensor([0.0, bad], device="cuda"))


def test_flow_dpm_solver_matches_reference(K):
    """FlowDPMSolver with the fused iris_dpm_update step against the reference's
    own samples (first order, second order with shift and CFG, unguided)."""
    from iris_b200.sampling import FlowDPMSolver

    fx = golden("samplers")
    dev = torch.device("cuda")
    z, cond, uncond = (fx["inputs"][k].to(dev) for k in ("z", "cond", "uncond"))

    def model_fn(x, t, text):
        return 0.3 * x + 0.05 * text + 1e-4 * t[:, None, None, None]

    for key, case in fx.items():
        if key.startswith("dpm_"):
            solver = FlowDPMSolver(model_fn, cfg_scale=case["cfg_scale"])
            out = solver.sample(z, cond, uncond, steps=case["steps"], order=case["order"], shift=case["shift"])
            torch.testing.assert_close(out.cpu(), case["sample"], rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError):
        FlowDPMSolver(model_fn).sample(z.cpu(), cond.cpu())


@pytest.mark.parametrize("guided,predict_x,second", [(1, 0, 1), (0, 1, 0), (1, 1, 1), (0, 0, 1)])
def test_dpm_update_kernel_matches_fp32(K, guided, predict_x, second):
    from iris_b200 import _lib
    from iris_b200.kernels import stream_of

    g = torch.Generator(device="cpu").manual_seed(7)
    images, per_image = 3, 3 * 40 * 24
    v = torch.randn((2 if guided else 1) * images, per_image, generator=g).cuda()
    x, x0p = (torch.randn(images, per_image, generator=g).cuda() for _ in range(2))
    s, cfg, a, b, c = 0.71, 3.0, 0.93, 0.41, (-0.17 if second else 0.0)
    x0, xn = torch.empty_like(x), torch.empty_like(x)
    _lib.call("iris_dpm_update", v.data_ptr(), x.data_ptr(), x0p.data_ptr(), x0.data_ptr(), xn.data_ptr(), images,
              per_image, cfg, guided, s, predict_x, a, b, c, stream_of(x))
    out = v[:images] + cfg * (v[images:] - v[:images]) if guided else v
    ref_x0 = out if predict_x else x - s * out
    ref = a * x + b * ref_x0 + c * (ref_x0 - x0p)
    torch.testing.assert_close(x0, ref_x0, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(xn, ref, rtol=1e-6, atol=1e-6)
