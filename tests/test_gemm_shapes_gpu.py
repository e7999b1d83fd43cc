"""The CTA-pair GEMM at the shapes of one B = 2 denoiser call (8704 rows per
linear: the last wave of 256 x 256 tiles is partly empty, e.g. 408 tiles over
74 pairs for the 3072-wide linears) and of the text adapter, against the fp32
product: every epilogue (bias, ADD in place, SwiGLU, the gate on aux rows in a
grouped text + image launch, the QK-norm + RoPE heads) and bit-identical
results across repeated launches."""

import pytest
import torch
import torch.nn.functional as F

from conftest import requires_gpu

pytestmark = requires_gpu


def rel_err(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max())


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from iris_b200 import kernels

    return kernels


@pytest.mark.parametrize("M,N,Kd", [
    (8704, 3072, 3072),  # B = 2 gate / out-projection: 408 tiles, 5.5 waves of 74 pairs
    (8704, 3072, 8192),  # B = 2 w2
    (8704, 9216, 3072),  # B = 2 QKV: 16.5 waves
    (2048, 1024, 3072),  # 32 tiles: fewer than the pairs
    (600, 416, 2560),  # ragged M and N (the text adapter's layer MLP)
])  # fmt: skip
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_at_call_shapes(K, M, N, Kd, out_dtype):
    gen = torch.Generator(device="cuda").manual_seed(M + N + Kd)
    a = torch.randn(M, Kd, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(N, Kd, device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=gen)
    outs = []
    for _ in range(3):
        out = torch.full((M, N), float("nan"), device="cuda", dtype=out_dtype)
        K.gemm(a, w, out, bias=bias)
        outs.append(out)
    torch.cuda.synchronize()
    expected = a.float() @ w.float().T + bias
    tol = 1e-2 if out_dtype == torch.bfloat16 else 1e-4
    assert all(torch.equal(o, outs[0]) for o in outs), "repeated launches must agree exactly"
    assert rel_err(outs[0], expected) < tol


def test_epilogues_at_call_shapes(K):
    """ADD (in place, applied once), SWIGLU, GATE and the grouped text + image
    launch at the B = 2 shapes."""
    from iris_b200 import _lib
    from iris_b200.model import pack_swiglu

    gen = torch.Generator(device="cuda").manual_seed(7)
    M, D, Fh = 8704, 3072, 8192
    h = torch.randn(M, D, device="cuda", generator=gen).to(torch.bfloat16)
    wp = (torch.randn(D, D, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    bias = torch.randn(D, device="cuda", generator=gen)
    res = torch.randn(M, D, device="cuda", generator=gen)
    got = res.clone()
    K.gemm(h, wp, got, bias=bias, epilogue=_lib.EPI_ADD)
    ref = h.float() @ wp.float().T + bias
    assert rel_err(got - res, ref) < 1e-3
    # SwiGLU: M = 8704, N = 16384 of interleaved w1 / w3 tiles, and a smaller M
    w1, w3 = ((torch.randn(Fh, D, device="cuda", generator=gen) * 0.02).to(torch.bfloat16) for _ in range(2))
    w2 = (torch.randn(D, Fh, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    w13, _ = pack_swiglu(w1, w3, w2)
    for m in (8704, 1280):
        act = torch.empty(m, Fh, device="cuda", dtype=torch.bfloat16)
        K.gemm(h[:m], w13, act, epilogue=_lib.EPI_SWIGLU)
        want = F.silu(h[:m].float() @ w1.float().T) * (h[:m].float() @ w3.float().T)
        assert rel_err(act, want) < 1e-2
    # gate on aux rows, grouped text (512 rows) + image (8192 rows) problems of one K
    aux = torch.randn(M, D, device="cuda", generator=gen).to(torch.bfloat16)
    wt = (torch.randn(D, D, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    og = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    problems = [
        K.gemm_problem(h[512:], wp, og[512:], epilogue=_lib.EPI_GATE, aux=aux[512:]),
        K.gemm_problem(h[:512], wt, og[:512], epilogue=_lib.EPI_GATE, aux=aux[:512]),
    ]
    K.gemm_grouped(problems, torch.cuda.current_stream().cuda_stream)
    want = torch.cat([aux[:512].float() * torch.sigmoid(h[:512].float() @ wt.float().T),
                      aux[512:].float() * torch.sigmoid(h[512:].float() @ wp.float().T)])  # fmt: skip
    assert rel_err(og, want) < 1e-2


def test_heads_epilogue_at_call_shape(K):
    """The B = 2 QKV projection with QK-norm + RoPE in the epilogue."""
    from oracle import ops

    B, N, H = 2, 4352, 24
    gen = torch.Generator(device="cuda").manual_seed(11)
    h = torch.randn(B * N, 3072, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(3 * 3072, 3072, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    qw, kw = (torch.rand(128, device="cuda", generator=gen) + 0.5 for _ in range(2))
    cis = torch.cat([ops.rope_1d(128, 256, 1e4), ops.rope_2d(128, 64, 64, 1e4, 16.0, "isotropic")])
    cos, sin = torch.view_as_real(cis)[..., 0].contiguous().cuda(), torch.view_as_real(cis)[..., 1].contiguous().cuda()
    q, k, v = (torch.empty(B, H, N, 128, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    heads = K.HeadsOut(q, k, v, qw, kw, cos, sin, 1e-6, H, H, N, B, N, N)
    K.gemm_grouped([K.gemm_problem(h, w, None, heads=heads)], torch.cuda.current_stream().cuda_stream)
    proj = (h.float() @ w.float().T).view(B, N, 3 * 3072)
    want_q = ops.qk_norm_rope_reference(proj[..., :3072], qw, cos, sin, 1e-6)
    want_v = proj[..., 6144:].view(B, N, H, 128).transpose(1, 2)
    assert rel_err(q, want_q) < 1e-2
    assert rel_err(v, want_v) < 1e-2
