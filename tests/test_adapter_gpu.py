"""The masked text adapters on the B200 (``lap_blocks2`` / ``blocks2``,
src/iris3b/nn/embeddings.py:79-266) and the kernels they add.

* kernels: ``iris_small_attention`` against fp32 SDPA with the adapter's mask
  rule (pad keys masked, the diagonal kept), with and without QK RMSNorm, at
  the layer-attention shape (12 keys, 80 wide) and the refiner's (300 keys,
  128 wide); ``iris_layer_pool``; the GEMM's ``EPI_ADD`` / ``EPI_SILU``;
* ``CudaIris.encode_text`` against the reference's own ``embed_text`` outputs
  (tests/golden/adapters.pt) on the toy topology;
* the released adapter's dimensions (12 layers x 2560, 32 + 24 heads, 300
  tokens, hidden 3072) against the fp32 oracle on the same GPU.
"""

import pytest
import torch
import torch.nn.functional as F

from conftest import golden, requires_gpu
from oracle.adapter import AdapterOracle, adapter_param_spec
from oracle.config import OracleConfig, PixelConfig
from oracle.params import seeded_init

pytestmark = requires_gpu

REL_TOL = 2e-2


def rel_err(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max())


def _config(d):
    d = dict(d)
    return OracleConfig(**{**d, "pixel": PixelConfig(**d["pixel"])})


@pytest.fixture(scope="module")
def iris():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    import iris_b200

    return iris_b200


def _attention_reference(qkv, seqs, n, heads, hd, gains, mask, eps=1e-6):
    q, k, v = qkv.float().reshape(seqs, n, 3, heads, hd).unbind(2)
    if gains is not None:
        q = F.rms_norm(q, (hd,), gains[0], eps)
        k = F.rms_norm(k, (hd,), gains[1], eps)
    attn_mask = None
    if mask is not None:
        attn_mask = mask.bool()[:, None, None, :] | torch.eye(n, dtype=torch.bool, device=qkv.device)
    out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), attn_mask=attn_mask)
    return out.transpose(1, 2).reshape(seqs * n, heads * hd)


@pytest.mark.parametrize("seqs,n,heads,hd,normed,masked", [
    (50, 12, 32, 80, False, False),  # layer attention over 12 encoder layers
    (3, 300, 24, 128, True, True),  # refiner over a padded prompt
    (2, 37, 3, 64, True, True),  # ragged key rounds
])  # fmt: skip
def test_small_attention_matches_sdpa(iris, seqs, n, heads, hd, normed, masked):
    from iris_b200 import _lib

    gen = torch.Generator(device="cuda").manual_seed(n)
    qkv = torch.randn(seqs * n, 3 * heads * hd + 16, device="cuda", generator=gen).to(torch.bfloat16)
    gains = (torch.rand(hd, device="cuda", generator=gen) + 0.5, torch.rand(hd, device="cuda", generator=gen) + 0.5)
    mask = None
    if masked:
        mask = torch.rand(seqs, n, device="cuda", generator=gen) > 0.4
        mask[0, :] = False  # a prompt of padding only: each query attends itself
        mask[-1, :] = True
    out = torch.empty(seqs * n, heads * hd, device="cuda", dtype=torch.bfloat16)
    _lib.call("iris_small_attention", qkv.data_ptr(), seqs, n, heads, hd, qkv.stride(0),
              gains[0].data_ptr() if normed else None, gains[1].data_ptr() if normed else None, 1e-6,
              None if mask is None else mask.to(torch.uint8).data_ptr(), hd**-0.5, out.data_ptr(), out.stride(0),
              torch.cuda.current_stream().cuda_stream)  # fmt: skip
    want = _attention_reference(qkv[:, : 3 * heads * hd], seqs, n, heads, hd, gains if normed else None, mask)
    err = rel_err(out, want)
    print(f"small attention n={n} hd={hd}: max rel err {err:.2e}")
    assert err < REL_TOL
    if masked:  # an all-pad prompt degenerates to identity attention: out = v
        v = qkv[:n, 2 * heads * hd : 3 * heads * hd].float()
        assert rel_err(out[:n], v) < REL_TOL


def test_small_attention_rejects_bad_shapes(iris):
    from iris_b200 import _lib

    qkv = torch.zeros(4 * 500, 3 * 128, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(4 * 500, 128, device="cuda", dtype=torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(ValueError, match="shared memory"):
        _lib.call("iris_small_attention", qkv.data_ptr(), 4, 500, 1, 128, 384, None, None, 1e-6, None, 1.0,
                  out.data_ptr(), 128, st)  # fmt: skip
    with pytest.raises(ValueError, match="head_dim"):
        _lib.call("iris_small_attention", qkv.data_ptr(), 4, 500, 1, 100, 384, None, None, 1e-6, None, 1.0,
                  out.data_ptr(), 128, st)  # fmt: skip
    with pytest.raises(ValueError, match="gains"):
        _lib.call("iris_small_attention", qkv.data_ptr(), 4, 50, 1, 128, 384, out.data_ptr(), None, 1e-6, None, 1.0,
                  out.data_ptr(), 128, st)  # fmt: skip


def test_layer_pool_and_gemm_add_silu_epilogues(iris):
    from iris_b200 import _lib
    from iris_b200 import kernels as K

    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(30 * 12, 640, device="cuda", generator=gen)
    w, b = torch.randn(12, device="cuda", generator=gen), torch.randn(1, device="cuda", generator=gen)
    out = torch.empty(30, 640, device="cuda", dtype=torch.bfloat16)
    _lib.call("iris_layer_pool", x.data_ptr(), 30, 12, 640, w.data_ptr(), b.data_ptr(), out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)  # fmt: skip
    want = torch.einsum("rlc,l->rc", x.view(30, 12, 640), w) + b
    assert rel_err(out, want) < 1e-2
    for M in (100, 700):  # one-SM and CTA-pair kernels
        a = torch.randn(M, 256, device="cuda", generator=gen).to(torch.bfloat16)
        wt = torch.randn(416, 256, device="cuda", generator=gen).to(torch.bfloat16)
        bias = torch.randn(416, device="cuda", generator=gen)
        res = torch.randn(M, 416, device="cuda", generator=gen)
        ref = a.float() @ wt.float().T + bias
        got = res.clone()
        K.gemm(a, wt, got, bias=bias, epilogue=_lib.EPI_ADD)
        assert rel_err(got - res, ref) < 1e-3
        act = torch.empty(M, 416, device="cuda", dtype=torch.bfloat16)
        K.gemm(a, wt, act, bias=bias, epilogue=_lib.EPI_SILU)
        assert rel_err(act, F.silu(ref)) < 1e-2
    with pytest.raises(ValueError, match="f32"):
        K.gemm(a, wt, act, bias=bias, epilogue=_lib.EPI_ADD)


@pytest.mark.parametrize("adapter", ["lap_blocks2", "blocks2"])
def test_encode_text_masked_adapter_matches_reference(iris, adapter):
    """encode_text on the engine's kernels against the reference's embed_text
    (the adapter plus y_pos_embedding): a right-padded prompt, scattered real
    tokens, an all-pad prompt; states longer than text_len are truncated; the
    caller's states are not written; without the mask it raises."""
    fx = golden("adapters")[adapter]
    cfg = _config(fx["config"])
    state = {k: v.cuda() for k, v in seeded_init(cfg, seed=0).items()}
    engine = iris.CudaIris(iris.IrisWeights(cfg, state))
    assert engine.masked_adapter is not None
    y = fx["y"].cuda()
    before = y.clone()
    text = engine.encode_text(y, fx["mask"].cuda())
    assert torch.equal(y, before), "encode_text must not write the caller's states"
    err = rel_err(text, fx["prepared_text"])
    print(f"{adapter}: max rel err {err:.2e}")
    assert text.shape == fx["prepared_text"].shape and text.dtype == torch.float32
    assert err < REL_TOL
    with pytest.raises(ValueError, match="mask"):
        engine.encode_text(y)
    # the adapted text drives the denoiser like the linear adapter's
    x = torch.randn(3, 3, 24, 24, device="cuda", generator=torch.Generator(device="cuda").manual_seed(2))
    v = engine(x, torch.full((3,), 500.0, device="cuda"), text)
    assert torch.isfinite(v).all()


def test_released_adapter_dimensions_match_fp32_oracle(iris):
    """The released lap_blocks2 adapter's shapes: 2 prompts of 300 tokens x 12
    encoder layers x 2560 (32 layer heads of 80), refiner at 3072 with 24 QK-normed
    heads and SwiGLU 8192; seeded weights, random padding; the fp32 oracle runs on
    the same GPU."""
    from iris_b200.adapter import TextAdapter
    from iris_b200.config import from_any

    cfg = OracleConfig(hidden_size=3072, num_heads=24, num_kv_heads=None, text_adapter="lap_blocks2")
    gen = torch.Generator(device="cuda").manual_seed(0)
    params = {}
    for name, shape, kind in adapter_param_spec(cfg):
        value = torch.randn(shape, generator=gen, device="cuda") * 0.02
        params[name] = value + 1.0 if kind == "g" else value
    states = torch.randn(2, 300, 12, 2560, generator=gen, device="cuda")
    mask = torch.zeros(2, 300, dtype=torch.bool, device="cuda")
    mask[0, :300] = True
    mask[1, :117] = True
    adapter = TextAdapter(from_any(cfg), {f"y_embedder.{k}": v for k, v in params.items()}, torch.device("cuda"))
    got = adapter(states, mask)
    with torch.no_grad():
        want = AdapterOracle(cfg, params)(states, mask)
    err = rel_err(got, want)
    print(f"released adapter dimensions: max rel err {err:.2e}")
    assert err < REL_TOL
