"""Sequence parallelism (Ulysses) on the B200.

* the kernels it adds: iris_block_copy, attention with fewer queries than
  keys, head-major Q/K/V with separate query / key lengths, and the
  token-range forms of patchify, pixel embed and the pixel head (bit-exact
  against slices of the whole-image calls);
* the peer-memory exchange: the Q/K/V epilogue's scatter / broadcast and the
  attention epilogue's scatter into other ranks' buffers, emulated on one GPU
  by giving the kernels local buffers as the "peers" (each rank's launch runs
  in turn); the barrier's bounded wait running out on a flag nothing sets; a
  CUDA IPC round trip through a second process;
* the engine: P ranks as threads on one GPU (tests/thread_comm.py, the
  collective exchange) against the same model run without sequence
  parallelism, and P = 2 processes (the peer-memory exchange) when the box has
  two GPUs.
"""

import os

import pytest
import torch

from conftest import golden, requires_gpu
from oracle import ops
from oracle.config import OracleConfig, PixelConfig
from oracle.params import seeded_init
from thread_comm import emulated_block_copy, run_ranks

pytestmark = requires_gpu

REL_TOL = 2e-2


def rel_err(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max())


@pytest.fixture(scope="module")
def iris():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import iris_b200

    return iris_b200


# ------------------------------------------------------------------------- kernels
def test_block_copy_matches_emulation(iris):
    from iris_b200 import kernels as K

    gen = torch.Generator().manual_seed(0)
    src = torch.randint(0, 255, (3 * 5 * 7 * 64,), generator=gen, dtype=torch.uint8)
    dst = torch.zeros(3 * 5 * 7 * 96 + 32, dtype=torch.uint8)
    # blocks of 48 bytes: src [5, 3, 7, 64 B] read as (i0 < 3, i1 < 5, i2 < 7), dst [7, 5, 3, 96 B] + 32
    args = ((96, 3 * 96, 5 * 3 * 96), (64 * 7, 64 * 7 * 3, 64), (3, 5, 7), 48)
    want = dst.clone()
    emulated_block_copy(want, args[0], src, args[1], args[2], args[3], dst_offset=32, src_offset=16)
    got = dst.cuda()
    K.block_copy(got, args[0], src.cuda(), args[1], args[2], args[3], dst_offset=32, src_offset=16)
    assert torch.equal(got.cpu(), want)
    # a large block (several 16 KB chunks per block)
    big = torch.randn(2, 3, 40000, device="cuda")
    out = torch.empty(3, 2, 40000, device="cuda")
    K.block_copy(out, (40000 * 4, 2 * 40000 * 4, 0), big, (3 * 40000 * 4, 40000 * 4, 0), (2, 3, 1), 40000 * 4)
    assert torch.equal(out, big.transpose(0, 1))


@pytest.mark.parametrize("n,n_kv", [(100, 300), (300, 52), (256, 4352)])
def test_attention_with_fewer_queries_than_keys(iris, n, n_kv):
    from iris_b200 import kernels as K

    B, H = 2, 3
    gen = torch.Generator(device="cuda").manual_seed(n + n_kv)
    q = torch.randn(B, H, n, 128, device="cuda", generator=gen).to(torch.bfloat16)
    k = torch.randn(B, H, n_kv, 128, device="cuda", generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n_kv, 128, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.empty(B, n, H * 128, device="cuda", dtype=torch.bfloat16)
    K.flash_attention(q, k, v, out)
    expected = ops.sdpa(q.float(), k.float(), v.float()).transpose(1, 2).reshape(B, n, H * 128)
    assert rel_err(out, expected) < REL_TOL


def test_qkv_heads_head_major_and_key_length(iris):
    from iris_b200 import _lib

    B, N, hq, hkv, pad = 2, 40, 4, 2, 48
    gen = torch.Generator(device="cuda").manual_seed(4)
    qkv = torch.randn(B * N, (hq + 2 * hkv) * 128, device="cuda", generator=gen).to(torch.bfloat16)
    qw, kw = (torch.rand(128, device="cuda", generator=gen) + 0.5 for _ in range(2))
    cos, sin = (torch.randn(N, 64, device="cuda", generator=gen) for _ in range(2))
    st = torch.cuda.current_stream().cuda_stream

    def run(head_major, n_kv):
        shape = (hq, B, N, 128) if head_major else (B, hq, N, 128)
        q = torch.zeros(*shape, device="cuda", dtype=torch.bfloat16)
        kshape = (hkv, B, n_kv, 128) if head_major else (B, hkv, n_kv, 128)
        k, v = (torch.zeros(*kshape, device="cuda", dtype=torch.bfloat16) for _ in range(2))
        _lib.call("iris_qkv_heads", qkv.data_ptr(), B, N, qkv.shape[1], hq, hkv, qw.data_ptr(), kw.data_ptr(),
                  cos.data_ptr(), sin.data_ptr(), 1e-6, q.data_ptr(), k.data_ptr(), v.data_ptr(), N, n_kv, 0,
                  head_major, st)  # fmt: skip
        return q, k, v

    q0, k0, v0 = run(0, N)
    q1, k1, v1 = run(1, N)
    assert torch.equal(q1.transpose(0, 1), q0) and torch.equal(k1.transpose(0, 1), k0)
    assert torch.equal(v1.transpose(0, 1), v0)
    q2, k2, v2 = run(0, pad)
    assert torch.equal(q2, q0) and torch.equal(k2[:, :, :N], k0) and torch.equal(v2[:, :, :N], v0)
    assert torch.all(k2[:, :, N:] == 0)


def _heads_problem_inputs(B, N, hq, hkv, K_dim, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = (0.5 * torch.randn(B * N, K_dim, device="cuda", generator=gen)).to(torch.bfloat16)
    w = (0.05 * torch.randn((hq + 2 * hkv) * 128, K_dim, device="cuda", generator=gen)).to(torch.bfloat16)
    qw, kw = (torch.rand(128, device="cuda", generator=gen) + 0.5 for _ in range(2))
    cos, sin = (torch.randn(N, 64, device="cuda", generator=gen) for _ in range(2))
    return a, w, qw, kw, cos, sin


@pytest.mark.parametrize("world", [2, 4])
def test_heads_epilogue_scatters_to_owner_ranks(iris, world):
    """Rank r's tokens, projected with the peer-scatter epilogue into every rank's
    full-sequence buffers, equal the one-rank projection of all tokens sliced
    by head group (the ranks' launches run in turn on one GPU)."""
    from iris_b200 import _lib
    from iris_b200 import kernels as K

    B, n, hq, hkv, K_dim = 2, 136, 8, 4, 256
    N = world * n
    a, w, qw, kw, cos, sin = _heads_problem_inputs(B, N, hq, hkv, K_dim, world)
    q_ref = torch.zeros(B, hq, N, 128, device="cuda", dtype=torch.bfloat16)
    k_ref, v_ref = (torch.zeros(B, hkv, N, 128, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    ref = K.HeadsOut(q_ref, k_ref, v_ref, qw, kw, cos, sin, 1e-6, hq, hkv, N, B, N, N)
    K.gemm_grouped([K.gemm_problem(a, w, None, heads=ref)], torch.cuda.current_stream().cuda_stream)
    qf = [torch.zeros(B, hq // world, N, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    kf = [torch.zeros(B, hkv // world, N, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    vf = [torch.zeros_like(t) for t in kf]
    for r in range(world):
        rows = a.view(B, N, K_dim)[:, r * n : (r + 1) * n].reshape(B * n, K_dim).contiguous()
        peers = K.PeerHeads(_lib.HEADS_PEER_SCATTER, [t.data_ptr() for t in qf], [t.data_ptr() for t in kf],
                            [t.data_ptr() for t in vf], r * n, N)  # fmt: skip
        heads = K.HeadsOut(None, None, None, qw, kw, cos[r * n :], sin[r * n :], 1e-6, hq, hkv, n, B, n, n,
                           peers=peers)  # fmt: skip
        K.gemm_grouped([K.gemm_problem(rows, w, None, heads=heads)], torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for j in range(world):
        hq_l, hkv_l = hq // world, hkv // world
        assert rel_err(qf[j], q_ref[:, j * hq_l : (j + 1) * hq_l]) < 1e-3
        assert rel_err(kf[j], k_ref[:, j * hkv_l : (j + 1) * hkv_l]) < 1e-3
        assert rel_err(vf[j], v_ref[:, j * hkv_l : (j + 1) * hkv_l]) < 1e-3


def test_heads_epilogue_broadcasts_keys_values(iris):
    """Pixel-stage form: q stays local, k and v of this rank's tokens go to every
    rank's full buffers at the rank's token offset."""
    from iris_b200 import _lib
    from iris_b200 import kernels as K

    world, B, n, h, K_dim = 3, 2, 72, 2, 128
    N = world * n
    a, w, qw, kw, cos, sin = _heads_problem_inputs(B, N, h, h, K_dim, 11)
    q_ref = torch.zeros(B, h, N, 128, device="cuda", dtype=torch.bfloat16)
    k_ref, v_ref = (torch.zeros(B, h, N, 128, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    ref = K.HeadsOut(q_ref, k_ref, v_ref, qw, kw, cos, sin, 1e-6, h, h, N, B, N, N)
    st = torch.cuda.current_stream().cuda_stream
    K.gemm_grouped([K.gemm_problem(a, w, None, heads=ref)], st)
    kf = [torch.zeros(B, h, N, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    vf = [torch.zeros_like(t) for t in kf]
    qs = []
    for r in range(world):
        rows = a.view(B, N, K_dim)[:, r * n : (r + 1) * n].reshape(B * n, K_dim).contiguous()
        q_loc = torch.zeros(B, h, n, 128, device="cuda", dtype=torch.bfloat16)
        peers = K.PeerHeads(_lib.HEADS_PEER_BROADCAST_KV, None, [t.data_ptr() for t in kf],
                            [t.data_ptr() for t in vf], r * n, N)  # fmt: skip
        heads = K.HeadsOut(q_loc, None, None, qw, kw, cos[r * n :], sin[r * n :], 1e-6, h, h, n, B, n, N,
                           peers=peers)  # fmt: skip
        K.gemm_grouped([K.gemm_problem(rows, w, None, heads=heads)], st)
        qs.append(q_loc)
    torch.cuda.synchronize()
    for j in range(world):
        assert rel_err(kf[j], k_ref) < 1e-3 and rel_err(vf[j], v_ref) < 1e-3
        assert rel_err(qs[j], q_ref[:, :, j * n : (j + 1) * n]) < 1e-3


def test_attention_epilogue_scatters_rows_to_token_owners(iris):
    """Attention of one rank's heads over every token, each output row stored into
    the token rows of the rank that owns the token (at this rank's columns),
    equals the plain output re-laid out."""
    from iris_b200 import kernels as K

    world, rank, B, hl, n = 2, 1, 2, 3, 160
    H, N = world * hl, world * n
    gen = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(B, hl, N, 128, device="cuda", generator=gen).to(torch.bfloat16) for _ in range(3))
    ref = torch.empty(B, N, hl * 128, device="cuda", dtype=torch.bfloat16)
    K.flash_attention(q, k, v, ref)
    rows = [torch.zeros(B * n, H * 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    K.flash_attention_peers(q, k, v, [t.data_ptr() for t in rows], n, rank * hl * 128, H * 128)
    torch.cuda.synchronize()
    for j in range(world):
        got = rows[j].view(B, n, H * 128)[:, :, rank * hl * 128 : (rank + 1) * hl * 128]
        assert torch.equal(got, ref[:, j * n : (j + 1) * n])
        others = rows[j].view(B, n, H * 128)[:, :, : rank * hl * 128]
        assert torch.all(others == 0)


def test_peer_barrier_wait_runs_out_and_reports(iris):
    """The barrier signals the peer's slot and, with no peer to answer, its bounded
    wait gives up and sets the device error bit; with the peer's flag already
    set it returns without one. (No second GPU: the "peer" is a local buffer.)"""
    from iris_b200 import kernels as K

    K.device_error(clear=True)
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    peer = torch.zeros(2, dtype=torch.int32, device="cuda")
    K.peer_barrier(flags, [0, peer.data_ptr()], 0, 7, timeout_s=0.02)
    assert K.device_error(clear=True) & 1, "the wait on a flag nothing sets must time out"
    assert int(peer[0]) == 7, "the barrier must signal the peer's slot for this rank"
    flags[1] = 9
    K.peer_barrier(flags, [0, peer.data_ptr()], 0, 8, timeout_s=0.02)
    assert K.device_error(clear=True) == 0 and int(peer[0]) == 8


def test_timed_out_wait_makes_the_result_raise(iris):
    """After a bounded wait has given up (the barrier on a flag nothing sets, as
    above), the next denoiser call's velocity is NaN-filled on the device and
    require_finite raises DeviceWaitTimeout naming the timeout (no host sync
    inside the call); the error word is then cleared and the engine recovers.
    The pipeline, which calls require_finite, raises the same way."""
    from iris_b200 import kernels as K
    from iris_b200.model import DeviceWaitTimeout

    fx = golden("released_mha")
    cfg = _config(fx["config"])
    engine = iris.CudaIris(iris.IrisWeights(cfg, {k: v.cuda() for k, v in seeded_init(cfg, seed=0).items()}))
    x, t, text = fx["x"].cuda(), fx["t"].cuda(), fx["prepared_text"].cuda()
    K.device_error(clear=True)
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    peer = torch.zeros(2, dtype=torch.int32, device="cuda")
    K.peer_barrier(flags, [0, peer.data_ptr()], 0, 1, timeout_s=0.02)
    v = engine(x, t, text)
    assert torch.isnan(v).all(), "a result computed after a timed-out wait must not look valid"
    with pytest.raises(DeviceWaitTimeout, match="timed out"):
        iris.require_finite(v)
    assert K.device_error(clear=False) == 0, "require_finite clears the word it reported"
    v = engine(x, t, text)
    assert rel_err(v, fx["v"]) < REL_TOL
    iris.require_finite(v)
    d = fx["euler_cfg"]
    pipe = iris.DenoisePipeline(engine, cfg_scale=d["cfg_scale"], cfg_interval=d["cfg_interval"])
    K.peer_barrier(flags, [0, peer.data_ptr()], 0, 2, timeout_s=0.02)
    with pytest.raises(DeviceWaitTimeout):
        pipe(d["noise"], d["cond"], d["uncond"], adapted=True)
    assert K.device_error(clear=True) == 0


def _ipc_child(handle, offset, numel, queue):
    import torch

    from iris_b200 import kernels as K

    torch.cuda.set_device(0)
    base = K.ipc_import(handle)
    out = torch.empty(numel, dtype=torch.float32, device="cuda")
    # read the parent's buffer through the mapping, then write into it
    K.block_copy(out.view(torch.uint8), (0, 0, 0), _raw(base + offset, numel * 4), (0, 0, 0), (1, 1, 1), numel * 4)
    K.block_copy(_raw(base + offset, numel * 4), (0, 0, 0), (out * 2).view(torch.uint8), (0, 0, 0), (1, 1, 1),
                 numel * 4)  # fmt: skip
    torch.cuda.synchronize()
    K.ipc_close(base)
    queue.put(float(out.sum()))


def _raw(ptr, nbytes):
    """A uint8 CUDA tensor viewing device memory at ``ptr`` (no ownership)."""
    import torch

    class _Mem:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}

    return torch.as_tensor(_Mem(), device="cuda")


def test_ipc_round_trip_through_a_second_process(iris):
    import torch.multiprocessing as mp

    from iris_b200 import kernels as K

    pool = torch.empty(1 << 20, dtype=torch.float32, device="cuda")
    buf = pool[4096 : 4096 + 1000]
    buf.copy_(torch.arange(1000, dtype=torch.float32, device="cuda"))
    torch.cuda.synchronize()
    handle, offset = K.ipc_export(buf)
    # the offset is from the base of the allocation holding the buffer (at or below the pool's start)
    assert offset >= buf.data_ptr() - pool.data_ptr() and len(handle) == 64
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    proc = ctx.Process(target=_ipc_child, args=(handle, offset, 1000, queue))
    proc.start()
    proc.join(timeout=120)
    assert proc.exitcode == 0
    assert queue.get(timeout=10) == float(sum(range(1000)))
    assert torch.equal(buf, 2 * torch.arange(1000, dtype=torch.float32, device="cuda"))


def test_token_range_layout_kernels_match_whole_image(iris):
    from iris_b200 import _lib

    st = torch.cuda.current_stream().cuda_stream
    B, H, W, p = 2, 32, 48, 16
    L, pp = (H // p) * (W // p), p * p
    t0, cnt = 1, 4
    gen = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(B, 3, H, W, device="cuda", generator=gen)
    full = torch.empty(B * L, 3 * pp, device="cuda", dtype=torch.bfloat16)
    part = torch.empty(B * cnt, 3 * pp, device="cuda", dtype=torch.bfloat16)
    _lib.call("iris_patchify", x.data_ptr(), full.data_ptr(), B, 3, H, W, p, 0, L, st)
    _lib.call("iris_patchify", x.data_ptr(), part.data_ptr(), B, 3, H, W, p, t0, cnt, st)
    assert torch.equal(part.view(B, cnt, -1), full.view(B, L, -1)[:, t0 : t0 + cnt])

    w, b = torch.randn(16, 3, device="cuda", generator=gen), torch.randn(16, device="cuda", generator=gen)
    pos = torch.randn(H * W, 16, device="cuda", generator=gen)
    gain = torch.rand(16, device="cuda", generator=gen) + 0.5
    pix_f, nrm_f = torch.empty(B * L * pp, 16, device="cuda"), torch.empty(B * L, pp * 16, device="cuda", dtype=torch.bfloat16)
    pix_p, nrm_p = torch.empty(B * cnt * pp, 16, device="cuda"), torch.empty(B * cnt, pp * 16, device="cuda", dtype=torch.bfloat16)
    for pix, nrm, start, count in ((pix_f, nrm_f, 0, L), (pix_p, nrm_p, t0, cnt)):
        _lib.call("iris_pixel_embed", x.data_ptr(), w.data_ptr(), b.data_ptr(), pos.data_ptr(), pix.data_ptr(),
                  _lib.F32, nrm.data_ptr(), gain.data_ptr(), 1e-6, B, 3, H, W, p, start, count, st)  # fmt: skip
    assert torch.equal(pix_p.view(B, cnt, -1), pix_f.view(B, L, -1)[:, t0 : t0 + cnt])
    assert torch.equal(nrm_p.view(B, cnt, -1), nrm_f.view(B, L, -1)[:, t0 : t0 + cnt])

    branch = torch.randn(B * L * pp, 16, device="cuda", generator=gen).to(torch.bfloat16)
    mods = (0.1 * torch.randn(B * L * pp, 64, device="cuda", generator=gen)).to(torch.bfloat16)
    fc1w, fc2w = (0.2 * torch.randn(64, 16, device="cuda", generator=gen)).to(torch.bfloat16), (
        0.2 * torch.randn(16, 64, device="cuda", generator=gen)
    ).to(torch.bfloat16)
    fc1b, fc2b = (0.1 * torch.randn(64, device="cuda", generator=gen)).to(torch.bfloat16), (
        0.1 * torch.randn(16, device="cuda", generator=gen)
    ).to(torch.bfloat16)
    fw, fb = torch.randn(3, 16, device="cuda", generator=gen), torch.randn(3, device="cuda", generator=gen)
    v_full = torch.zeros(B, 3, H, W, device="cuda")
    v_part = torch.zeros(B, 3, H, W, device="cuda")

    def sl(t):
        return t.view(B, L, -1)[:, t0 : t0 + cnt].reshape(B * cnt * pp, -1).contiguous()

    args_f = (pix_f, branch, mods, v_full, 0, L)
    args_p = (sl(pix_f), sl(branch), sl(mods), v_part, t0, cnt)
    for pix, br, md, v, start, count in (args_f, args_p):
        _lib.call("iris_pixel_mlp_head", pix.data_ptr(), _lib.F32, br.data_ptr(), md.data_ptr(), gain.data_ptr(),
                  fc1w.data_ptr(), fc1b.data_ptr(), fc2w.data_ptr(), fc2b.data_ptr(), gain.data_ptr(), fw.data_ptr(),
                  fb.data_ptr(), v.data_ptr(), B, H, W, p, start, count, 1e-6, st)  # fmt: skip
    mask = torch.zeros(B, 3, H // p, W // p, dtype=torch.bool, device="cuda")
    for l in range(t0, t0 + cnt):
        mask[:, :, l // (W // p), l % (W // p)] = True
    mask = mask.repeat_interleave(p, 2).repeat_interleave(p, 3)
    assert torch.equal(v_part[mask], v_full[mask])
    assert torch.all(v_part[~mask] == 0)


# -------------------------------------------------------------------------- engine
def _config(d):
    d = dict(d)
    return OracleConfig(**{**d, "pixel": PixelConfig(**d["pixel"])})


def _four_head_config():
    cfg = _config(golden("released_mha")["config"])
    d = {**cfg.__dict__, "hidden_size": 512, "num_heads": 4}
    d["pixel"] = PixelConfig(**{**cfg.pixel.__dict__, "attn_hidden_size": 512, "num_heads": 4})
    return OracleConfig(**d)


def _sequence_parallel_matches(iris, cfg, x, t, text, world):
    state = {k: v.cuda() for k, v in seeded_init(cfg, seed=0).items()}
    weights = iris.IrisWeights(cfg, state)
    reference = iris.CudaIris(weights)(x, t, text)
    text_before = text.clone()

    def rank_fn(rank, comm):
        engine = iris.CudaIris(weights, comm=comm)
        return engine(x, t, text)

    outs = run_ranks(world, rank_fn)
    assert torch.equal(text, text_before), "the engine must not write its text input"
    for v in outs:
        assert torch.equal(v, outs[0]), "every rank returns the same velocity"
    err = rel_err(outs[0], reference)
    print(f"P={world}: max rel err vs one device {err:.3e}")
    assert err < REL_TOL


def test_engine_sequence_parallel_two_ranks(iris):
    fx = golden("released_mha")
    cfg = _config(fx["config"])
    _sequence_parallel_matches(iris, cfg, fx["x"].cuda(), fx["t"].cuda(), fx["prepared_text"].cuda(), 2)


def test_engine_sequence_parallel_four_ranks(iris):
    cfg = _four_head_config()
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(2, 3, 32, 32, generator=gen).cuda()  # 64 image + 16 text tokens: 20 per rank
    text = torch.randn(2, 16, cfg.hidden_size, generator=gen).cuda()
    t = torch.tensor([125.0, 850.0]).cuda()
    _sequence_parallel_matches(iris, cfg, x, t, text, 4)


def test_engine_sequence_parallel_rejects_indivisible_heads(iris):
    fx = golden("released_gqa")  # one key/value head
    cfg = _config(fx["config"])
    state = {k: v.cuda() for k, v in seeded_init(cfg, seed=0).items()}

    class Two:
        rank, world = 0, 2

    with pytest.raises(ValueError, match="head counts"):
        iris.CudaIris(iris.IrisWeights(cfg, state), comm=Two())


def _nccl_worker(rank, world, port, queue):
    import torch.distributed as dist

    import iris_b200
    from iris_b200.ulysses import TorchComm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        fx = golden("released_mha")
        cfg = _config(fx["config"])
        state = {k: v.cuda() for k, v in seeded_init(cfg, seed=0).items()}
        weights = iris_b200.IrisWeights(cfg, state)
        x, t, text = fx["x"].cuda(), fx["t"].cuda(), fx["prepared_text"].cuda()
        v = iris_b200.CudaIris(weights, comm=TorchComm())(x, t, text)
        ref = iris_b200.CudaIris(weights)(x, t, text)
        torch.cuda.synchronize()
        queue.put((rank, rel_err(v, ref)))
    finally:
        dist.destroy_process_group()


def test_engine_sequence_parallel_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    errs = dict(queue.get(timeout=10) for _ in procs)
    print("NCCL P=2 max rel err per rank:", errs)
    assert all(e < REL_TOL for e in errs.values())
