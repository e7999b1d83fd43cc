"""B200 kernels behind the reference's kernel-level Python API.

Same names, signatures, conventions and errors as
``src/iris_metal/kernels.py``:

- ``qk_norm_rope`` (``kernels.py:334-397``), ``rms_norm_modulate``
  (``:413-452``), ``gated_residual_rms_norm_`` (``:455-480``, in place),
  ``pixel_rms_norm`` (``:486-498``), ``pixel_mlp_`` (``:527-584``, in place);
- gains, rotary tables and modulation rows must be contiguous FP32 (a BF16
  gain would be misread silently, ``kernels.py:304-306``); modulation rows may
  be strided ``[B, 1, D]`` views and are copied only if misaligned
  (``_per_batch``, ``kernels.py:404-410``);
- arguments are validated before any launch and rejected with ``ValueError``.

The work runs in ``libiris_b200.so`` on the current CUDA stream; there is no
CPU path, so CPU tensors are rejected too. Further entry points used by the
engine (``gemm``, ``flash_attention``, ...) follow the same rules.
"""

from __future__ import annotations

import ctypes
import math

import torch

from iris_b200 import _lib

HEAD_DIM = 128
PIXEL_WIDTH, PIXEL_HIDDEN = 16, 64

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _require(condition: bool, message: str) -> None:
    if not condition:
        raise ValueError(message)


def _require_fp32(**tensors: torch.Tensor) -> None:
    for name, tensor in tensors.items():
        _require(tensor.dtype == torch.float32 and tensor.is_contiguous(), f"{name} must be contiguous FP32")


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        _require(t.device.type == "cuda", "the B200 kernels need CUDA tensors (there is no CPU path)")


def _dtype(t: torch.Tensor | torch.dtype) -> int:
    dt = t if isinstance(t, torch.dtype) else t.dtype
    _require(dt in _DTYPES, f"unsupported dtype {dt}")
    return _DTYPES[dt]


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _per_batch(vector: torch.Tensor, batch: int, width: int) -> tuple[torch.Tensor, int]:
    """``[B, 1, D]`` modulation slice -> FP32 ``[B, D]`` rows, read in place when
    possible, and the element stride between them (``kernels.py:404-410``)."""
    rows = vector.reshape(batch, width).float()
    if rows.stride(1) != 1 or rows.stride(0) % 4 or rows.storage_offset() % 4:
        rows = rows.clone(memory_format=torch.contiguous_format)  # 16-byte vector loads
    return rows, rows.stride(0)


# ---------------------------------------------------------------- reference API
def qk_norm_rope(
    x: torch.Tensor,
    weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float,
    heads: int,
    col_offset: int = 0,
    out: torch.Tensor | None = None,
    offset: int = 0,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Fused per-head RMSNorm + RoPE + ``[B, N, H, D] -> [B, H, N, D]`` layout.

    ``x``: contiguous ``[B, N, W]`` projection whose columns
    ``[col_offset, col_offset + heads*128)`` hold the heads. ``cos``/``sin``: FP32
    ``[N_out, 64]``. With ``out`` (``[B, heads, N_out, 128]``) rows are written from
    token ``offset`` on. The result has ``out_dtype`` (default: the input dtype).
    """
    _require(heads > 0 and col_offset >= 0 and offset >= 0, "heads must be positive and offsets nonnegative")
    batch, tokens, width = x.shape
    _require(
        col_offset + heads * HEAD_DIM <= width and x.is_contiguous(),
        "qk_norm_rope needs a contiguous [B, N, W] input holding the heads",
    )
    if out is None:
        _require_cuda(x)
        out = x.new_empty(batch, heads, tokens, HEAD_DIM, dtype=out_dtype or x.dtype)
    _require(
        out.shape[:2] == (batch, heads) and out.shape[3] == HEAD_DIM and out.is_contiguous(),
        f"qk_norm_rope output must be a contiguous [{batch}, {heads}, N, {HEAD_DIM}] tensor",
    )
    _require(
        cos.shape == sin.shape == (cos.shape[0], HEAD_DIM // 2) and offset + tokens <= min(cos.shape[0], out.shape[2]),
        "qk_norm_rope rotary tables or output do not cover the written rows",
    )
    _require_fp32(weight=weight, cos=cos, sin=sin)
    _require(weight.numel() == HEAD_DIM, f"qk_norm_rope gain must have {HEAD_DIM} entries")
    _require_cuda(x, weight, cos, sin, out)
    _lib.call(
        "iris_qk_norm_rope", x.data_ptr(), _dtype(x), batch, tokens, width, col_offset, heads, weight.data_ptr(),
        cos.data_ptr(), sin.data_ptr(), float(eps), out.data_ptr(), _dtype(out), out.shape[2], offset, stream_of(x),
    )  # fmt: skip
    return out


def rms_norm_modulate(
    x: torch.Tensor,
    weight: torch.Tensor,
    shift: torch.Tensor,
    scale: torch.Tensor,
    eps: float,
    out_dtype: torch.dtype,
) -> torch.Tensor:
    """``(rms_norm(x) * weight * (1 + scale) + shift).to(out_dtype)`` for ``x``: ``[B, N, D]``
    and per-sample ``shift``/``scale``: ``[B, 1, D]``."""
    batch, tokens, width = x.shape
    _require(width % 128 == 0 and x.is_contiguous(), "rms_norm_modulate needs a contiguous input, width % 128 == 0")
    _require_fp32(weight=weight)
    _require(weight.numel() == width, "rms_norm_modulate gain width mismatch")
    _require(x.dtype in (torch.float32, torch.bfloat16), "rms_norm_modulate reads FP32 or BF16 rows")
    _require_cuda(x, weight, shift, scale)
    out = torch.empty(x.shape, device=x.device, dtype=out_dtype)
    shift, shift_stride = _per_batch(shift, batch, width)
    scale, scale_stride = _per_batch(scale, batch, width)
    if shift_stride != scale_stride:  # the kernel takes one stride
        shift, scale = shift.contiguous(), scale.contiguous()
        shift_stride = width
    rows = batch * tokens
    _lib.call(
        "iris_rms_norm_modulate", x.data_ptr(), _dtype(x), max(rows, 1), 0, 0, out.data_ptr(), _dtype(out_dtype),
        weight.data_ptr(), shift.data_ptr(), scale.data_ptr(), shift_stride, rows, max(tokens, 1), width, float(eps),
        stream_of(x),
    )  # fmt: skip
    return out


def gated_residual_rms_norm_(
    residual: torch.Tensor, branch: torch.Tensor, weight: torch.Tensor, gate: torch.Tensor, eps: float
) -> torch.Tensor:
    """``residual += gate * rms_norm(branch) * weight`` in place; ``residual``: FP32 ``[B, N, D]``."""
    batch, tokens, width = residual.shape
    _require(width % 128 == 0 and branch.shape == residual.shape, "gated_residual_rms_norm_ shape mismatch")
    _require(branch.is_contiguous(), "gated_residual_rms_norm_ needs a contiguous branch")
    _require_fp32(residual=residual, weight=weight)
    _require(weight.numel() == width, "gated_residual_rms_norm_ gain width mismatch")
    _require_cuda(residual, branch, weight, gate)
    gate, gate_stride = _per_batch(gate, batch, width)
    rows = batch * tokens
    _lib.call(
        "iris_gated_residual_rms_norm", residual.data_ptr(), max(rows, 1), 0, 0, branch.data_ptr(), _dtype(branch),
        max(rows, 1), 0, 0, weight.data_ptr(), gate.data_ptr(), gate_stride, rows, max(tokens, 1), width, float(eps),
        _lib.NEXT_NONE, None, None, None, 0, None, _lib.BF16, 1, 0, 0, stream_of(residual),
    )  # fmt: skip
    return residual


def pixel_rms_norm(pixels: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``rms_norm(pixels) * weight`` over the 16 channels of each pixel (BF16 out)."""
    _require(pixels.shape[-1] == PIXEL_WIDTH and pixels.is_contiguous(), "pixel_rms_norm needs 16-wide pixels")
    _require(pixels.dtype in (torch.bfloat16, torch.float32), "pixel_rms_norm reads BF16 or FP32 pixels")
    _require_fp32(weight=weight)
    _require(weight.numel() == PIXEL_WIDTH, "pixel_rms_norm gain width mismatch")
    _require_cuda(pixels, weight)
    out = torch.empty(pixels.shape, device=pixels.device, dtype=torch.bfloat16)
    n_pixels = pixels.numel() // PIXEL_WIDTH
    _lib.call(
        "iris_pixel_rms_norm", pixels.data_ptr(), _dtype(pixels), out.data_ptr(), weight.data_ptr(), n_pixels,
        float(eps), stream_of(pixels),
    )  # fmt: skip
    return out


def _mlp_params(fc1, fc2) -> tuple[torch.Tensor, ...]:
    _require(
        fc1.weight.shape == (PIXEL_HIDDEN, PIXEL_WIDTH)
        and fc2.weight.shape == (PIXEL_WIDTH, PIXEL_HIDDEN)
        and fc1.bias is not None
        and fc1.bias.shape == (PIXEL_HIDDEN,)
        and fc2.bias is not None
        and fc2.bias.shape == (PIXEL_WIDTH,),
        "pixel_mlp_ needs the released pixel-stage widths",
    )
    params = (fc1.weight, fc1.bias, fc2.weight, fc2.bias)
    _require(
        all(t.dtype == torch.bfloat16 and t.is_contiguous() for t in params),
        "pixel_mlp_ needs contiguous BF16 activations and MLP parameters",
    )
    return params


def pixel_mlp_(
    pixels: torch.Tensor,
    branch: torch.Tensor,
    mods: torch.Tensor,
    norm_weight: torch.Tensor,
    fc1,
    fc2,
    next_norm_weight: torch.Tensor,
    eps: float,
) -> torch.Tensor:
    """Finish a post-modulated PiT block in place; return the next block's normed input.

    ``pixels``/``branch``: BF16 ``[..., 16]`` (stream, attention branch); ``mods``:
    BF16 ``[..., 64]`` per pixel (scale1, shift1, scale2, shift2). An FP32 ``pixels``
    stream is also accepted and kept unrounded.
    """
    _require(
        pixels.shape[-1] == PIXEL_WIDTH
        and branch.shape == pixels.shape
        and mods.shape == (*pixels.shape[:-1], 4 * PIXEL_WIDTH),
        "pixel_mlp_ needs the released pixel-stage widths",
    )
    w1, b1, w2, b2 = _mlp_params(fc1, fc2)
    _require(
        pixels.dtype in (torch.bfloat16, torch.float32)
        and all(t.dtype == torch.bfloat16 and t.is_contiguous() for t in (branch, mods))
        and pixels.is_contiguous(),
        "pixel_mlp_ needs contiguous BF16 activations and MLP parameters",
    )
    _require_fp32(norm_weight=norm_weight, next_norm_weight=next_norm_weight)
    _require(norm_weight.numel() == next_norm_weight.numel() == PIXEL_WIDTH, "pixel_mlp_ gain width mismatch")
    _require_cuda(pixels, branch, mods, norm_weight, next_norm_weight, w1)
    next_input = torch.empty(pixels.shape, device=pixels.device, dtype=torch.bfloat16)
    n_pixels = pixels.numel() // PIXEL_WIDTH
    _lib.call(
        "iris_pixel_mlp", pixels.data_ptr(), _dtype(pixels), branch.data_ptr(), mods.data_ptr(), norm_weight.data_ptr(),
        w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(), next_norm_weight.data_ptr(), next_input.data_ptr(),
        n_pixels, float(eps), stream_of(pixels),
    )  # fmt: skip
    return next_input


# ----------------------------------------------------------- engine entry points
def gemm_problem(
    a: torch.Tensor,
    w: torch.Tensor,
    out: torch.Tensor | None,
    *,
    bias: torch.Tensor | None = None,
    epilogue: int = _lib.EPI_STORE,
    aux: torch.Tensor | None = None,
    out_rows: tuple[int, int, int] | None = None,
    aux_rows: tuple[int, int, int] | None = None,
    heads: "HeadsOut | None" = None,
) -> "_lib.GemmProblem":
    """Validate one ``out = epilogue(a @ w.T)`` and describe it for the library:
    ``a``: bf16 ``[M, K]`` (row stride may exceed K), ``w``: bf16 ``[N, K]``;
    ``out`` rows through the row map ``(seg_rows, seg_stride, seg_offset)``.
    With ``heads`` (:class:`HeadsOut`) the epilogue is ``EPI_HEADS`` and ``out``
    is unused: the ``[q | k | v]`` columns go normed and rotated to the head
    tensors, row ``m`` being token position ``map(m) % tokens``."""
    _require(a.dim() == 2 and w.dim() == 2 and a.dtype == w.dtype == torch.bfloat16, "gemm needs bf16 [M, K] x [N, K]")
    _require(a.stride(1) == 1 and w.stride(1) == 1, "gemm operands must be row-major")
    M, K = a.shape
    N = w.shape[0]
    _require(w.shape[1] == K, "gemm: inner dimensions differ")
    if bias is not None:
        _require_fp32(bias=bias)
        _require(bias.numel() == N, "gemm: bias width")
    out_rows = out_rows or (M, 0, 0)
    aux_rows = aux_rows or (M, 0, 0)
    if heads is not None:
        _require_cuda(a, w)
        problem = _lib.GemmProblem(
            a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), None, _lib.BF16, 0, M, N, K, _lib.EPI_HEADS, None,
            None, 0, *out_rows, *aux_rows, ctypes.pointer(heads.struct),
        )  # fmt: skip
        problem._keep = heads  # the struct must outlive the launch call
        return problem
    _require(out.stride(-1) == 1, "gemm operands must be row-major")
    _require_cuda(a, w, out)
    return _lib.GemmProblem(
        a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), _dtype(out),
        out.stride(-2) if out.dim() >= 2 else N, M, N, K, epilogue, _ptr(bias), _ptr(aux),
        aux.stride(-2) if aux is not None else 0, *out_rows, *aux_rows, None,
    )  # fmt: skip


class HeadsOut:
    """Targets of the ``EPI_HEADS`` GEMM epilogue (``iris_heads_epilogue``):
    ``q`` / ``k`` / ``v`` bf16 head tensors holding ``[B, H, n, 128]`` (or
    ``[H, B, n, 128]`` with ``head_major``) of ``hq`` / ``hkv`` heads, the q / k
    gains (FP32 ``[128]``), rotary tables (FP32 ``[tokens, 64]``, row = token
    position), ``tokens`` positions per sample."""

    def __init__(self, q, k, v, q_weight, k_weight, cos, sin, eps, hq, hkv, tokens, batch, n_out, n_out_kv,
                 head_major=False, peers=None):  # fmt: skip
        _require_fp32(q_weight=q_weight, cos=cos, sin=sin)
        _require(q_weight.numel() == HEAD_DIM and (k_weight is None or k_weight.numel() == HEAD_DIM),
                 "heads epilogue gains must have 128 entries")  # fmt: skip
        _require(cos.shape == sin.shape and cos.shape[-1] == HEAD_DIM // 2 and cos.shape[0] >= tokens,
                 "heads epilogue rotary tables must cover the token positions")  # fmt: skip
        _require(all(t is None or t.dtype == torch.bfloat16 for t in (q, k, v)), "heads epilogue writes bf16")
        mode = _lib.HEADS_LOCAL if peers is None else peers.mode
        local_q, local_kv = mode != _lib.HEADS_PEER_SCATTER, mode == _lib.HEADS_LOCAL
        _require(not local_q or q.numel() >= batch * hq * n_out * HEAD_DIM, "heads epilogue q output is too small")
        _require(not local_kv or hkv == 0 or min(k.numel(), v.numel()) >= batch * hkv * n_out_kv * HEAD_DIM,
                 "heads epilogue k / v outputs are too small")  # fmt: skip
        _require_cuda(*(t for t in (q, k, v, q_weight, k_weight, cos, sin) if t is not None))
        self._tensors = (q, k, v, q_weight, k_weight, cos, sin)
        self.struct = _lib.HeadsEpilogue(
            _ptr(q), _ptr(k), _ptr(v), q_weight.data_ptr(), _ptr(k_weight), cos.data_ptr(), sin.data_ptr(),
            float(eps), int(bool(head_major)), hq, hkv, tokens, batch, n_out, n_out_kv,
        )  # fmt: skip
        if peers is not None:
            peers.fill(self.struct)


class PeerHeads:
    """Sequence-parallel destinations of the ``EPI_HEADS`` epilogue: ``mode``
    ``_lib.HEADS_PEER_SCATTER`` (head ``h`` of q / k / v to rank
    ``h // (heads / world)``) or ``_lib.HEADS_PEER_BROADCAST_KV`` (k and v to
    every rank, q local); per rank ``j`` the device pointers (valid in this
    process) of its ``[B, heads', n_dest, 128]`` q / k / v buffers; this rank's
    tokens land at positions ``token_offset + t``."""

    def __init__(self, mode: int, q_ptrs, k_ptrs, v_ptrs, token_offset: int, n_dest: int):
        world = len(k_ptrs)
        _require(1 <= world <= _lib.MAX_PEERS and len(v_ptrs) == world, "peer heads: 1 to 8 ranks")
        _require(mode != _lib.HEADS_PEER_SCATTER or len(q_ptrs) == world, "peer heads: q pointers per rank")
        self.mode, self.world = mode, world
        self.q, self.k, self.v = list(q_ptrs or [0] * world), list(k_ptrs), list(v_ptrs)
        self.token_offset, self.n_dest = token_offset, n_dest

    def fill(self, st) -> None:
        st.peer_mode, st.world, st.token_offset, st.n_dest = self.mode, self.world, self.token_offset, self.n_dest
        for j in range(self.world):
            st.q_peer[j], st.k_peer[j], st.v_peer[j] = self.q[j] or None, self.k[j], self.v[j]


def gemm_grouped(problems: list, stream: int) -> None:
    """Run 1 to 4 problems from :func:`gemm_problem` in one persistent launch."""
    _require(1 <= len(problems) <= 4, "gemm_grouped takes 1 to 4 problems")
    array = (_lib.GemmProblem * len(problems))(*problems)
    timing = _gemm_profile is not None
    if timing:
        # inside a CUDA-graph capture the events become record nodes of the graph
        captured = torch.cuda.is_current_stream_capturing()
        start = torch.cuda.Event(enable_timing=True, external=captured)
        end = torch.cuda.Event(enable_timing=True, external=captured)
        start.record()
    _lib.call("iris_gemm_bf16_grouped", array, len(problems), stream)
    if timing:
        end.record()
        _gemm_profile.append((start, end, sum(2.0 * q.M * q.N * q.K for q in problems),
                              sum(_gemm_bytes(q) for q in problems), captured))  # fmt: skip
        if captured:  # the graph's record nodes address these events for as long as the graph lives
            _graph_events.append((start, end))


def _gemm_bytes(q) -> float:
    """Algorithmic HBM bytes of one problem: A and W read once, the output
    (and a gate's aux rows) once."""
    cols = q.N // 2 if q.epilogue == _lib.EPI_SWIGLU else q.N
    out = q.M * cols * (4 if q.out_dtype == _lib.F32 else 2)
    aux = q.M * q.N * 2 if q.epilogue == _lib.EPI_GATE else 0
    return 2.0 * (q.M + q.N) * q.K + out + aux + (4 * q.N if q.bias else 0)


def gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, **kwargs) -> torch.Tensor:
    """``out = epilogue(a @ w.T)`` on the tensor cores (see :func:`gemm_problem`)."""
    gemm_grouped([gemm_problem(a, w, out, **kwargs)], stream_of(a))
    return out


_gemm_profile: list | None = None
# events recorded by nodes of captured CUDA graphs: kept for the life of the process,
# since a graph replay records them again whether or not timing is still on
_graph_events: list = []


def profile_gemms(enable: bool):
    """Start (``True``) or stop (``False``) timing every GEMM launch with CUDA
    events on its stream. Stopping synchronises and returns
    ``(algorithmic FLOPs, milliseconds, launches, algorithmic bytes)`` summed
    over the launches. GEMMs captured into a CUDA graph while timing is on carry
    event-record nodes, which every replay records again: their times are those
    of the latest replay, and when there are any, only they are summed (the
    eager forward that precedes a capture is left out)."""
    global _gemm_profile
    if enable:
        _gemm_profile = []
        return None
    records, _gemm_profile = _gemm_profile or [], None
    torch.cuda.synchronize()
    use = [r for r in records if r[4]] or records
    flops = sum(r[2] for r in use)
    ms = sum(r[0].elapsed_time(r[1]) for r in use)
    return flops, ms, len(use), sum(r[3] for r in use)


def score_bound(q_gains, k_gains, scale: float | None = None, head_dim: int = 128) -> float:
    """An upper bound on ``|q . k| * scale`` for RMS-normed (QK-norm) heads:
    an RMS-normed row has norm at most ``sqrt(head_dim)`` before its gain, and
    RoPE is a rotation, so ``|q . k| <= head_dim * max|q gain| * max|k gain|``
    (Cauchy-Schwarz). 2% slack covers the bf16 rounding of q and k. Every
    stream's gains of a joint attention go into one bound."""
    gq = max(float(g.abs().max()) for g in q_gains)
    gk = max(float(g.abs().max()) for g in k_gains)
    scale = head_dim**-0.5 if scale is None else scale
    bound = 1.02 * head_dim * gq * gk * scale
    return bound if math.isfinite(bound) else 0.0  # 0: no bound, every block runs the row-max pass


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, scale: float | None = None,
                    bound: float = 0.0):  # fmt: skip
    """``softmax(q k^T * scale) v`` for ``q``: ``[B, H, N, 128]``, ``k``/``v``:
    ``[B, H_kv, N_kv, 128]`` (bf16, contiguous; ``N_kv`` may differ from ``N``);
    ``out``: ``[B, N, >= H*128]`` bf16. ``bound``: 0 or :func:`score_bound` of
    the heads' QK-norm gains (rows then skip the row-max pass once settled)."""
    _check_qkv(q, k, v)
    batch, heads, n, d = q.shape
    _require(out.dtype == torch.bfloat16 and out.stride(-1) == 1 and out.shape[-2] == n, "flash_attention: out layout")
    _require(out.dim() == 3 and out.stride(0) == n * out.stride(1), "flash_attention: out rows must be [B*N, stride]")
    _require_cuda(q, k, v, out)
    _lib.call(
        "iris_flash_attn_fwd_split", q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, k.shape[1], n,
        k.shape[2], d, float(scale if scale is not None else d**-0.5), float(bound), 0, None, out.data_ptr(), None,
        None, out.stride(1), stream_of(q),
    )  # fmt: skip
    return out


def flash_attention_peers(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out_ptrs, tokens_per_rank: int,
                          col0: int, row_stride: int, scale: float | None = None, bound: float = 0.0) -> None:  # fmt: skip
    """Sequence-parallel attention of this rank's heads over every token: the
    output row of query ``i`` (bf16, ``q.shape[1] * 128`` columns from ``col0``)
    goes to rank ``i // tokens_per_rank``'s token rows ``out_ptrs[j]`` (device
    pointers valid in this process), row ``b * tokens_per_rank + i %
    tokens_per_rank`` of ``row_stride`` elements."""
    _check_qkv(q, k, v)
    batch, heads, n, d = q.shape
    world = len(out_ptrs)
    _require(1 <= world <= _lib.MAX_PEERS and n == world * tokens_per_rank, "flash_attention_peers: n = world * tokens")
    _require_cuda(q, k, v)
    ptrs = (ctypes.c_void_p * world)(*out_ptrs)
    _lib.call(
        "iris_flash_attn_fwd_peers", q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, k.shape[1], n,
        k.shape[2], d, float(scale if scale is not None else d**-0.5), float(bound), ptrs, world, tokens_per_rank, col0,
        row_stride, stream_of(q),
    )  # fmt: skip


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(IPC handle, byte offset) of the allocation holding ``t``'s storage."""
    _require_cuda(t)
    handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    offset = ctypes.c_int64(0)
    _lib.call("iris_ipc_export", t.data_ptr(), handle, ctypes.byref(offset))
    return handle.raw, int(offset.value)


def ipc_import(handle: bytes) -> int:
    """Map another process's allocation; returns its base device pointer."""
    _require(len(handle) == _lib.IPC_HANDLE_BYTES, "ipc_import: bad handle")
    base = ctypes.c_void_p(0)
    _lib.call("iris_ipc_import", ctypes.create_string_buffer(handle, len(handle)), ctypes.byref(base))
    return int(base.value)


def ipc_close(base: int) -> None:
    _lib.call("iris_ipc_close", base)


def peer_barrier(flags: torch.Tensor, peer_flag_ptrs, rank: int, epoch: int, timeout_s: float = 2.0) -> None:
    """Signal the ranks (slot ``rank`` of each peer's flags) and wait for theirs in
    ``flags`` (int32 ``[world]`` of this rank), on the current stream."""
    world = len(peer_flag_ptrs)
    _require(flags.dtype == torch.int32 and flags.numel() >= world, "peer_barrier: flags must be int32 [world]")
    ptrs = (ctypes.c_void_p * world)(*[p or None for p in peer_flag_ptrs])
    _lib.call("iris_peer_barrier", flags.data_ptr(), ptrs, rank, world, epoch & 0xFFFFFFFF, int(timeout_s * 1e9),
              stream_of(flags))  # fmt: skip


def _check_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    _require(q.dim() == 4 and k.shape == v.shape and q.shape[0] == k.shape[0] and q.shape[3] == k.shape[3],
             "flash_attention: q [B, H, N, D], k/v [B, H_kv, N_kv, D]")  # fmt: skip
    _require(all(t.dtype == torch.bfloat16 and t.is_contiguous() for t in (q, k, v)), "flash_attention: contiguous bf16")


def flash_attention_split(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    split: int,
    o_text: torch.Tensor | None,
    o_image: torch.Tensor,
    gate_text: torch.Tensor | None = None,
    gate_image: torch.Tensor | None = None,
    scale: float | None = None,
    bound: float = 0.0,
) -> None:
    """Attention whose token ``i < split`` rows land densely in ``o_text`` (row
    ``b * split + i``) and the rest in ``o_image`` (row ``b * (N - split) + i - split``),
    each multiplied by ``sigmoid`` of the bf16 gate logits in the same rows."""
    _check_qkv(q, k, v)
    batch, heads, n, d = q.shape
    outs = [t for t in (o_text, o_image, gate_text, gate_image) if t is not None]
    _require(all(t.dtype == torch.bfloat16 and t.stride(-1) == 1 for t in outs), "flash_attention: bf16 row-major outputs")
    stride = o_image.stride(-2)
    _require(all(t.stride(-2) == stride for t in outs), "flash_attention: outputs and gates share one row stride")
    _require_cuda(q, k, v, *outs)
    _lib.call(
        "iris_flash_attn_fwd_split", q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, k.shape[1], n,
        k.shape[2], d, float(scale if scale is not None else d**-0.5), float(bound), split, _ptr(o_text),
        o_image.data_ptr(), _ptr(gate_text), _ptr(gate_image), stride, stream_of(q),
    )  # fmt: skip


def block_copy(
    dst: torch.Tensor,
    dst_strides: tuple[int, int, int],
    src: torch.Tensor,
    src_strides: tuple[int, int, int],
    counts: tuple[int, int, int],
    block_bytes: int,
    dst_offset: int = 0,
    src_offset: int = 0,
) -> None:
    """``counts[0] x counts[1] x counts[2]`` blocks of ``block_bytes`` from
    ``src`` to ``dst``; strides and offsets in bytes (multiples of 16)."""
    _require_cuda(dst, src)
    _require(dst.device == src.device, "block_copy: one device")
    for name, t, off, strides in (("dst", dst, dst_offset, dst_strides), ("src", src, src_offset, src_strides)):
        span = off + sum((c - 1) * st for c, st in zip(counts, strides) if c > 0) + block_bytes
        _require(min(counts) == 0 or span <= t.numel() * t.element_size(), f"block_copy: {name} range out of bounds")
    _lib.call(
        "iris_block_copy", dst.data_ptr() + dst_offset, *dst_strides, src.data_ptr() + src_offset, *src_strides,
        *counts, block_bytes, stream_of(dst),
    )  # fmt: skip


def device_error(clear: bool = True, device: torch.device | None = None) -> int:
    """The device error word (bit 0: a bounded wait timed out); synchronises the stream."""
    import ctypes

    value = ctypes.c_uint(0)
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.call("iris_device_error", int(clear), ctypes.byref(value), stream)
    return int(value.value)
