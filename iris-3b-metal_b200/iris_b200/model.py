"""``CudaIris``: the per-step Iris-3B denoiser forward on B200 kernels.

Drop-in for ``MetalIris`` (``src/iris_metal/model.py:113-345``): same
constructor (a loaded model exposing ``.cfg`` and ``.state_dict()`` -- the
upstream ``IrisDiT`` or :class:`iris_b200.weights.IrisWeights`), same
``encode_text`` and ``__call__(x, t, text) -> v`` contract. ``text`` is never
written, the host is never synchronised, outputs are allocated fresh and the
residual streams are internal workspace. Every launch goes to
``libiris_b200.so``.

Per step (``dit.py:283-375`` restructured):

* conditioning: timestep features -> MLP -> silu -> both shared adaLN cores,
  once per step; per-block modulation rows = core + block bias in one launch;
* residual stream: one FP32 ``[B, T + L, D]`` buffer, text rows first. The
  dual-stream blocks address its text and image rows through row maps, so the
  single-stream tail needs no concatenation;
* every branch input is written by the kernel that finishes the previous
  residual update (gated post-norm + residual + next RMSNorm-modulate fused);
* GEMMs on the tensor cores with fused epilogues (bias, SwiGLU, sigmoid gate),
  attention by the tcgen05 flash kernel; the Q/K/V GEMM's epilogue applies
  the QK-norm and RoPE and writes the head layout directly;
* pixel stage: per-pixel adaLN GEMM, compress / attention / expand on the
  tensor cores, the post-modulated per-pixel MLP fused, and the last block
  fused with the FinalLayer and the fold into the velocity image.

Precision plan: BF16 GEMM operands and attention, FP32 accumulation, FP32
residual streams, norms, modulation and conditioning, FP32 pixel stream
(the reference keeps BF16 there; FP32 is closer to the fp32 model).

With a communicator (``comm``, see :mod:`iris_b200.ulysses`) one call is
spread over its ranks by sequence parallelism: each rank runs the step on its
slice of the joint sequence and every rank returns the whole velocity.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from iris_b200 import _lib
from iris_b200 import kernels as K
from iris_b200.adapter import TextAdapter
from iris_b200.config import ModelConfig, from_any
from iris_b200.tables import cos_sin, rope_1d, rope_2d, sincos_pos_embed_2d
from iris_b200.ulysses import PeerBuffers, SequenceShard, gather_image_tokens, gather_tokens, scatter_heads

HEAD_DIM = 128
SWIGLU_TILE = 128  # w1/w3 rows per SwiGLU GEMM tile half


def check_supported(cfg: ModelConfig, state: dict) -> None:
    """Reject topologies the fused forward does not handle (``model.py:68-99``)."""
    requirements = {
        "a pixel stage with post-modulated blocks of 16 channels": cfg.pixel.enabled
        and cfg.pixel.modulation == "post"
        and cfg.pixel.hidden_size == 16
        and cfg.pixel.mlp_ratio == 4.0,
        "shared_bias modulation": cfg.modulation == "shared_bias",
        "a single-stream tail after the dual-stream prefix": cfg.block == "single_stream" and cfg.depth > cfg.dual_depth,
        "gated, sandwich-normed, QK-normed attention without QKV bias": cfg.gated_attention
        and cfg.sandwich_norm
        and cfg.qk_norm
        and not cfg.qkv_bias,
        f"{HEAD_DIM}-wide attention heads": cfg.hidden_size // cfg.num_heads == HEAD_DIM
        and cfg.pixel.attn_hidden_size // cfg.pixel.num_heads == HEAD_DIM
        and cfg.num_heads % cfg.kv_heads == 0,
        "text RoPE without frame pairs": cfg.text_rope and cfg.rope_frame_pairs == 0,
        "text output kept in the final block": cfg.final_block_text == "keep",
        "a hidden size that is a multiple of 128": cfg.hidden_size % 128 == 0,
    }
    missing = [name for name, ok in requirements.items() if not ok]
    if missing:
        raise ValueError(f"CudaIris supports the released Iris-3B topology family; this model lacks {missing}")
    for key in ("s_embedder.proj.weight", "t_embedder.mlp.0.weight", "final_layer.linear.weight"):
        if key not in state:
            raise ValueError(f"CudaIris: missing parameter {key}")


def pack_swiglu(w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, tile: int = SWIGLU_TILE):
    """SwiGLU weights (``src/iris3b/nn/mlp.py:24-40``) in the layout of the GEMM's
    SwiGLU epilogue: each 256-row tile of ``w13`` holds ``tile`` rows of ``w1``
    followed by the same rows of ``w3``; the hidden width is zero-padded to a
    multiple of ``tile`` (``silu(0) * 0 = 0`` and the padded ``w2`` columns are 0)."""
    ffn, d = w1.shape
    pad = -(-ffn // tile) * tile
    tiles = pad // tile
    w1p = torch.zeros(pad, d, device=w1.device, dtype=w1.dtype)
    w3p = torch.zeros(pad, d, device=w3.device, dtype=w3.dtype)
    w1p[:ffn], w3p[:ffn] = w1, w3
    w13 = torch.stack([w1p.view(tiles, tile, d), w3p.view(tiles, tile, d)], dim=1)  # [tiles, 2, tile, d]
    w2p = torch.zeros(w2.shape[0], pad, device=w2.device, dtype=w2.dtype)
    w2p[:, :ffn] = w2
    return w13.reshape(2 * pad, d).contiguous(), w2p


ERR_WAIT_TIMEOUT = 1  # bit of the device error word: a kernel's bounded wait gave up


class DeviceWaitTimeout(RuntimeError):
    """A bounded wait on the device gave up: a sequence-parallel peer did not
    reach a barrier in time, or a tensor-core pipeline stage never completed.
    Buffers the result depends on may be stale, so the result is rejected."""


def require_finite(result: torch.Tensor) -> torch.Tensor:
    """Raise rather than let an overflowed result become a black image
    (``src/iris_metal/model.py:102-110``); one device flag, one sync. The same
    sync reads the device error word: a result computed after a timed-out
    bounded wait raises :class:`DeviceWaitTimeout` (the engine has also filled
    it with NaN, so callers that only test finiteness reject it too)."""
    flag = torch.empty(1, device=result.device, dtype=torch.int32)
    data = result.float().contiguous()
    _lib.call("iris_all_finite", data.data_ptr(), data.numel(), flag.data_ptr(), K.stream_of(data))
    finite = int(flag.item()) == 1
    if K.device_error(clear=False, device=result.device) & ERR_WAIT_TIMEOUT:
        K.device_error(clear=True, device=result.device)
        raise DeviceWaitTimeout(
            "a bounded wait on the device timed out (a sequence-parallel rank stopped answering, or a kernel "
            "pipeline stalled); the result was discarded"
        )
    if not finite:
        raise FloatingPointError("the model produced non-finite values; please report the input and settings")
    return result


@dataclass
class _Block:
    dual: bool
    norms: dict
    qkv: dict  # stream -> bf16 [(H + 2 Hkv) 128, D]
    qk_norm: dict  # stream -> (q gain, k gain)
    gate: dict
    proj: dict  # stream -> (weight, bias)
    w13: dict
    w2: dict
    mod_index: dict  # stream -> row in the stacked modulation table
    score_bound: float = field(init=False)  # of |q . k| * scale, from the QK-norm gains of every stream

    def __post_init__(self):
        self.score_bound = K.score_bound(*zip(*self.qk_norm.values()))


class CudaIris:
    """Velocity predictor ``(x, t, text) -> v`` for a loaded Iris model."""

    def __init__(
        self,
        dit,
        attention_dtype: torch.dtype | None = None,
        pixel_dtype: torch.dtype = torch.float32,
        comm=None,
        graphs: bool = False,
    ):
        """``graphs=True``: every call of a one-GPU engine replays a CUDA graph of
        the whole forward, captured at the first call of each input geometry (that
        first call runs the forward once eagerly, captures it, and synchronises the
        host once; later calls of the geometry copy the inputs into the graph's
        buffers, replay it and return a fresh copy of its output). The kernels are
        the same; the graph removes the host's per-kernel launch cost (a B = 2 call
        at 1024^2: 62.2 ms eager, 61.9 ms replayed). Sequence-parallel engines
        (``comm``) always run eagerly: their barriers count epochs on the host."""
        cfg = from_any(dit.cfg)
        state = dit.state_dict()
        check_supported(cfg, state)
        if attention_dtype not in (None, torch.bfloat16):
            raise ValueError("CudaIris computes attention in BF16")
        if pixel_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("pixel_dtype must be torch.float32 or torch.bfloat16")
        self.dit = dit
        self.cfg = cfg
        self.device = state["s_embedder.proj.weight"].device
        if self.device.type != "cuda":
            raise ValueError("CudaIris needs the model's weights on a CUDA device")
        self.dtype = torch.bfloat16
        self.attention_dtype = torch.bfloat16
        self.pixel_dtype = pixel_dtype
        self.text_dtype = torch.bfloat16
        self.comm = comm if comm is not None and comm.world > 1 else None
        if self.comm is not None:
            world = self.comm.world
            if cfg.num_heads % world or cfg.kv_heads % world:
                raise ValueError(f"sequence parallelism over {world} ranks needs the trunk's query and key/value "
                                 f"head counts ({cfg.num_heads}, {cfg.kv_heads}) divisible by {world}")  # fmt: skip
            if world > _lib.MAX_PEERS:
                raise ValueError(f"sequence parallelism spans at most {_lib.MAX_PEERS} ranks")
        # one process per GPU: the exchanges are the producing kernels' stores into peer memory
        self.peer = self.comm is not None and bool(getattr(self.comm, "peer_capable", False))
        self.peer_timeout_s = 2.0
        self._epoch = 0
        self._pack(state)
        self._tables: dict = {}
        self._work: dict = {}
        self.graphs = bool(graphs) and self.comm is None
        self._graphs: dict = {}

    # -- weight repacking (once) --------------------------------------------------
    def _pack(self, state: dict) -> None:
        cfg, dev = self.cfg, self.device
        d = cfg.hidden_size
        ffn = cfg.swiglu_hidden
        self.ffn_pad = -(-ffn // SWIGLU_TILE) * SWIGLU_TILE

        def bf(name):
            return state[name].detach().to(dev, torch.bfloat16).contiguous()

        def f32(name):
            return state[name].detach().to(dev, torch.float32).contiguous()

        def pad_k(w: torch.Tensor) -> torch.Tensor:
            k = w.shape[1]
            kp = -(-k // 8) * 8
            if kp == k:
                return w.contiguous()
            out = torch.zeros(w.shape[0], kp, device=dev, dtype=w.dtype)
            out[:, :k] = w
            return out

        def qkv(prefix, suffix):
            fused = f"{prefix}.qkv{suffix}.weight"
            if fused in state:
                return bf(fused)
            parts = [bf(f"{prefix}.{n}_proj{suffix}.weight") for n in ("q", "k", "v")]
            return torch.cat(parts).contiguous()

        def swiglu(prefix):
            return pack_swiglu(bf(f"{prefix}.w1.weight"), bf(f"{prefix}.w3.weight"), bf(f"{prefix}.w2.weight"))

        self.s_embed = (bf("s_embedder.proj.weight"), f32("s_embedder.proj.bias"))
        # input channels from the patch embedder: cfg.in_channels, or one more for
        # task exports with a widened embedder (src/iris3b/downstream/depth.py:30-38);
        # the velocity keeps the final layer's cfg.in_channels
        pp = cfg.patch_size**2
        self.in_channels = self.s_embed[0].shape[1] // pp
        if self.s_embed[0].shape[1] != self.in_channels * pp or not 1 <= self.in_channels <= 4:
            raise ValueError("CudaIris: s_embedder.proj takes 1 to 4 channels of patch_size^2 pixels")
        if (self.in_channels * pp) % 8:
            raise ValueError("CudaIris needs in_channels * patch_size^2 to be a multiple of 8")
        # conditioning linears in BF16 like every other trunk linear (the GEMV reads them once per step)
        self.t_mlp = [(bf(f"t_embedder.mlp.{i}.weight"), f32(f"t_embedder.mlp.{i}.bias")) for i in (0, 2)]
        self.cores = {s: (bf(f"modulation_cores.adaln_{s}.weight"), f32(f"modulation_cores.adaln_{s}.bias"))
                      for s in ("img", "txt")}  # fmt: skip
        self.blocks: list[_Block] = []
        img_bias, txt_bias = [], []
        for i in range(cfg.depth):
            b = f"blocks.{i}"
            if i < cfg.dual_depth:
                streams = {"x": "img", "y": "txt"}
                norms = {
                    s: {
                        "norm1": f32(f"{b}.norm_{s}1.weight"),
                        "norm2": f32(f"{b}.norm_{s}2.weight"),
                        "post_attn": f32(f"{b}.attn_post_norm_{s}.weight"),
                        "post_mlp": f32(f"{b}.mlp_post_norm_{s}.weight"),
                    }
                    for s in streams
                }
                w13, w2 = {}, {}
                for s in streams:
                    w13[s], w2[s] = swiglu(f"{b}.mlp_{s}")
                mod_index = {"x": len(img_bias), "y": len(txt_bias)}
                img_bias.append(f32(f"{b}.adaln_img.bias"))
                txt_bias.append(f32(f"{b}.adaln_txt.bias"))
                self.blocks.append(
                    _Block(
                        dual=True,
                        norms=norms,
                        qkv={s: qkv(f"{b}.attn", f"_{s}") for s in streams},
                        qk_norm={s: (f32(f"{b}.attn.q_norm_{s}.weight"), f32(f"{b}.attn.k_norm_{s}.weight"))
                                 for s in streams},  # fmt: skip
                        gate={s: bf(f"{b}.attn_gate_{s}.weight") for s in streams},
                        proj={s: (bf(f"{b}.attn.proj_{s}.weight"), f32(f"{b}.attn.proj_{s}.bias")) for s in streams},
                        w13=w13,
                        w2=w2,
                        mod_index=mod_index,
                    )
                )
            else:
                w13, w2 = swiglu(f"{b}.mlp")
                mod_index = {"j": len(img_bias)}
                img_bias.append(f32(f"{b}.adaln.bias"))
                self.blocks.append(
                    _Block(
                        dual=False,
                        norms={"j": {
                            "norm1": f32(f"{b}.norm1.weight"),
                            "norm2": f32(f"{b}.norm2.weight"),
                            "post_attn": f32(f"{b}.attn_post_norm.weight"),
                            "post_mlp": f32(f"{b}.mlp_post_norm.weight"),
                        }},  # fmt: skip
                        qkv={"j": qkv(b, "")},
                        qk_norm={"j": (f32(f"{b}.q_norm.weight"), f32(f"{b}.k_norm.weight"))},
                        gate={"j": bf(f"{b}.attn_gate.weight")},
                        proj={"j": (bf(f"{b}.attn_proj.weight"), f32(f"{b}.attn_proj.bias"))},
                        w13={"j": w13},
                        w2={"j": w2},
                        mod_index=mod_index,
                    )
                )
        self.img_bias = torch.stack(img_bias).contiguous()
        self.txt_bias = torch.stack(txt_bias).contiguous() if txt_bias else None
        pix = cfg.pixel
        self.pixel_embed_w = (f32("pixel_embedder.proj.weight"), f32("pixel_embedder.proj.bias"))
        if tuple(self.pixel_embed_w[0].shape) != (pix.hidden_size, self.in_channels):
            raise ValueError("CudaIris: pixel_embedder.proj must take the patch embedder's input channels")
        self.pixel_blocks = []
        for i in range(pix.depth):
            b = f"pixel_blocks.{i}"
            self.pixel_blocks.append(
                {
                    "norm1": f32(f"{b}.norm1.weight"),
                    "norm2": f32(f"{b}.norm2.weight"),
                    "adaln": (bf(f"{b}.adaln.weight"), f32(f"{b}.adaln.bias")),
                    "compress": (pad_k(bf(f"{b}.compress.weight")), f32(f"{b}.compress.bias")),
                    "qkv": bf(f"{b}.attn.qkv.weight"),
                    "qk_norm": (f32(f"{b}.attn.q_norm.weight"), f32(f"{b}.attn.k_norm.weight")),
                    "score_bound": K.score_bound([state[f"{b}.attn.q_norm.weight"]], [state[f"{b}.attn.k_norm.weight"]]),
                    "proj": (bf(f"{b}.attn.proj.weight"), f32(f"{b}.attn.proj.bias")),
                    "expand": (bf(f"{b}.expand.weight"), f32(f"{b}.expand.bias")),
                    "fc1": (bf(f"{b}.mlp.fc1.weight"), bf(f"{b}.mlp.fc1.bias")),
                    "fc2": (bf(f"{b}.mlp.fc2.weight"), bf(f"{b}.mlp.fc2.bias")),
                }
            )
        self.final = (f32("final_layer.norm.weight"), f32("final_layer.linear.weight"), f32("final_layer.linear.bias"))
        if tuple(self.final[1].shape) != (3, pix.hidden_size):
            raise ValueError("CudaIris: the final layer must emit 3 channels per pixel")
        self.text_adapter = None
        self.masked_adapter = None
        self.y_pos = f32("y_pos_embedding").reshape(-1, d) if "y_pos_embedding" in state else None
        if cfg.text_adapter == "linear" and "y_embedder.proj.weight" in state:
            self.text_adapter = (pad_k(bf("y_embedder.proj.weight")), f32("y_embedder.proj.bias"),
                                 f32("y_embedder.norm.weight"))  # fmt: skip
        elif cfg.text_adapter in ("lap_blocks2", "blocks2") and any(k.startswith("y_embedder.") for k in state):
            self.masked_adapter = TextAdapter(cfg, state, dev)

    # -- conditioning ---------------------------------------------------------------
    @torch.no_grad()
    def encode_text(self, states: torch.Tensor, mask: torch.Tensor | None = None) -> torch.Tensor:
        """Encoder states -> trunk text tokens ``[B, T, D]`` (FP32), once per prompt
        (``MetalIris.encode_text``, ``src/iris_metal/model.py:133-145``).

        Both adapter families run on this engine's kernels: the linear one
        (``TextEmbedder``: Linear + RMSNorm, then ``y_pos_embedding``,
        ``dit.py:263-281``) and the masked transformers ``lap_blocks2`` /
        ``blocks2`` over ``[B, T, layers, dim]`` / ``[B, T, dim]`` states
        (:class:`iris_b200.adapter.TextAdapter`), which need the encoder's
        ``[B, T]`` mask (nonzero = real token)."""
        cfg = self.cfg
        n = cfg.text_len
        if self.masked_adapter is not None:
            if mask is None:
                raise ValueError(f"encode_text: the {cfg.text_adapter!r} text adapter needs the encoder's [B, T] mask")
            return self.masked_adapter(states[:, :n].to(self.device, torch.float32), mask[:, :n], pos=self.y_pos)
        if self.text_adapter is None:
            raise ValueError(f"encode_text: the model has no weights for its {cfg.text_adapter!r} text adapter")
        w, b, norm_w = self.text_adapter
        states = states[:, :n].to(self.device)
        batch, n, dim = states.shape
        a = torch.zeros(batch * n, w.shape[1], device=self.device, dtype=torch.bfloat16)
        a[:, :dim] = states.reshape(batch * n, dim)
        out = torch.empty(batch, n, cfg.hidden_size, device=self.device, dtype=torch.float32)
        K.gemm(a, w, out.view(batch * n, -1), bias=b)
        pos = self.y_pos
        add = pos[:n].contiguous() if pos is not None else torch.zeros(n, cfg.hidden_size, device=self.device)
        _lib.call("iris_rms_norm_add_rows", out.data_ptr(), norm_w.data_ptr(), add.data_ptr(), batch * n, n,
                  cfg.hidden_size, float(cfg.norm_eps), K.stream_of(out))  # fmt: skip
        return out

    def _rope(self, grid: tuple[int, int], n_text: int):
        key = (grid, n_text)
        if key not in self._tables:
            cfg = self.cfg
            image = rope_2d(HEAD_DIM, *grid, cfg.rope_theta, cfg.rope_scale, cfg.rope_aspect)
            text = rope_1d(HEAD_DIM, n_text, cfg.text_rope_theta)
            trunk = cos_sin(text, image, device=self.device)
            pixel = cos_sin(image, device=self.device)  # pixel heads are 128 wide too
            pos = None
            if cfg.pixel.abs_pos_embed:
                p = cfg.patch_size
                pos = sincos_pos_embed_2d(cfg.pixel.hidden_size, grid[0] * p, grid[1] * p).to(self.device)
            if len(self._tables) >= 4:
                self._tables.pop(next(iter(self._tables)))
            self._tables[key] = (trunk, pixel, pos)
        return self._tables[key]

    def _workspace(self, batch: int, grid: tuple[int, int], shard: SequenceShard) -> dict:
        """Buffers of one geometry; token-row buffers hold this rank's rows only
        (all of them without sequence parallelism)."""
        key = (batch, grid, shard)
        if key in self._work:
            return self._work[key]
        for old in self._work.values():
            if "_peers" in old:
                old["_peers"].close()
        self._work.clear()
        cfg, dev = self.cfg, self.device
        d = cfg.hidden_size
        pp = cfg.patch_size**2
        n, L_loc = shard.n, shard.image
        hq, hkv = cfg.num_heads, cfg.kv_heads
        pix = cfg.pixel
        bf16 = torch.bfloat16
        e = lambda *shape, dtype=bf16: torch.empty(*shape, device=dev, dtype=dtype)  # noqa: E731
        ws = {
            "tokens": e(batch * n, d, dtype=torch.float32),
            "patches": e(batch * L_loc, self.s_embed[0].shape[1]),
            "h": e(batch * n, d),  # dual-stream branch inputs (text rows, then image rows)
            "hj": e(batch * n, d),  # single-stream branch inputs ([text | image] per sample)
            "h2": e(batch * n, d),
            # [B, H, n, 128]; head-major [H, B, n, 128] under sequence parallelism
            "q": e(batch, hq, n, HEAD_DIM),
            "k": e(batch, hkv, n, HEAD_DIM),
            "v": e(batch, hkv, n, HEAD_DIM),
            "glog": e(batch * n, d),  # gate logits, dense per stream (text rows, then image rows)
            "og": e(batch * n, d),  # gated attention output, same rows
            "branch": e(batch * n, d),
            "act": e(batch * n, self.ffn_pad),
            "s_cond": e(batch * L_loc, d),
            "pixels": e(batch * L_loc * pp, pix.hidden_size, dtype=self.pixel_dtype),
            "ph": e(batch * L_loc, pp * pix.hidden_size),
            "pmods": e(batch * L_loc, pp * 4 * pix.hidden_size),
            "comp": e(batch * L_loc, pix.attn_hidden_size),
            "pq": e(batch, pix.num_heads, L_loc, HEAD_DIM),
            "pk": e(batch, pix.num_heads, shard.L, HEAD_DIM),
            "pv": e(batch, pix.num_heads, shard.L, HEAD_DIM),
            "po": e(batch * L_loc, pix.attn_hidden_size),
            "pproj": e(batch * L_loc, pix.attn_hidden_size),
            "pbranch": e(batch * L_loc, pp * pix.hidden_size),
            "t_freq": e(batch, 256, dtype=torch.float32),
            "t_h": e(batch, d, dtype=torch.float32),
            "t_emb": e(batch, d, dtype=torch.float32),
            "core_img": e(batch, 6 * d, dtype=torch.float32),
            "core_txt": e(batch, 6 * d, dtype=torch.float32),
            "mods_img": e(self.img_bias.shape[0], batch, 6 * d, dtype=torch.float32),
            "mods_txt": e(max(1, 0 if self.txt_bias is None else self.txt_bias.shape[0]), batch, 6 * d,
                          dtype=torch.float32),  # fmt: skip
        }
        if shard.world > 1 and self.peer:
            P, N = shard.world, shard.N
            hql, hkvl = hq // P, hkv // P
            ws.update({
                # written by every rank's kernels: this rank's heads over the whole sequence,
                # its token rows of every head's attention output, the pixel keys / values of
                # every patch token (two buffers, alternating by pixel block), barrier flags
                "qf": e(batch, hql, N, HEAD_DIM),
                "kf": e(batch, hkvl, N, HEAD_DIM),
                "vf": e(batch, hkvl, N, HEAD_DIM),
                "o_loc": e(batch * n, hq * HEAD_DIM),
                "pk1": e(batch, pix.num_heads, shard.L, HEAD_DIM),
                "pv1": e(batch, pix.num_heads, shard.L, HEAD_DIM),
                "flags": torch.zeros(P, device=dev, dtype=torch.int32),
            })  # fmt: skip
            shared = ("qf", "kf", "vf", "o_loc", "pk", "pv", "pk1", "pv1", "flags")
            ws["_peers"] = PeerBuffers(self.comm, {name: ws[name] for name in shared})
        elif shard.world > 1:
            P, N = shard.world, shard.N
            hql, hkvl = hq // P, hkv // P
            ws.update({
                # all-to-all receive buffers [P, H/P, B, n, 128] and the full-sequence heads
                "q_r": e(P * hql * batch * n * HEAD_DIM),
                "k_r": e(P * hkvl * batch * n * HEAD_DIM),
                "v_r": e(P * hkvl * batch * n * HEAD_DIM),
                "qf": e(batch, hql, N, HEAD_DIM),
                "kf": e(batch, hkvl, N, HEAD_DIM),
                "vf": e(batch, hkvl, N, HEAD_DIM),
                "of": e(batch, N, hql * HEAD_DIM),  # attention output of this rank's heads
                "o_s": e(batch * n * hq * HEAD_DIM),  # [P(dst), B, n, H/P 128]
                "o_r": e(batch * n * hq * HEAD_DIM),  # [P(src), B, n, H/P 128]
                "o_loc": e(batch * n, hq * HEAD_DIM),  # ungated attention output of the local rows
                # pixel keys / values: local (padded), gathered
                "pk_s": e(batch, pix.num_heads, shard.image_max, HEAD_DIM),
                "pv_s": e(batch, pix.num_heads, shard.image_max, HEAD_DIM),
                "pk_g": e(P * batch * pix.num_heads * shard.image_max * HEAD_DIM),
                "pv_g": e(P * batch * pix.num_heads * shard.image_max * HEAD_DIM),
            })  # fmt: skip
        self._work[key] = ws
        return ws

    # -- forward ----------------------------------------------------------------------
    @torch.no_grad()
    def __call__(
        self, x: torch.Tensor, t: torch.Tensor, text: torch.Tensor, capture: dict | None = None
    ) -> torch.Tensor:
        """``x``: ``[B, 3, H, W]``; ``t``: model time ``[B]``; ``text``: ``[B, T, D]``
        from :meth:`encode_text`. Returns the FP32 velocity ``[B, 3, H, W]``.

        ``capture`` (diagnostics only): when a dict is given, copies of the image
        tokens after every block (``block{i}``), ``s_cond``, the embedded pixels
        (``pixels_in``) and the pixel stream after every pixel block but the last
        are stored in it."""
        if self.graphs and capture is None:
            return self._graph_call(x, t, text)
        return self._forward(x, t, text, capture)

    # -- CUDA graphs (one GPU) ------------------------------------------------------
    _GRAPH_CACHE = 4  # geometries kept (each holds its workspace and graph memory)

    def _graph_call(self, x: torch.Tensor, t: torch.Tensor, text: torch.Tensor) -> torch.Tensor:
        self._check_inputs(x, text)
        key = (tuple(x.shape), tuple(text.shape))
        entry = self._graphs.get(key)
        if entry is None:
            entry = self._capture_graph(x, t, text)
        entry["x"].copy_(x, non_blocking=True)
        entry["t"].copy_(t.reshape(-1), non_blocking=True)
        entry["text"].copy_(text, non_blocking=True)
        entry["graph"].replay()
        _lib.count_launches(entry["kernels"])
        return entry["out"].clone()

    def _capture_graph(self, x: torch.Tensor, t: torch.Tensor, text: torch.Tensor) -> dict:
        dev = self.device
        static = {
            "x": torch.empty(x.shape, device=dev, dtype=torch.float32),
            "t": torch.empty(x.shape[0], device=dev, dtype=torch.float32),
            "text": torch.empty(text.shape, device=dev, dtype=torch.float32),
        }
        static["x"].copy_(x)
        static["t"].copy_(t.reshape(-1))
        static["text"].copy_(text)
        # one eager forward on a side stream first: workspace, tables and library set-up exist before capture
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._forward(static["x"], static["t"], static["text"])
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        before = _lib.launch_count()
        with torch.cuda.graph(graph):
            out = self._forward(static["x"], static["t"], static["text"])
        entry = dict(static, graph=graph, out=out, kernels=_lib.launch_count() - before,
                     # the buffers the graph's kernels address stay alive with it
                     keep=(dict(self._work), dict(self._tables)))  # fmt: skip
        _lib.count_launches(-entry["kernels"])  # captured, not run; each replay counts them
        if len(self._graphs) >= self._GRAPH_CACHE:
            self._graphs.pop(next(iter(self._graphs)))
        self._graphs[(tuple(x.shape), tuple(text.shape))] = entry
        return entry

    def _check_inputs(self, x: torch.Tensor, text: torch.Tensor) -> None:
        p = self.cfg.patch_size
        batch, channels, height, width = x.shape
        if height % p or width % p:
            raise ValueError(f"input {height}x{width} is not divisible by patch_size {p}")
        if channels != self.in_channels:
            raise ValueError(f"expected {self.in_channels} input channels, got {channels}")
        if text.shape[0] != batch or text.shape[2] != self.cfg.hidden_size:
            raise ValueError("text must be [B, T, hidden_size] for the same batch as x")

    def _forward(self, x, t, text, capture=None) -> torch.Tensor:
        cfg = self.cfg
        p = cfg.patch_size
        batch, channels, height, width = x.shape
        self._check_inputs(x, text)
        grid = (height // p, width // p)
        L, T = grid[0] * grid[1], text.shape[1]
        comm = self.comm
        shard = SequenceShard(comm.rank, comm.world, T, L) if comm is not None else SequenceShard(0, 1, T, L)
        n, T_loc, L_loc = shard.n, shard.text, shard.image  # this rank's joint / text / image tokens
        d = cfg.hidden_size
        dev = self.device
        x = x.to(dev, torch.float32).contiguous()
        t = t.to(dev, torch.float32).reshape(batch).contiguous()
        ws = self._workspace(batch, grid, shard)
        (cos, sin), (pcos, psin), pos = self._rope(grid, T)
        # rotary tables are indexed by global position: start at this rank's first token
        cos, sin = cos[shard.start :], sin[shard.start :]
        pcos, psin = pcos[shard.image_start :], psin[shard.image_start :]
        st = torch.cuda.current_stream(dev).cuda_stream
        eps = float(cfg.norm_eps)
        tokens = ws["tokens"]

        # conditioning: t -> t_emb -> silu -> shared cores -> per-block rows
        _lib.call("iris_timestep_embedding", t.data_ptr(), ws["t_freq"].data_ptr(), batch, 256,
                  float(cfg.timestep_max_period), st)  # fmt: skip
        (w0, b0), (w2, b2) = self.t_mlp
        _lib.call("iris_gemv", ws["t_freq"].data_ptr(), batch, 256, w0.data_ptr(), _lib.BF16, b0.data_ptr(),
                  ws["t_h"].data_ptr(), d, 0, 1, st)  # fmt: skip
        _lib.call("iris_gemv", ws["t_h"].data_ptr(), batch, d, w2.data_ptr(), _lib.BF16, b2.data_ptr(),
                  ws["t_emb"].data_ptr(), d, 0, 0, st)  # fmt: skip
        for name, bias_table in (("img", self.img_bias), ("txt", self.txt_bias)):
            if bias_table is None:
                continue
            w, b = self.cores[name]
            core = ws[f"core_{name}"]
            _lib.call("iris_gemv", ws["t_emb"].data_ptr(), batch, d, w.data_ptr(), _lib.BF16, b.data_ptr(),
                      core.data_ptr(), 6 * d, 1, 0, st)  # fmt: skip
            _lib.call("iris_add_bias_rows", core.data_ptr(), bias_table.data_ptr(), ws[f"mods_{name}"].data_ptr(),
                      batch, bias_table.shape[0], 6 * d, st)  # fmt: skip

        # residual stream: [text | image] rows per sample (this rank's slice)
        if T_loc:
            text_rows = text[:, shard.text_start : shard.text_start + T_loc]
            tokens.view(batch, n, d)[:, :T_loc].copy_(text_rows.to(dev, torch.float32))
        _lib.call("iris_patchify", x.data_ptr(), ws["patches"].data_ptr(), batch, channels, height, width, p,
                  shard.image_start, L_loc, st)  # fmt: skip
        K.gemm(ws["patches"], self.s_embed[0], tokens, bias=self.s_embed[1], out_rows=(L_loc, n, T_loc))

        geom = _Geometry(batch=batch, T=T_loc, L=L_loc, N=n, d=d, shard=shard)
        self._first_norm(self.blocks[0], ws, geom, eps, st)
        for i, block in enumerate(self.blocks):
            nxt = self.blocks[i + 1] if i + 1 < len(self.blocks) else None
            self._block(block, nxt, ws, geom, cos, sin, eps, st)
            if capture is not None:
                capture[f"block{i}"] = tokens.view(batch, n, d)[:, T_loc:].clone()
        if capture is not None:
            capture["s_cond"] = ws["s_cond"].float().clone()

        # pixel stage
        out_channels = cfg.in_channels  # 3, also for task models with an extra input channel
        if comm is None:
            v = torch.empty(batch, out_channels, height, width, device=dev, dtype=torch.float32)
        else:  # every rank writes its own patches; the sum assembles the image
            v = torch.zeros(batch, out_channels, height, width, device=dev, dtype=torch.float32)
        self._pixel_stage(x, ws, geom, grid, pcos, psin, pos, v, eps, st, capture)
        # a bounded wait that gave up (dead peer, stalled pipeline) leaves stale buffers behind:
        # the velocity becomes NaN (before the sum, so every rank's copy does) and require_finite raises
        _lib.call("iris_poison_on_error", v.data_ptr(), v.numel(), ERR_WAIT_TIMEOUT, st)
        if comm is not None:
            comm.all_reduce_sum(v)
        return v

    # -- trunk --------------------------------------------------------------------------
    def _mods(self, ws, block: _Block, stream: str) -> torch.Tensor:
        """``[B, 6D]`` modulation rows of a block's stream (shift1, scale1, gate1, shift2, scale2, gate2)."""
        if stream == "y":
            return ws["mods_txt"][block.mod_index["y"]]
        return ws["mods_img"][block.mod_index["x" if stream == "x" else "j"]]

    @staticmethod
    def _chunk(mods: torch.Tensor, k: int, d: int) -> int:
        return mods.data_ptr() + k * d * 4

    def _segments(self, block: _Block, g: "_Geometry"):
        """(stream, rows, rows per batch, token map, dense offset) for a block."""
        if block.dual:
            segs = [("y", g.batch * g.T, g.T, (g.T, g.N, 0), 0), ("x", g.batch * g.L, g.L, (g.L, g.N, g.T), g.batch * g.T)]
            return [seg for seg in segs if seg[1] > 0]  # a sequence-parallel rank may hold no text
        rows = g.batch * g.N
        return [("j", rows, g.N, (rows, 0, 0), 0)]

    def _first_norm(self, block: _Block, ws, g, eps, st) -> None:
        for stream, rows, rpb, tmap, off in self._segments(block, g):
            mods = self._mods(ws, block, stream)
            _lib.call(
                "iris_rms_norm_modulate", ws["tokens"].data_ptr(), _lib.F32, *tmap, ws[_hkey(block)][off:].data_ptr(), _lib.BF16,
                block.norms[stream]["norm1"].data_ptr(), self._chunk(mods, 0, g.d), self._chunk(mods, 1, g.d), 6 * g.d,
                rows, rpb, g.d, eps, st,
            )  # fmt: skip

    def _block(self, block, nxt, ws, g, cos, sin, eps, st) -> None:
        """One trunk block. Dual-stream blocks run each linear as one grouped
        launch over both streams (image problem first, so the small text problem
        fills the tail of its tile list); the sigmoid gate is applied in the
        attention epilogue, which writes each stream's rows densely."""
        cfg = self.cfg
        segs = self._segments(block, g)
        order = segs[::-1]
        h = ws[_hkey(block)]

        def grouped(a_key, weights, out_key, **kw):
            problems = []
            for s, rows, _, _, off in order:
                w = weights[s]
                extra = dict(kw)
                if isinstance(w, tuple):
                    w, extra["bias"] = w
                a = h if a_key is None else ws[a_key]
                problems.append(K.gemm_problem(a[off : off + rows], w, ws[out_key][off : off + rows], **extra))
            K.gemm_grouped(problems, st)

        # Q/K/V projection with QK-norm + RoPE + the head layout in its epilogue
        problems = []
        peers = None
        if self.peer:  # each head row straight into the full-sequence buffer of the rank that owns the head
            pb = ws["_peers"]
            peers = K.PeerHeads(_lib.HEADS_PEER_SCATTER, pb.ptrs["qf"], pb.ptrs["kf"], pb.ptrs["vf"], g.shard.start,
                                g.shard.N)  # fmt: skip
        for s, rows, _, tmap, off in order:
            qn, kn = block.qk_norm[s]
            heads = K.HeadsOut(
                ws["q"], ws["k"], ws["v"], qn, kn, cos, sin, eps, cfg.num_heads, cfg.kv_heads, g.N, g.batch, g.N, g.N,
                head_major=self.comm is not None, peers=peers,
            )  # fmt: skip
            problems.append(K.gemm_problem(h[off : off + rows], block.qkv[s], None, out_rows=tmap, heads=heads))
        K.gemm_grouped(problems, st)
        if self.comm is None:
            grouped(None, block.gate, "glog")  # gate logits; sigmoid in the attention epilogue
            split = g.T if block.dual else 0
            bt = g.batch * split
            K.flash_attention_split(
                ws["q"], ws["k"], ws["v"], split, ws["og"][:bt] if bt else None, ws["og"][bt:],
                ws["glog"][:bt] if bt else None, ws["glog"][bt:], bound=block.score_bound,
            )  # fmt: skip
        else:
            self._attention_sequence_parallel(block, segs, ws, g, st)
        grouped("og", block.proj, "branch")
        # one launch for both streams' residual rows, as for the GEMMs
        _residuals([self._attn_residual(block, *seg, ws, g) for seg in segs], g.d, eps, st)
        grouped("h2", block.w13, "act", epilogue=_lib.EPI_SWIGLU)
        grouped("act", block.w2, "branch")
        _residuals([self._mlp_residual(block, nxt, *seg, ws, g) for seg in segs if nxt is not None or seg[0] != "y"],
                   g.d, eps, st)  # fmt: skip

    def _attention_sequence_parallel(self, block, segs, ws, g, st) -> None:
        """Ulysses attention: Q/K/V (head-major, this rank's tokens) -> all-to-all
        -> this rank's heads over the whole sequence -> attention -> all-to-all
        back -> the gate GEMM applies sigmoid(h W_g^T) to the local token rows."""
        comm, P = self.comm, self.comm.world
        B, n = g.batch, g.N
        hql, hkvl = self.cfg.num_heads // P, self.cfg.kv_heads // P
        if self.peer:
            # the Q/K/V epilogue has stored into every rank's qf / kf / vf; attention
            # stores each output row into the token rows of the rank that owns it
            self._barrier(ws)
            K.flash_attention_peers(ws["qf"], ws["kf"], ws["vf"], ws["_peers"].ptrs["o_loc"], n,
                                    comm.rank * hql * HEAD_DIM, self.cfg.num_heads * HEAD_DIM,
                                    bound=block.score_bound)  # fmt: skip
            self._barrier(ws)
        else:
            for name, heads in (("q", hql), ("k", hkvl), ("v", hkvl)):
                scatter_heads(comm, K.block_copy, ws[name], ws[name + "_r"], ws[name + "f"], heads, B, n, HEAD_DIM)
            K.flash_attention(ws["qf"], ws["kf"], ws["vf"], ws["of"], bound=block.score_bound)
            gather_tokens(comm, K.block_copy, ws["of"], ws["o_s"], ws["o_r"], ws["o_loc"], B, n, hql * HEAD_DIM)
        h = ws[_hkey(block)]
        problems = [
            K.gemm_problem(h[off : off + rows], block.gate[s], ws["og"][off : off + rows], epilogue=_lib.EPI_GATE,
                           aux=ws["o_loc"], aux_rows=tmap)  # fmt: skip
            for s, rows, _, tmap, off in segs[::-1]
        ]
        K.gemm_grouped(problems, st)

    def close(self) -> None:
        """Unmap the other ranks' exchange buffers (sequence parallelism over
        processes); the engine stays usable and maps them again when needed."""
        for ws in self._work.values():
            if "_peers" in ws:
                ws["_peers"].close()
        self._work.clear()

    def _barrier(self, ws) -> None:
        """All ranks' work enqueued so far (their stores into this rank's buffers
        included) completes before this rank's next kernel; bounded wait."""
        self._epoch += 1
        K.peer_barrier(ws["flags"], ws["_peers"].ptrs["flags"], self.comm.rank, self._epoch, self.peer_timeout_s)

    def _attn_residual(self, block, stream, rows, rpb, tmap, off, ws, g) -> "_lib.ResidualProblem":
        """Post-norm + gate + residual of the attention branch, fused with the
        MLP branch's input norm-modulate (written to ``h2``)."""
        d = g.d
        mods = self._mods(ws, block, stream)
        norms = block.norms[stream]
        h2, branch = ws["h2"][off : off + rows], ws["branch"][off : off + rows]
        return _lib.ResidualProblem(
            ws["tokens"].data_ptr(), *tmap, branch.data_ptr(), rows, 0, 0, norms["post_attn"].data_ptr(),
            self._chunk(mods, 2, d), 6 * d, rows, rpb, _lib.NEXT_NORM_MODULATE, norms["norm2"].data_ptr(),
            self._chunk(mods, 3, d), self._chunk(mods, 4, d), 6 * d, h2.data_ptr(), rows, 0, 0,
        )  # fmt: skip

    def _mlp_residual(self, block, nxt, stream, rows, rpb, tmap, off, ws, g) -> "_lib.ResidualProblem":
        """Post-norm + gate + residual of the MLP branch; it also writes the next
        block's input (or, after the last block, ``silu(t_emb + x)`` of the image rows)."""
        d = g.d
        mods = self._mods(ws, block, stream)
        norms = block.norms[stream]
        branch = ws["branch"][off : off + rows]
        tok = ws["tokens"].data_ptr()
        if nxt is None:
            # last block: only image rows continue; they leave as s = silu(t_emb + x)
            image_map = (g.L, g.N, g.T)
            return _lib.ResidualProblem(
                tok, *image_map, branch.data_ptr(), *image_map, norms["post_mlp"].data_ptr(), self._chunk(mods, 5, d),
                6 * d, g.batch * g.L, g.L, _lib.NEXT_SILU_ADD, None, ws["t_emb"].data_ptr(), None, d,
                ws["s_cond"].data_ptr(), g.batch * g.L, 0, 0,
            )  # fmt: skip
        nstream = stream if nxt.dual else "j"
        nmods = self._mods(ws, nxt, nstream)
        if nxt.dual:
            next_map = (rows, 0, 0)
            next_out = ws["h"][off:]
        else:
            next_map = tmap if stream != "j" else (rows, 0, 0)
            # a separate buffer: the other stream of this dual block may still read ws["h"]
            next_out = ws["hj"]
        return _lib.ResidualProblem(
            tok, *tmap, branch.data_ptr(), rows, 0, 0, norms["post_mlp"].data_ptr(), self._chunk(mods, 5, d), 6 * d,
            rows, rpb, _lib.NEXT_NORM_MODULATE, nxt.norms[nstream]["norm1"].data_ptr(), self._chunk(nmods, 0, d),
            self._chunk(nmods, 1, d), 6 * d, next_out.data_ptr(), *next_map,
        )  # fmt: skip

    # -- pixel stage ------------------------------------------------------------------
    def _pixel_stage(self, x, ws, g, grid, pcos, psin, pos, v, eps, st, capture=None) -> None:
        cfg = self.cfg
        pix = cfg.pixel
        p = cfg.patch_size
        height, width = grid[0] * p, grid[1] * p
        pdt = _lib.F32 if self.pixel_dtype == torch.float32 else _lib.BF16
        sp = self.comm is not None
        pw, pb = self.pixel_embed_w
        blocks = self.pixel_blocks
        _lib.call(
            "iris_pixel_embed", x.data_ptr(), pw.data_ptr(), pb.data_ptr(), None if pos is None else pos.data_ptr(),
            ws["pixels"].data_ptr(), pdt, ws["ph"].data_ptr(), blocks[0]["norm1"].data_ptr(), eps, g.batch,
            self.in_channels, height, width, p, g.shard.image_start, g.L, st,
        )  # fmt: skip
        heads = pix.num_heads
        if capture is not None:
            capture["pixels_in"] = ws["pixels"].float().view(g.batch * g.L, -1, pix.hidden_size).clone()
        for i, blk in enumerate(blocks):
            if capture is not None and i > 0:
                capture[f"pixel_block{i - 1}"] = ws["pixels"].float().view(g.batch * g.L, -1, pix.hidden_size).clone()
            K.gemm(ws["s_cond"], blk["adaln"][0], ws["pmods"], bias=blk["adaln"][1])
            K.gemm(ws["ph"], blk["compress"][0], ws["comp"], bias=blk["compress"][1])
            qn, kn = blk["qk_norm"]
            kv = ("pk_s", "pv_s") if sp and not self.peer else ("pk", "pv")
            peers = None
            if self.peer:  # every rank's keys / values of all patch tokens; two buffers, alternating by block
                kv = ("pk", "pv") if i % 2 == 0 else ("pk1", "pv1")
                pb = ws["_peers"]
                peers = K.PeerHeads(_lib.HEADS_PEER_BROADCAST_KV, None, pb.ptrs[kv[0]], pb.ptrs[kv[1]],
                                    g.shard.image_start, g.shard.L)  # fmt: skip
            targets = K.HeadsOut(
                ws["pq"], ws[kv[0]], ws[kv[1]], qn, kn, pcos, psin, eps, heads, heads, g.L, g.batch, g.L,
                ws[kv[0]].shape[2], peers=peers,
            )  # fmt: skip
            K.gemm_grouped([K.gemm_problem(ws["comp"], blk["qkv"], None, heads=targets)], st)
            if self.peer:
                self._barrier(ws)
            elif sp:  # local queries over the keys / values of every patch token
                for name in ("pk", "pv"):
                    gather_image_tokens(self.comm, K.block_copy, g.shard, ws[name + "_s"], ws[name + "_g"], ws[name],
                                        g.batch, heads, HEAD_DIM)  # fmt: skip
            full = kv if self.peer else ("pk", "pv")
            K.flash_attention(ws["pq"], ws[full[0]], ws[full[1]], ws["po"].view(g.batch, g.L, -1),
                              bound=blk["score_bound"])  # fmt: skip
            K.gemm(ws["po"], blk["proj"][0], ws["pproj"], bias=blk["proj"][1])
            K.gemm(ws["pproj"], blk["expand"][0], ws["pbranch"], bias=blk["expand"][1])
            (w1, b1), (w2, b2) = blk["fc1"], blk["fc2"]
            if i + 1 < len(blocks):
                _lib.call(
                    "iris_pixel_mlp", ws["pixels"].data_ptr(), pdt, ws["pbranch"].data_ptr(), ws["pmods"].data_ptr(),
                    blk["norm2"].data_ptr(), w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(),
                    blocks[i + 1]["norm1"].data_ptr(), ws["ph"].data_ptr(), ws["pixels"].numel() // 16, eps, st,
                )  # fmt: skip
            else:
                fn, fw, fb = self.final
                _lib.call(
                    "iris_pixel_mlp_head", ws["pixels"].data_ptr(), pdt, ws["pbranch"].data_ptr(),
                    ws["pmods"].data_ptr(), blk["norm2"].data_ptr(), w1.data_ptr(), b1.data_ptr(), w2.data_ptr(),
                    b2.data_ptr(), fn.data_ptr(), fw.data_ptr(), fb.data_ptr(), v.data_ptr(), g.batch, height, width,
                    p, g.shard.image_start, g.L, eps, st,
                )  # fmt: skip


def _residuals(problems: list, width: int, eps: float, st: int) -> None:
    """The residual updates of a block's streams (bf16 branches and next inputs) in one launch."""
    array = (_lib.ResidualProblem * len(problems))(*problems)
    _lib.call("iris_gated_residual_rms_norm_grouped", array, len(problems), _lib.BF16, _lib.BF16, width, eps, st)


def _hkey(block: _Block) -> str:
    """Workspace key of a block's branch-input buffer."""
    return "h" if block.dual else "hj"


@dataclass
class _Geometry:
    """This rank's token counts per sample (all tokens without sequence parallelism)."""

    batch: int
    T: int
    L: int
    N: int
    d: int
    shard: SequenceShard
