"""The masked text adapters on the B200 kernels, once per prompt.

``lap_blocks2`` (``LayerwiseTextEmbedder``, ``src/iris3b/nn/embeddings.py:209-266``)
and ``blocks2`` (``TransformerTextEmbedder``, ``:144-207``): what
``MetalIris.encode_text`` evaluates with the upstream modules under autocast
(``src/iris_metal/model.py:133-145``) runs here on this library's kernels:

* every Linear on the tensor-core GEMM: residual updates ``x + f(x)`` through
  the ``EPI_ADD`` epilogue (FP32 residual rows updated in place), the
  layer-block MLP's ``SiLU`` and the refiner's SwiGLU in their GEMMs'
  epilogues;
* the pre-norms on ``iris_rms_norm_modulate`` (no modulation), the output
  RMSNorm with ``y_pos_embedding`` added in the same pass
  (``iris_rms_norm_add_rows``);
* attention on ``iris_small_attention``, read straight from the Q/K/V
  projection: over each token's encoder layers (12 keys) in the layer blocks,
  over the prompt's tokens with pad keys masked (the diagonal kept) and
  per-head QK RMSNorm in the refiner;
* the layer pool on ``iris_layer_pool``.

Precision: BF16 GEMM operands and attention inputs, FP32 accumulation, FP32
residual streams and norms.
"""

from __future__ import annotations

import torch

from iris_b200 import _lib
from iris_b200 import kernels as K


def _pad_rows(w: torch.Tensor, rows: int) -> torch.Tensor:
    out = torch.zeros(rows, *w.shape[1:], device=w.device, dtype=w.dtype)
    out[: w.shape[0]] = w
    return out


def _pad_cols(w: torch.Tensor, cols: int) -> torch.Tensor:
    out = torch.zeros(w.shape[0], cols, device=w.device, dtype=w.dtype)
    out[:, : w.shape[1]] = w
    return out


class TextAdapter:
    """``y_embedder(states, mask)`` of a masked adapter, from a state dict with
    the reference's parameter names under ``prefix``."""

    def __init__(self, cfg, state: dict, device: torch.device, prefix: str = "y_embedder."):
        from iris_b200.model import pack_swiglu

        self.cfg, self.device = cfg, device
        self.kind = cfg.text_adapter
        if self.kind not in ("lap_blocks2", "blocks2"):
            raise ValueError(f"TextAdapter handles the masked adapters, not {self.kind!r}")
        d, dt = cfg.hidden_size, cfg.text_dim
        if d % 128 or dt % 128:
            raise ValueError("TextAdapter needs hidden_size and text_dim to be multiples of 128")

        def get(name):
            key = prefix + name
            if key not in state:
                raise ValueError(f"TextAdapter: missing parameter {key}")
            return state[key].detach().to(device)

        bf = lambda name: get(name).to(torch.bfloat16).contiguous()  # noqa: E731
        f32 = lambda name: get(name).to(torch.float32).contiguous()  # noqa: E731
        opt = lambda name: f32(name) if prefix + name in state else None  # noqa: E731
        self.layer_blocks = []
        if self.kind == "lap_blocks2":
            if dt % cfg.text_lap_num_heads or (dt // cfg.text_lap_num_heads) % 8:
                raise ValueError("TextAdapter: layer-attention heads must be a multiple of 8 wide")
            hidden = int(dt * cfg.text_lap_mlp_ratio)
            pad = -(-hidden // 32) * 32  # zero rows / columns: silu(0) = 0 contributes nothing
            for i in range(2):
                b = f"layer_blocks.{i}"
                self.layer_blocks.append({
                    "norm1": f32(f"{b}.norm1.weight"),
                    "qkv": bf(f"{b}.attn.qkv.weight"),
                    "proj": (bf(f"{b}.attn.proj.weight"), f32(f"{b}.attn.proj.bias")),
                    "norm2": f32(f"{b}.norm2.weight"),
                    "fc1": (_pad_rows(bf(f"{b}.mlp.0.weight"), pad), _pad_rows(f32(f"{b}.mlp.0.bias"), pad)),
                    "fc2": (_pad_cols(bf(f"{b}.mlp.2.weight"), pad), f32(f"{b}.mlp.2.bias")),
                })  # fmt: skip
            self.pool = (f32("layer_pool.weight").reshape(-1), f32("layer_pool.bias").reshape(-1))
            if self.pool[0].numel() != cfg.text_lap_num_layers:
                raise ValueError("TextAdapter: layer_pool does not match text_lap_num_layers")
            prefix_r = "refiner."
        else:
            prefix_r = ""
        hd = d // cfg.num_heads
        if d % cfg.num_heads or hd % 8 or hd > 128:
            raise ValueError("TextAdapter: refiner heads must be a multiple of 8 wide, at most 128")
        self.proj = (bf(f"{prefix_r}proj.weight"), f32(f"{prefix_r}proj.bias"))
        self.blocks = []
        for i in range(2):
            b = f"{prefix_r}blocks.{i}"
            w13, w2 = pack_swiglu(bf(f"{b}.mlp.w1.weight"), bf(f"{b}.mlp.w3.weight"), bf(f"{b}.mlp.w2.weight"))
            self.blocks.append({
                "norm1": f32(f"{b}.norm1.weight"),
                "qkv": (bf(f"{b}.attn.qkv.weight"), opt(f"{b}.attn.qkv.bias")),
                "qk_norm": (opt(f"{b}.attn.q_norm.weight"), opt(f"{b}.attn.k_norm.weight")),
                "proj": (bf(f"{b}.attn.proj.weight"), f32(f"{b}.attn.proj.bias")),
                "norm2": f32(f"{b}.norm2.weight"),
                "w13": w13,
                "w2": w2,
            })  # fmt: skip
        self.norm = f32(f"{prefix_r}norm.weight")
        self._zeros = torch.zeros(max(d, dt), device=device, dtype=torch.float32)

    # -- pieces ------------------------------------------------------------------
    def _rms(self, x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, st: int) -> None:
        rows, width = x.shape
        _lib.call("iris_rms_norm_modulate", x.data_ptr(), _lib.F32, rows, 0, 0, out.data_ptr(), _lib.BF16,
                  weight.data_ptr(), self._zeros.data_ptr(), self._zeros.data_ptr(), 0, rows, rows, width,
                  float(self.cfg.norm_eps), st)  # fmt: skip

    def _attention(self, qkv, seqs, n, heads, out, gains, mask, st) -> None:
        hd = out.shape[1] // heads
        qg, kg = gains
        _lib.call("iris_small_attention", qkv.data_ptr(), seqs, n, heads, hd, qkv.stride(0),
                  None if qg is None else qg.data_ptr(), None if kg is None else kg.data_ptr(),
                  float(self.cfg.norm_eps), None if mask is None else mask.data_ptr(), hd**-0.5, out.data_ptr(),
                  out.stride(0), st)  # fmt: skip

    # -- forward ------------------------------------------------------------------
    @torch.no_grad()
    def __call__(self, states: torch.Tensor, mask: torch.Tensor, pos: torch.Tensor | None = None) -> torch.Tensor:
        """``states``: ``[B, T, layers, text_dim]`` (``lap_blocks2``) or ``[B, T,
        text_dim]`` (``blocks2``); ``mask``: ``[B, T]``, nonzero = real token.
        Returns FP32 ``[B, T, hidden]``, plus ``pos`` (``[T, hidden]``) when given."""
        cfg, dev = self.cfg, self.device
        if mask.shape != states.shape[:2]:
            raise ValueError(f"text mask must be {tuple(states.shape[:2])}, got {tuple(mask.shape)}")
        batch, n = mask.shape
        dt, d = cfg.text_dim, cfg.hidden_size
        if batch == 0 or n == 0:
            return torch.zeros(batch, n, d, device=dev)
        st = torch.cuda.current_stream(dev).cuda_stream
        bf16 = torch.bfloat16
        keep = (mask.to(dev) != 0).to(torch.uint8).contiguous()
        rows = batch * n
        if self.kind == "lap_blocks2":
            layers = cfg.text_lap_num_layers
            if states.shape != (batch, n, layers, dt):
                raise ValueError(f"layerwise text states must be {(batch, n, layers, dt)}, got {tuple(states.shape)}")
            R = rows * layers
            x = torch.empty(R, dt, device=dev, dtype=torch.float32)
            x.copy_(states.reshape(R, dt))  # the residual stream; never the caller's tensor
            h = torch.empty(R, dt, device=dev, dtype=bf16)
            qkv = torch.empty(R, 3 * dt, device=dev, dtype=bf16)
            o = torch.empty(R, dt, device=dev, dtype=bf16)
            f = torch.empty(R, self.layer_blocks[0]["fc1"][0].shape[0], device=dev, dtype=bf16)
            for blk in self.layer_blocks:
                self._rms(x, blk["norm1"], h, st)
                K.gemm(h, blk["qkv"], qkv)
                self._attention(qkv, rows, layers, cfg.text_lap_num_heads, o, (None, None), None, st)
                K.gemm(o, blk["proj"][0], x, bias=blk["proj"][1], epilogue=_lib.EPI_ADD)
                self._rms(x, blk["norm2"], h, st)
                K.gemm(h, blk["fc1"][0], f, bias=blk["fc1"][1], epilogue=_lib.EPI_SILU)
                K.gemm(f, blk["fc2"][0], x, bias=blk["fc2"][1], epilogue=_lib.EPI_ADD)
            pooled = torch.empty(rows, dt, device=dev, dtype=bf16)
            _lib.call("iris_layer_pool", x.data_ptr(), rows, layers, dt, self.pool[0].data_ptr(),
                      self.pool[1].data_ptr(), pooled.data_ptr(), st)  # fmt: skip
        else:
            if states.shape != (batch, n, dt):
                raise ValueError(f"text states must be {(batch, n, dt)}, got {tuple(states.shape)}")
            pooled = states.reshape(rows, dt).to(dev, bf16).contiguous()
        y = torch.empty(rows, d, device=dev, dtype=torch.float32)
        K.gemm(pooled, self.proj[0], y, bias=self.proj[1])
        h = torch.empty(rows, d, device=dev, dtype=bf16)
        qkv = torch.empty(rows, 3 * d, device=dev, dtype=bf16)
        o = torch.empty(rows, d, device=dev, dtype=bf16)
        act = torch.empty(rows, self.blocks[0]["w2"].shape[1], device=dev, dtype=bf16)
        for blk in self.blocks:
            self._rms(y, blk["norm1"], h, st)
            K.gemm(h, blk["qkv"][0], qkv, bias=blk["qkv"][1])
            self._attention(qkv, batch, n, cfg.num_heads, o, blk["qk_norm"], keep, st)
            K.gemm(o, blk["proj"][0], y, bias=blk["proj"][1], epilogue=_lib.EPI_ADD)
            self._rms(y, blk["norm2"], h, st)
            K.gemm(h, blk["w13"], act, epilogue=_lib.EPI_SWIGLU)
            K.gemm(act, blk["w2"], y, epilogue=_lib.EPI_ADD)
        add = pos[:n].to(dev, torch.float32).contiguous() if pos is not None else self._zeros[:d].expand(n, d).contiguous()
        _lib.call("iris_rms_norm_add_rows", y.data_ptr(), self.norm.data_ptr(), add.data_ptr(), rows, n, d,
                  float(cfg.norm_eps), st)  # fmt: skip
        return y.view(batch, n, d)
