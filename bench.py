#!/usr/bin/env python
"""Benchmark: Iris-3B-shaped denoising at 1024^2 on B200s.

One bench step = the 4-step guided flow-Euler loop (sigmas 1.0, 0.938, 0.833,
0.625; CFG 3 on [uncond; cond], so every denoiser call has 2 rows per image)
over this rank's share of 8 images; images are split data-parallel across the
N GPUs with no collective in the timed region. ``value`` = 8 images / the
slowest rank's step time. The model is the BASELINE config-3 architecture
(d = 3072, 24 blocks, 24 heads x 128, SwiGLU 8192, 4096 + 256 tokens) with
random weights (std 0.02); inputs are seeded N(0, 1) noise and text states.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --workload step2048 [--gpus N] ...

``--workload step2048`` is BASELINE config 5 instead: one guided denoiser call
(B = 2) at 2048^2 per step, spread over the N GPUs by Ulysses sequence
parallelism (value = ms per step, the slowest rank's). ``--workload ops`` is
config 2: the reference's two fused-op microbenchmarks (rms_norm_modulate and
the qk_norm_rope pair) against the HBM roofline.

For N > 1 run one process per GPU under torchrun. Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO), str(REPO / "iris-3b-metal_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "ms per denoise step and images/sec at 1024² (B=2 CFG) at 1/2/4/8 B200; % roofline"
UNIT = "images/s"
IMAGES = 8
RESOLUTION = 1024
SIGMAS = (1.0, 0.938, 0.833, 0.625)
CFG_SCALE = 3.0
TEXT_LEN, TEXT_DIM = 256, 2560
WORKLOAD = (
    "BASELINE config 4: 8 images of 1024^2 noise, 4 flow-Euler steps with CFG 3 on [uncond; cond] "
    "(2 denoiser rows per image per step), DP split by image across N GPUs"
)


# DRAM bytes (read + write) per GEMM launch of the N = 1 workload (the 141 GEMM
# launches of a 16-row call, 4 calls per step), from one capture of the small
# model's 16-row call, whose 16 GEMM launches have the full model's shapes (one
# launch of each kind: patch embed, the dual and single blocks' QKV / gate / proj /
# w13 / w2, the pixel block's five):
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum --clock-control none \
#       --nvtx --nvtx-include "profiled/" -k regex:gemm_bf16 --csv --log-file gemm_traffic_small16.csv \
#       python bench.py --profile small16
# weighted by the kinds' launch counts in the full model (1 + 8 x 5 + 16 x 5 + 4 x 5).
GEMM_TRAFFIC_PER_LAUNCH = 2750.4e6


def peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16": data["bf16_tflops"], "bf16_sustained": data["bf16_tflops_sustained"],
                "source": "measured"}  # fmt: skip
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def step_flops(batch_rows: int, L: int = 4096, T: int = 256) -> float:
    """Algorithmic FLOPs of one denoiser call (GEMMs + attention) for the
    benchmark model, as scripts/flops.py of the reference counts them."""
    d, ffn, heads, hd = 3072, 8192, 24, 128
    N = T + L
    per_block = 2 * N * d * (3 * d) + 2 * N * d * d * 2 + 2 * N * d * ffn * 3 + 4 * N * N * heads * hd
    pp, da = 256, 1280
    pit = 2 * L * d * (4 * 16 * pp) + 2 * L * (pp * 16) * da * 2 + 2 * L * da * 3 * da + 2 * L * da * da
    pit += 4 * L * L * da + 2 * L * pp * (16 * 64 * 2)
    embed = 2 * L * 768 * d
    return batch_rows * (24 * per_block + 4 * pit + embed)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, device: int):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            ident = str(device)
        self.cmd = ["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, sm_max, reasons = [], None, set()
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        busy = [s for s in sm if sm_max and s > 0.3 * sm_max] or sm
        return {
            "sm_mhz": statistics.median(busy) if busy else None,
            "sm_max_mhz": sm_max,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


MODEL = ("iris-3b-shaped: d3072, 8 dual + 16 single-stream blocks, 24 MHA heads x 128, SwiGLU 8192, "
         "4 post-modulated PiT blocks; random-init weights (std 0.02)")


def bench_config(world: int) -> dict:
    """The ``config`` of the default workload's JSON line; both arms print the same dict."""
    return {
        "workload": WORKLOAD,
        "model": MODEL,
        "global_batch": IMAGES,
        "rows_per_call_per_gpu": 2 * (IMAGES // world + (1 if IMAGES % world else 0)),
        "seq_len": 4352,
        "parallelism": f"dp{world}",
        "l2": "no flush: every step streams 8.7 GB of weights, far above the 126 MB L2",
    }


def make_inputs(seed_noise: int = 0, seed_text: int = 4):
    gen = torch.Generator().manual_seed(seed_noise)
    noise = torch.randn(IMAGES, 3, RESOLUTION, RESOLUTION, generator=gen)
    tgen = torch.Generator().manual_seed(seed_text)
    cond = torch.randn(IMAGES, TEXT_LEN, TEXT_DIM, generator=tgen)
    uncond = torch.randn(1, TEXT_LEN, TEXT_DIM, generator=tgen)
    return noise, cond, uncond


def cpu_baseline_sample(threads: int) -> dict:
    """The oracle (fp32 PyTorch restatement of the reference's path) on the host
    cores: one block of each kind at B = 2, 1024^2, extrapolated to a forward."""
    from oracle.config import baseline_step_config
    from oracle.timing import BlockSampler

    torch.set_num_threads(threads)
    sampler = BlockSampler(baseline_step_config(), batch=2, height=RESOLUTION, width=RESOLUTION)
    seconds = sampler.forward_seconds(repeats=1)
    per_image = len(SIGMAS) * seconds["forward"]  # 4 guided calls of B = 2 per image
    return {"seconds": seconds, "images_per_s": 1.0 / per_image}


def reference_arm(args, rank: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from oracle.config import baseline_step_config
    from oracle.timing import BlockSampler

    torch.set_num_threads(threads)
    sampler = BlockSampler(baseline_step_config(), batch=2, height=RESOLUTION, width=RESOLUTION)
    cfg = sampler.cfg
    # each step: one block of each kind -> a forward estimate by block counts -> images/s
    per_kind = {"dual": [], "single": [], "pixel": []}
    times = []
    with torch.no_grad():
        for _ in range(args.warmup):
            sampler.single()
        for _ in range(args.steps):
            step_start = time.perf_counter()
            for kind in per_kind:
                t0 = time.perf_counter()
                getattr(sampler, kind)()
                per_kind[kind].append(time.perf_counter() - t0)
            times.append(time.perf_counter() - step_start)
    med = {kind: statistics.median(v) for kind, v in per_kind.items()}
    forward = cfg.dual_depth * med["dual"] + (cfg.depth - cfg.dual_depth) * med["single"] + cfg.pixel.depth * med["pixel"]
    value = 1.0 / (len(SIGMAS) * forward)
    step_s = statistics.median(times)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_s * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": bench_config(args.gpus),
        "cpu_baseline": {
            "value": value,
            "unit": UNIT,
            "cores": threads,
            "kind": "port",
            "sample": "oracle fp32 PyTorch path, one dual + one single + one pixel block at B=2 1024^2 per step, "
            f"extrapolated by block counts to a forward ({forward:.1f} s) and 4 guided calls per image",
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def profile_run(kind: str) -> None:
    """Workloads for ncu: two warm B = 2 denoiser calls at 1024^2, then one call
    inside the NVTX range ``profiled`` (select it with ``--nvtx --nvtx-include
    profiled/``). ``forward``: the benchmark model. ``small``: the same shapes
    with one dual and one single-stream block and one pixel block (< 1 GB of
    weights), for multi-pass captures. ``sampler``: the small model, and in the
    range the 4-step guided Euler loop of one image (four B = 2 calls and the
    fused CFG + Euler updates). ``forward16`` / ``small16``: the benchmark's
    16-row calls (8 images x [uncond; cond]) on the full / small model."""
    from dataclasses import replace

    from iris_b200 import CudaIris, IrisWeights, baseline_step_config, synthetic_state
    from iris_b200.config import PixelStageConfig

    cfg = baseline_step_config()
    if kind in ("small", "sampler", "small16"):
        cfg = replace(cfg, depth=2, dual_depth=1, pixel=PixelStageConfig(depth=1))
    device = torch.device("cuda", 0)
    engine = CudaIris(IrisWeights(cfg, synthetic_state(cfg, device, seed=0)))
    noise, cond_states, uncond_states = make_inputs()
    x = noise[:1].repeat(2, 1, 1, 1).to(device)
    text = torch.cat([engine.encode_text(uncond_states.to(device)), engine.encode_text(cond_states[:1].to(device))])
    t = torch.full((2,), 625.0, device=device)
    if kind in ("forward16", "small16"):  # the benchmark's calls: 8 images x [uncond; cond]
        x = torch.cat([noise, noise]).to(device)
        cond = engine.encode_text(cond_states.to(device))
        text = torch.cat([engine.encode_text(uncond_states.to(device)).expand(IMAGES, -1, -1), cond]).contiguous()
        t = torch.full((2 * IMAGES,), 1000.0, device=device)
    for _ in range(2):
        engine(x, t, text)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profiled")
    if kind == "sampler":
        from iris_b200.sampling import euler_cfg

        v = euler_cfg(engine, x[:1], text[1:], text[:1], cfg_scale=CFG_SCALE, sigmas=SIGMAS)
    else:
        v = engine(x, t, text)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"profile": kind, "finite": bool(torch.isfinite(v).all())}))


def fused_ops(args) -> None:
    """BASELINE config 2 through the reference's kernel API: rms_norm_modulate
    on x bf16 [2, 4096, 3072] (bf16 out) and qk_norm_rope on the Q and K
    projections bf16 [2, 4352, 3072] (24 heads, the 1024^2 RoPE table). Before
    each timed call a 512 MB write evicts L2 (the operands fit in it) and a
    256 MB read then replaces its dirty lines with clean ones, so the timed call
    pays for no write-back of the flush; a ~100 us device sleep then keeps the
    GPU busy while the host enqueues the call. Each call is bracketed by CUDA events
    on its stream; the mean over the calls is reported (the event clock ticks in
    2.048 us steps, so a median would snap to a tick)."""
    from iris_b200 import kernels as K
    from iris_b200.tables import cos_sin, rope_1d, rope_2d

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device="cpu").manual_seed(2)
    x = torch.randn(2, 4096, 3072, generator=g).to(device, torch.bfloat16)
    w = (1 + 0.02 * torch.randn(3072, generator=g)).to(device)
    shift, scale = (0.1 * torch.randn(2, 1, 3072, generator=g)).to(device), (0.1 * torch.randn(2, 1, 3072, generator=g)).to(device)
    g3 = torch.Generator(device="cpu").manual_seed(3)
    q, k = (torch.randn(2, 4352, 3072, generator=g3).to(device, torch.bfloat16) for _ in range(2))
    qw, kw = (1 + 0.02 * torch.randn(128, generator=g3)).to(device), (1 + 0.02 * torch.randn(128, generator=g3)).to(device)
    cos, sin = cos_sin(rope_1d(128, 256, 1e4), rope_2d(128, 64, 64, 1e4, 16.0, "isotropic"), device=device)
    qo, ko = (torch.empty(2, 24, 4352, 128, device=device, dtype=torch.bfloat16) for _ in range(2))
    flush = torch.empty(512 * 2**20, dtype=torch.uint8, device=device)
    clean = torch.ones(64 * 2**20, dtype=torch.float32, device=device)

    def timed(fn, reps):
        # the first pass (same calls, discarded) warms the clocks under the same
        # back-to-back load as the measured one
        for _pass in range(2):
            times = []
            for _ in range(reps):
                flush.fill_(1)  # evicts L2 and keeps the GPU busy while the events and the call are enqueued
                clean.sum()  # clean lines replace the flush's dirty ones
                torch.cuda._sleep(200_000)  # ~100 us of queued device time: host launch latency stays outside the events
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                times.append((s, e))
            torch.cuda.synchronize()
        # CUDA events tick in 2.048 us steps on these boxes: the median snaps to
        # a tick, the mean over many calls (random start phase) does not.
        return statistics.mean(a.elapsed_time(b) for a, b in times)

    norm_ms = timed(lambda: K.rms_norm_modulate(x, w, shift, scale, 1e-6, torch.bfloat16), max(args.steps, 100))

    def qk():
        K.qk_norm_rope(q, qw, cos, sin, 1e-6, 24, out=qo)
        K.qk_norm_rope(k, kw, cos, sin, 1e-6, 24, out=ko)

    qk_ms = timed(qk, max(args.steps, 100))
    pk = peaks()
    norm_bytes = 2 * (2 * 4096 * 3072 * 2) + 3072 * 4 + 2 * 2 * 3072 * 4
    qk_bytes = 4 * (2 * 4352 * 24 * 128 * 2) + 2 * 4352 * 64 * 4 + 2 * 128 * 4
    norm_gbs, qk_gbs = norm_bytes / norm_ms / 1e6, qk_bytes / qk_ms / 1e6
    line = {
        "metric": "GB/s of the fused norm ops (BASELINE config 2) vs the HBM roofline",
        "value": min(norm_gbs, qk_gbs),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": max(args.steps, 100),
        "warmup": "one discarded pass of the same calls per op",
        "higher_is_better": True,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "BASELINE config 2 (i) rms_norm_modulate x bf16 [2,4096,3072] -> bf16, "
                               "(ii) qk_norm_rope Q and K bf16 [2,4352,3072] -> [2,24,4352,128]",
                   "l2": "flushed before every timed call (512 MB write, then a 256 MB read)"},  # fmt: skip
        "ops": {
            "rms_norm_modulate": {"us": norm_ms * 1e3, "bytes": norm_bytes, "gbs": norm_gbs,
                                  "frac": norm_gbs / pk["hbm_gbs"]},  # fmt: skip
            "qk_norm_rope_pair": {"us": qk_ms * 1e3, "bytes": qk_bytes, "gbs": qk_gbs, "frac": qk_gbs / pk["hbm_gbs"]},
        },
        "roofline": {"bound": "hbm", "achieved": min(norm_gbs, qk_gbs), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": min(norm_gbs, qk_gbs) / pk["hbm_gbs"], "traffic": None,
                     "peak_source": f"{pk['source']} hbm copy"},  # fmt: skip
    }
    print(json.dumps(line), flush=True)


def attention_compare(args) -> None:
    """The config-3 attention (B = 2, 24 heads x 128, 4352 joint tokens, QK-normed
    rows as in the model) through this library's tcgen05 kernel (with and without
    the QK-norm score bound) and through the library kernels the reference's
    attention call site would reach on this box (src/iris3b/nn/attention.py:61-91:
    F.scaled_dot_product_attention, and the flash_attn backend): torch SDPA with
    the cuDNN and flash backends, flash_attn 2. Each launch after an L2 flush
    (the operands, 160 MB, exceed L2 anyway), CUDA events on the stream, the mean
    of ``max(steps, 20)`` launches after ``warmup``."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from iris_b200 import kernels as K

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    B, H, N, D = 2, 24, 4352, 128
    g = torch.Generator(device=device).manual_seed(3)
    gains = [1 + 0.02 * torch.randn(D, generator=g, device=device) for _ in range(2)]
    q, k = (F.rms_norm(torch.randn(B, H, N, D, generator=g, device=device), (D,), gn, 1e-6).to(torch.bfloat16)
            for gn in gains)  # fmt: skip
    v = torch.randn(B, H, N, D, generator=g, device=device).to(torch.bfloat16)
    out = torch.empty(B * N, H * D, device=device, dtype=torch.bfloat16)
    bound = K.score_bound([gains[0]], [gains[1]])
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)
    flops = 4.0 * B * H * N * N * D
    reps = max(args.steps, 20)

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        times = []
        for _ in range(reps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            times.append((s, e))
        torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in times)
        return {"us": ms * 1e3, "tflops": flops / (ms / 1e3) / 1e12}

    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float()).transpose(1, 2).reshape(B * N, H * D)
    results, errors = {}, {}

    def check(name, o):
        errors[name] = float((o.float() - ref).abs().max() / ref.abs().max())

    K.flash_attention(q, k, v, out.view(B, N, H * D))
    check("iris_tcgen05", out)
    results["iris_tcgen05_score_bound"] = timed(lambda: K.flash_attention(q, k, v, out.view(B, N, H * D), bound=bound))
    results["iris_tcgen05"] = timed(lambda: K.flash_attention(q, k, v, out.view(B, N, H * D)))
    for name, backend in (("torch_sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("torch_sdpa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel(backend):
                check(name, F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B * N, H * D))
                results[name] = timed(lambda: F.scaled_dot_product_attention(q, k, v))
        except RuntimeError as exc:
            results[name] = {"unavailable": str(exc).splitlines()[0][:200]}
    try:
        from flash_attn import flash_attn_func

        qt, kt, vt = (t.transpose(1, 2).contiguous() for t in (q, k, v))
        check("flash_attn2", flash_attn_func(qt, kt, vt).reshape(B * N, H * D))
        results["flash_attn2"] = timed(lambda: flash_attn_func(qt, kt, vt))
    except Exception as exc:  # noqa: BLE001 - report, do not fail the comparison
        results["flash_attn2"] = {"unavailable": f"{type(exc).__name__}: {str(exc)[:200]}"}
    pk = peaks()
    best = max((r["tflops"] for n, r in results.items() if "tflops" in r and not n.startswith("iris")), default=None)
    ours = results["iris_tcgen05_score_bound"]["tflops"]
    line = {
        "metric": "TFLOP/s of the config-3 joint attention (B=2, 24 heads x 128, N=4352) vs library kernels",
        "value": ours,
        "unit": "TFLOP/s",
        "n_gpus": 1,
        "steps": reps,
        "warmup": max(args.warmup, 3),
        "higher_is_better": True,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "one attention launch, q/k RMS-normed rows (gains 1 + N(0, 0.02)), v ~ N(0, 1)",
                   "l2": "flushed before every launch (256 MB write)"},  # fmt: skip
        "results": results,
        "max_rel_err_vs_fp32": errors,
        "best_library_tflops": best,
        "roofline": {"bound": "tensor", "achieved": ours, "peak": pk["bf16"], "unit": "TFLOP/s",
                     "frac": ours / pk["bf16"], "traffic": None, "peak_source": f"{pk['source']} bf16 burst"},  # fmt: skip
    }
    print(json.dumps(line), flush=True)


RES_2048 = 2048


def inputs_2048(engine, device):
    """Config 5 inputs: one seeded 2048^2 noise image as the CFG pair, text states
    [uncond; cond] adapted by the engine, model time 625."""
    gen = torch.Generator().manual_seed(1)
    x_h = torch.randn(1, 3, RES_2048, RES_2048, generator=gen).repeat(2, 1, 1, 1).pin_memory()
    states = torch.randn(2, TEXT_LEN, TEXT_DIM, generator=torch.Generator().manual_seed(4)).to(device)
    text = engine.encode_text(states)
    return x_h, text, torch.full((2,), 625.0, device=device)


def time_calls(fn, steps: int, warmup: int, world: int, local: int, device) -> float:
    """ms per ``fn()`` over ``steps`` calls after ``warmup`` untimed ones; CUDA events
    on the current stream, barrier + synchronize on both sides, max over ranks."""
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    ms = s.elapsed_time(e) / steps
    if world > 1:
        m = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    return ms


def measure_2048(engine, single, rank: int, world: int, local: int, steps: int, warmup: int, e2e: bool = False) -> dict:
    """one B = 2 call at 2048^2 per step on ``engine``
    (Ulysses sequence parallel over the ranks when it has a communicator).
    With N > 1, rank 0 also runs the same call on ``single`` (one GPU, no
    communicator) and reports the max relative error of the sequence-parallel
    velocity against it."""
    from iris_b200 import _lib

    device = torch.device("cuda", local)
    x_h, text, t = inputs_2048(engine, device)
    x = x_h.to(device)
    launches0 = _lib.launch_count()
    with ClockSampler(local) as clocks:
        ms = time_calls(lambda: engine(x, t, text), steps, warmup, world, local, device)
    launches = (_lib.launch_count() - launches0) // (steps + warmup)
    flops = step_flops(2, L=(RES_2048 // 16) ** 2)
    pk = peaks()
    per_gpu = flops / world / (ms / 1e3) / 1e12
    record = {
        "ms_per_step": ms,
        "n_gpus": world,
        "parallelism": f"ulysses{world}" if world > 1 else "one GPU",
        "steps": steps,
        "warmup": warmup,
        "step_tflop": flops / 1e12,
        "tflops_per_gpu": per_gpu,
        "frac_of_bf16_sustained": per_gpu / pk["bf16_sustained"],
        "gpu_launches_per_step": launches,
        "clocks": clocks.summary(),
    }
    if e2e:
        text_h = text.cpu().pin_memory()
        v_h = torch.empty_like(x_h).pin_memory()

        def through_host():
            xd = x_h.to(device, non_blocking=True)
            td = text_h.to(device, non_blocking=True)
            v_h.copy_(engine(xd, t, td), non_blocking=True)

        record["e2e_ms"] = time_calls(through_host, steps, warmup, world, local, device)
        record["h2d_bytes_per_step"] = x_h.numel() * 4 + text_h.numel() * 4
        record["d2h_bytes_per_step"] = v_h.numel() * 4
    if world > 1:
        import torch.distributed as dist

        v = engine(x, t, text)
        if rank == 0:
            ref = single(x, t, text)
            err = float((v.double() - ref.double()).abs().max() / ref.double().abs().max())
            record["max_rel_err_vs_one_gpu"] = err
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
    return record


def measure_restore(engine, rank: int, world: int, local: int, steps: int, warmup: int) -> dict:
    """The restoration / 4x upscaling task at the reference's largest budgeted
    image (a 512 x 1024 input, 2048 x 4096 output: 21 overlapping 1024^2 tiles,
    src/iris3b/downstream/restoration.py:18-21,104-107), tiles split over the
    ranks, Gaussian-window fusion, one sum all-reduce of the image at the end.
    Synthetic input and prompt (random weights, random adapted text)."""
    import torch.distributed as dist

    from iris_b200.restoration import TiledRestorer, tile_plan

    device = torch.device("cuda", local)
    gen = torch.Generator().manual_seed(9)
    x = (torch.rand(1, 3, 2048, 4096, generator=gen) * 2 - 1).to(device)
    states = torch.randn(1, TEXT_LEN, TEXT_DIM, generator=torch.Generator().manual_seed(10)).to(device)
    group = dist.group.WORLD if world > 1 else None
    restorer = TiledRestorer(engine, engine.encode_text(states), sigma=0.5, tile=1024, tiles_per_call=8, group=group)
    tiles, mine = tile_plan(2048, 4096, 1024, rank, world)
    with ClockSampler(local) as clocks:
        ms = time_calls(lambda: restorer(x), steps, warmup, world, local, device)
    return {
        "image": "2048x4096 output (4x of a 512x1024 input)",
        "tiles": len(tiles),
        "tiles_on_busiest_rank": -(-len(tiles) // world),
        "ms_per_image": ms,
        "tiles_per_s": len(tiles) / (ms / 1e3),
        "n_gpus": world,
        "parallelism": f"tiles split over {world} GPU(s)",
        "steps": steps,
        "warmup": warmup,
        "clocks": clocks.summary(),
    }


def step2048(args, rank: int, world: int, local: int) -> None:
    """BASELINE config 5 as the whole bench line (``--workload step2048``)."""
    import torch.distributed as dist

    from iris_b200 import CudaIris, IrisWeights, baseline_step_config, synthetic_state
    from iris_b200.parallel import init_process_group
    from iris_b200.ulysses import TorchComm

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    comm = None
    if world > 1:
        init_process_group("nccl", timeout_s=600)
        comm = TorchComm()
    cfg = baseline_step_config()
    weights = IrisWeights(cfg, synthetic_state(cfg, device, seed=0))
    engine = CudaIris(weights, comm=comm)
    single = CudaIris(weights) if world > 1 and rank == 0 else None
    rec = measure_2048(engine, single, rank, world, local, args.steps, args.warmup, e2e=True)
    engine.close()
    if rank != 0:
        dist.destroy_process_group()
        return
    pk = peaks()
    ms = rec["ms_per_step"]
    line = {
        "metric": "ms per denoise step at 2048² (B=2 CFG), Ulysses sequence parallel over N B200",
        "value": ms,
        "unit": "ms",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {
            "workload": "BASELINE config 5: one guided denoiser call (B=2: [uncond; cond]) at 2048^2, t = 625, "
            "tokens split across N GPUs (Ulysses: the producing kernels store Q/K/V and attention rows into "
            "the owning rank's memory over NVLink)",
            "model": MODEL,
            "global_batch": 2,
            "seq_len": 256 + (RES_2048 // 16) ** 2,
            "parallelism": f"ulysses{world}",
            "l2": "no flush: every step streams 8.7 GB of weights, far above the 126 MB L2",
        },
        "roofline": {
            "kernel": "whole step (GEMMs + attention), per GPU",
            "bound": "tensor",
            "achieved": rec["tflops_per_gpu"],
            "peak": pk["bf16_sustained"],
            "unit": "TFLOP/s",
            "frac": rec["frac_of_bf16_sustained"],
            "traffic": None,
            "peak_source": f"{pk['source']} bf16 sustained",
        },
        "e2e": {"value": rec["e2e_ms"], "unit": "ms", "h2d_bytes_per_step": rec["h2d_bytes_per_step"],
                "d2h_bytes_per_step": rec["d2h_bytes_per_step"]},  # fmt: skip
        "gpu_launches": rec["gpu_launches_per_step"] * args.steps,
        "clocks": rec["clocks"],
    }
    if "max_rel_err_vs_one_gpu" in rec:
        line["max_rel_err_vs_one_gpu"] = rec["max_rel_err_vs_one_gpu"]
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--profile", choices=["forward", "small", "sampler", "forward16", "small16"],
                        help="NVTX-marked work for ncu")  # fmt: skip
    parser.add_argument("--workload", default="loop1024", choices=["loop1024", "step2048", "ops", "attention"])
    args = parser.parse_args()
    from iris_b200.parallel import env_world, gather_images, image_shard, init_process_group  # noqa: F401

    rank, world, local = env_world()
    if args.profile:
        profile_run(args.profile)
        return
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    args.warmup = max(args.warmup, 3)
    if args.workload == "step2048":
        step2048(args, rank, world, local)
        return
    if args.workload == "ops":
        if rank == 0:
            fused_ops(args)
        return
    if args.workload == "attention":
        if rank == 0:
            attention_compare(args)
        return
    import torch.distributed as dist

    from iris_b200 import CudaIris, IrisWeights, _lib, baseline_step_config, synthetic_state
    from iris_b200 import kernels as K
    from iris_b200.pipeline import DenoisePipeline
    from iris_b200.sampling import euler_cfg

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        init_process_group("nccl", timeout_s=600)
    cfg = baseline_step_config()
    weights = IrisWeights(cfg, synthetic_state(cfg, device, seed=0))
    engine = CudaIris(weights, graphs=True)  # each call geometry replays one CUDA graph
    noise, cond_states, uncond_states = make_inputs()
    lo, hi = image_shard(IMAGES, rank, world)
    noise_d = noise[lo:hi].to(device)
    cond = engine.encode_text(cond_states[lo:hi].to(device))
    uncond = engine.encode_text(uncond_states.to(device))

    def step():
        return euler_cfg(engine, noise_d, cond, uncond, cfg_scale=CFG_SCALE, sigmas=SIGMAS)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------------------------------------------------------- device-resident
    # GEMM timing is on before the warm-up: the graph captured in it carries an event
    # pair around every GEMM, recorded again by each replay in the timed region
    K.profile_gemms(True)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = (_lib.launch_count() - launches0) // args.steps
    gemm_flops, gemm_ms, gemm_n, gemm_bytes = K.profile_gemms(False)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    value = IMAGES / (ms / 1e3)

    # ------------------------------------------------------- e2e through the public API
    pipe = DenoisePipeline(engine, cfg_scale=CFG_SCALE, sigmas=SIGMAS)
    noise_h = noise[lo:hi].pin_memory()
    cond_h = cond_states[lo:hi].pin_memory()
    uncond_h = uncond_states.pin_memory()
    out_h = torch.empty_like(noise_h).pin_memory()
    for _ in range(args.warmup):
        pipe(noise_h, cond_h, uncond_h, out=out_h)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        pipe(noise_h, cond_h, uncond_h, out=out_h)
    e_end.record()
    torch.cuda.synchronize()
    barrier()
    e_ms = max_over_ranks(e_start.elapsed_time(e_end) / args.steps)
    h2d = sum(t.numel() * t.element_size() for t in (noise_h, cond_h, uncond_h))
    d2h = out_h.numel() * out_h.element_size()

    # ---------------------------------------------------- one B = 2 denoiser call (rank 0)
    b2 = None
    if rank == 0:
        x2 = noise_d[:1].repeat(2, 1, 1, 1)
        text2 = torch.cat([uncond, cond[:1]])
        t2 = torch.full((2,), 625.0, device=device)
        with ClockSampler(local) as b2_clocks:
            b2_ms = time_calls(lambda: engine(x2, t2, text2), 10, 3, 1, local, device)
        b2_tflops = step_flops(2) / (b2_ms / 1e3) / 1e12
        b2 = {"ms": b2_ms, "tflop": step_flops(2) / 1e12, "tflops": b2_tflops,
              "frac_of_bf16_burst": b2_tflops / peaks()["bf16"], "calls": 10, "warmup": 3,
              "clocks": b2_clocks.summary()}  # fmt: skip

    # ------------------------------------- BASELINE config 5 (2048^2) on the same N GPUs
    sp_engine = engine
    if world > 1:
        from iris_b200.ulysses import TorchComm

        sp_engine = CudaIris(weights, comm=TorchComm())
    step2048_rec = measure_2048(sp_engine, engine, rank, world, local, min(args.steps, 5), 3)
    if sp_engine is not engine:
        sp_engine.close()
        del sp_engine

    # -------------------------------------- tiled 4x restoration (21 tiles) on the same N GPUs
    restore_rec = measure_restore(engine, rank, world, local, 2, 1)

    pk = peaks()
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        base = cpu_baseline_sample(threads)
        cpu = {
            "value": base["images_per_s"],
            "unit": UNIT,
            "cores": threads,
            "kind": "port",
            "sample": "oracle fp32 PyTorch path on the host, one dual + one single + one pixel block at B=2 1024^2 "
            f"(s: {', '.join(f'{k} {v:.2f}' for k, v in base['seconds'].items())}), extrapolated to 4 guided "
            "calls per image",
        }
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": bench_config(world),
        "roofline": {
            "kernel": "gemm_bf16_pair_kernel (tcgen05 cta_group::2): the GEMM launches of the timed region's last "
            "denoiser call, each bracketed by CUDA events recorded by the call's graph replay",
            "bound": "tensor",
            "achieved": achieved,
            "peak": pk["bf16_sustained"],
            "unit": "TFLOP/s",
            "frac": (achieved / pk["bf16_sustained"]) if achieved else None,
            "traffic": GEMM_TRAFFIC_PER_LAUNCH if world == 1 else None,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of each GEMM kind of a "
            "16-row call (small model, same shapes), weighted by the full model's launch counts; bytes per launch",
            "algorithmic_bytes_per_launch": gemm_bytes / gemm_n if gemm_n else None,
            "launches": gemm_n,
            "peak_source": f"{pk['source']} bf16 sustained",
        },
        "e2e": {"value": IMAGES / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches * args.steps,
        "clocks": clocks.summary(),
        "denoise_step_b2": b2,
        "step2048": step2048_rec,
        "restore_4x": restore_rec,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
