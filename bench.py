#!/usr/bin/env python
"""Headline benchmark: one Qwen-Image-style dual-stream DiT denoiser step at
1024x1344 in bf16 (benchmark configuration 3: 60 blocks x 3072, 24 heads,
MLP 12288, 5376 image + 256 text tokens), per B200, images sharded one per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg3|cfg1|cfg2|cfg4|cfg5]

Under torchrun (N > 1) each rank drives its own GPU with its own image; the
only collective is the final NCCL gather of the predicted latents to rank 0.
Rank 0 prints ONE JSON line.

  value   images/s over all ranks, one denoiser step per image, inputs
          already in HBM (device-resident predict replaying the captured step)
  e2e     the same metric through the host C-ABI predict (latent + context
          copied in from pinned host memory, the prediction copied back)
  roofline  the dominant kernel class (the tcgen05 GEMMs -- and for the UNet
          the implicit-GEMM convolutions) from per-launch CUDA events of a
          profiled step
  cpu_baseline  the CPU oracle (C++ restatement of the reference's CPU
          layer arithmetic) on a bounded sample: one block at full size,
          extrapolated to a step

--config picks another benchmark configuration for the same line (default
cfg3, the headline): cfg1 one Anima block in fp32, cfg2 the 28-block Anima
step (two CFG branches), cfg4 cfg3 with int8 per-channel weights, cfg5 the
SDXL UNet (fp16, two CFG branches), vae the SDXL VAE decoder (a 128 x 128
latent to a 1024 x 1024 image; not a benchmark configuration: the step after
the denoiser).

--impl reference times that CPU restatement alone (the reference is C# over
DirectML and cannot run here or on the GPU box); rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Qwen-Image-style DiT s/step @1024×1344 bf16; images/s at 1/2/4/8 B200"
UNIT = "images/s (one denoiser step per image)"


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sustained=d["bf16_tflops_sustained"],
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


class Clocks:
    """nvidia-smi samples of SM clock / throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        if not shutil.which("nvidia-smi"):
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.proc = subprocess.Popen(
            ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
             "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)

    def stop(self) -> dict | None:
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(",") for r in Path(self.path).read_text().splitlines() if r.strip()]
        os.unlink(self.path)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _configs():
    """benchmark configurations: (model config, workload text, dtype, metric)."""
    from naivediffusion_b200 import _lib
    from naivediffusion_b200.denoiser import (AnimaConfig, MMDiTConfig, QwenImageConfig, UNetConfig,
                                              VaeDecoderConfig, WanVaeConfig)
    return {
        "cfg3": (MMDiTConfig(), "cfg3: Qwen-Image-style MMDiT 60x3072, 24x128 heads, MLP 12288 GELU-tanh, "
                 "5376 img + 256 txt tokens, batch 1, guidance 1", "bf16", METRIC),
        "cfg4": (MMDiTConfig(weight_dtype=_lib.ND_I8, quant_group=0, quant_scale_dtype=_lib.ND_F32),
                 "cfg4: cfg3 with int8 weight-only storage, per-output-channel fp32 scales (absmax/127), "
                 "dequant fused into the GEMM mainloop, batch 1", "bf16 (int8 weights)",
                 "Qwen-Image-style DiT int8 weight-only s/step @1024×1344; images/s"),
        "cfg2": (AnimaConfig(), "cfg2: Anima 28x2048, 16x128 heads, MLP 8192 GELU, 4096 tokens per image, "
                 "cross-attention to 256x1024, batch 2 (CFG branches of one image)", "bf16",
                 "Anima DiT s/step @1024×1024 bf16 (2 CFG branches); images/s"),
        "cfg1": (AnimaConfig(blocks=1, latent_height=64, latent_width=64, batch=1, compute=_lib.ND_F32),
                 "cfg1: one Anima block 2048 wide, 16x128 heads, 1024 tokens, cross-attention to 256x1024, "
                 "MLP 8192, fp32 compute (bf16 hi|lo operand pairs on the tensor cores, fp32 attention), "
                 "with the embedder and final layer", "f32",
                 "Anima DiT block fp32 s/step (1024 tokens); blocks/s"),
        "cfg5": (UNetConfig(), "cfg5: SDXL UNet 320/640/1280, transformer depths 0/2/10, 4x128x128 latent, "
                 "context 77x2048, add 2816, batch 2 (CFG branches of one image)", "f16",
                 "SDXL UNet s/step @1024×1024 fp16 (2 CFG branches); images/s"),
        "vae": (VaeDecoderConfig(), "SDXL VAE decoder (AutoencoderKL 128/256/512/512, 2 layers per block): "
                "4x128x128 latent -> 3x1024x1024 image, fp16", "f16",
                "SDXL VAE decode s/image @1024×1024 fp16; images/s"),
        "qwen21": (QwenImageConfig(), "Qwen-Image 2.1 single-stream DiT (the reference's own QwenImageDit): "
                   "32x4096, 32x128 heads, SwiGLU 12288, 4096 img + 256 txt tokens (1024x1024), batch 1, "
                   "fp16 compute (the reference's half-precision option)", "f16",
                   "Qwen-Image 2.1 DiT s/step @1024×1024 fp16; images/s"),
        "wan21": (WanVaeConfig(), "Wan 2.1 VAE decoder on one frame (Anima's): widths 384/192/96, "
                  "16x128x128 latent -> 3x1024x1024 image, fp16", "f16",
                  "Wan 2.1 VAE decode s/image @1024×1024 fp16; images/s"),
        "wan22": (WanVaeConfig(version=22, width=144, latent_channels=64, latent_height=64, latent_width=64),
                  "Qwen-Image 2.1's Wan 2.2-layout VAE decoder on one frame: widths 1152/576/288/144, "
                  "64x64x64 latent -> 3x1024x1024 image, fp16", "f16",
                  "Qwen-Image 2.1 VAE decode s/image @1024×1024 fp16; images/s"),
    }


def _inputs(cfg, rank):
    """Seeded device inputs of one step: latent, conditioning dict, timestep."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    b = getattr(cfg, "batch", 1)
    latent = torch.randn(b, cfg.latent_channels, cfg.latent_height, cfg.latent_width, device="cuda", generator=g)
    cond = {}
    if hasattr(cfg, "context_rows"):
        cond["context"] = torch.randn(b, cfg.context_rows, cfg.context_width, device="cuda", generator=g)
    if hasattr(cfg, "add_width"):
        cond["add"] = torch.randn(b, cfg.add_width, device="cuda", generator=g)
    return latent, cond, 500.0


def host_cpu() -> dict:
    """The host the CPU baseline ran on: CPU model, logical CPUs, and the
    oracle's OpenMP thread count."""
    import oracle as O
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count(), "omp_threads": O.threads()}


def _timed(fn, repeats: int, budget_s: float) -> list:
    """Time fn() up to `repeats` times, stopping early once `budget_s` is spent."""
    times = []
    t_start = time.perf_counter()
    for _ in range(max(1, repeats)):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    return times


def cpu_block_sample(cfg, repeats: int = 1, budget_s: float = 150.0):
    """Time one full-size dual-stream block on the CPU oracle (the reference's
    CPU layer arithmetic, all host threads). Returns (per-sample seconds,
    step / sample FLOP ratio, description)."""
    import oracle as O
    import torch
    D, F, N, ni = cfg.width, cfg.mlp_width, cfg.tokens, cfg.image_tokens
    torch.manual_seed(0)
    g = lambda *s: (torch.randn(*s) * 0.02).numpy()  # noqa: E731
    streams = []
    for _ in range(2):
        streams.append(dict(mod_w=g(6 * D, D), mod_b=g(6 * D), q_w=g(D, D), q_b=g(D), k_w=g(D, D), k_b=g(D),
                            v_w=g(D, D), v_b=g(D), norm_q=1 + g(128), norm_k=1 + g(128), out_w=g(D, D), out_b=g(D),
                            up_w=g(F, D), up_b=g(F), down_w=g(D, F), down_b=g(D)))
    x = torch.randn(N, D).numpy()
    temb = torch.randn(D).numpy()
    cs, sn = O.qwen_rope_tables(cfg.latent_height // 2, cfg.latent_width // 2, cfg.context_rows, cfg.context_rows)
    times = _timed(lambda: O.mmdit_block(streams[0], streams[1], x, ni, temb, cs, sn, cfg.heads), repeats, budget_s)
    block_flops = 2.0 * (N * (4 * D * D + 2 * D * F) + 2 * N * N * D + 2 * 6 * D * D)
    scale = cfg.flops_per_step() / block_flops
    return times, scale, (f"one full-size dual-stream block ({N} tokens, width {D}) on the CPU oracle, "
                          f"{len(times)} sample(s), extrapolated x{scale:.2f} by FLOPs to a {cfg.blocks}-block step")


def cpu_anima_sample(cfg, repeats: int = 1, budget_s: float = 150.0):
    """One full-size Anima block (batch 1, with the embedder and final layer)
    through the CPU oracle's AnimaDit step, extrapolated by FLOPs to the
    configuration's whole step (x blocks x batch)."""
    import numpy as np
    import oracle as O
    from dataclasses import replace
    from naivediffusion_b200.denoiser import synthetic_weights
    one = replace(cfg, blocks=1, batch=1)
    w = dict(synthetic_weights(one, seed=0))
    rng = np.random.default_rng(0)
    lat = rng.standard_normal((1, 16, one.latent_height, one.latent_width)).astype(np.float32)
    ctx = rng.standard_normal((1, one.context_rows, one.context_width)).astype(np.float32)
    times = _timed(lambda: O.anima_forward(w, one, lat, ctx, 0.5), repeats, budget_s)
    scale = cfg.flops_per_step() / one.flops_per_step()
    return times, scale, (f"one full-size Anima block ({one.tokens} tokens, width {one.width}, batch 1) through the "
                          f"CPU oracle's step, {len(times)} sample(s)"
                          + (f", extrapolated x{scale:.0f} by FLOPs" if scale > 1 else ""))


def cpu_qwen_image_sample(cfg, repeats: int = 1, budget_s: float = 150.0):
    """One full-size Qwen-Image 2.1 block (with the embeddings and the final
    layer) through the CPU oracle's step, extrapolated by FLOPs to the whole
    step."""
    import numpy as np
    import oracle as O
    from dataclasses import replace
    from naivediffusion_b200.denoiser import synthetic_weights
    one = replace(cfg, blocks=1)
    w = dict(synthetic_weights(one, seed=0))
    rng = np.random.default_rng(0)
    lat = rng.standard_normal((1, one.latent_channels, one.latent_height, one.latent_width)).astype(np.float32)
    ctx = rng.standard_normal((one.context_rows, one.context_width)).astype(np.float32)
    times = _timed(lambda: O.qwen_image_forward(w, one, lat, ctx, 0.5), repeats, budget_s)
    scale = cfg.flops_per_step() / one.flops_per_step()
    return times, scale, (f"one full-size Qwen-Image 2.1 block ({one.tokens} tokens, width {one.width}) with the "
                          f"embeddings and final layer through the CPU oracle's step, {len(times)} sample(s), "
                          f"extrapolated x{scale:.1f} by FLOPs to the {cfg.blocks}-block step")


def cpu_unet_sample(cfg, repeats: int = 1, budget_s: float = 150.0):
    """The SDXL UNet's two dominant units at full size and batch 1 through the
    CPU oracle: a level-0 ResBlock (320 -> 320 channels over 128 x 128) and a
    level-1 Transformer2d with one block (640 wide over 64 x 64, 10 heads,
    cross-attention to 77 x 2048), extrapolated by FLOPs to the step."""
    import numpy as np
    import oracle as O
    from dataclasses import replace
    from naivediffusion_b200.denoiser import synthetic_weights
    one = replace(cfg, depth=(0, 1, 1), batch=1)
    res, t2d = "down_blocks.0.resnets.0", "down_blocks.1.attentions.0"
    w = dict(synthetic_weights(one, seed=0, only=(res + ".", t2d + ".")))
    rng = np.random.default_rng(0)
    c0, c1 = cfg.width * cfg.mult[0], cfg.width * cfg.mult[1]
    h, wd = cfg.latent_height, cfg.latent_width
    x0 = rng.standard_normal((c0, h, wd)).astype(np.float32)
    x1 = rng.standard_normal((c1, h // 2, wd // 2)).astype(np.float32)
    temb = rng.standard_normal(1280).astype(np.float32)
    ctx = rng.standard_normal((cfg.context_rows, cfg.context_width)).astype(np.float32)

    def run():
        O.unet_resblock(w, res, x0, temb)
        O.unet_transformer2d(w, t2d, x1, ctx)

    times = _timed(run, repeats, budget_s)
    sample_flops = one.resblock_flops(c0, c0, h * wd) + one.transformer2d_flops(c1, h * wd // 4, 1)
    scale = cfg.flops_per_step() / sample_flops
    return times, scale, (f"a level-0 ResBlock ({c0} ch, {h}x{wd}) and a level-1 Transformer2d block ({c1} ch, "
                          f"{h // 2}x{wd // 2}, 77 context rows) at batch 1 on the CPU oracle, {len(times)} sample(s), "
                          f"extrapolated x{scale:.1f} by FLOPs to the batch-{cfg.batch} UNet step")


def cpu_sample(name, cfg, repeats=1, budget_s=150.0):
    """(per-sample seconds, step / sample ratio, description) or None."""
    if name == "qwen21":
        return cpu_qwen_image_sample(cfg, repeats, budget_s)
    if name in ("cfg3", "cfg4"):
        return cpu_block_sample(cfg, repeats, budget_s)
    if name in ("cfg1", "cfg2"):
        return cpu_anima_sample(cfg, repeats, budget_s)
    if name == "cfg5":
        return cpu_unet_sample(cfg, repeats, budget_s)
    return None  # the VAE decoders: no bounded sample is timed


def run_reference(args):
    """The reference's CPU layer path (the oracle port) on the host cores.
    Each timed step is one bounded sample of the workload (one full-size
    block, or the UNet's two dominant units); `value` extrapolates the median
    sample by FLOPs to one whole denoiser step per image."""
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    cfg, workload, _dt, metric = _configs()[args.config]
    if args.config in ("vae", "wan21", "wan22"):
        print(json.dumps({"impl": "reference", "unavailable": f"{args.config} has no bounded CPU sample of the step"}))
        return 0
    for _ in range(args.warmup):
        cpu_sample(args.config, cfg, 1, 1e9)
    times, scale, sample = cpu_sample(args.config, cfg, args.steps, 120.0)
    per_sample = statistics.median(times)
    per_step = per_sample * scale
    value = 1.0 / per_step
    host = host_cpu()
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": len(times), "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": per_sample * 1e3,
        "ms_per_image_extrapolated": per_step * 1e3, "sample_fraction_of_step": 1.0 / scale,
        "timed_s": sum(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": workload, "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": host["omp_threads"], "kind": "port",
                         "sample": sample, **host},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "each step is one bounded sample (ms_per_step is what one sample took); value extrapolates the "
                "median sample by FLOPs to one denoiser step per image. The reference is C# over DirectML/D3D12 "
                "(Windows); its CPU layer arithmetic is timed through the C++ restatement in oracle/",
    }
    print(json.dumps(line), flush=True)
    return 0


TEXT_CONFIGS = ("qwen3vl8b", "qwen3", "adapter")


def _text_config(name):
    """The text towers (the step before the path): Qwen3-VL-8B's language
    model as Qwen-Image 2.1 reads it, Qwen3-0.6B as Anima reads it, Anima's
    LLM adapter. A step is one prompt of PROMPT_ROWS tokens."""
    from naivediffusion_b200.denoiser import LlmAdapterConfig, Qwen3TextConfig
    if name == "qwen3vl8b":
        return (Qwen3TextConfig.qwen3_vl_8b(context_rows=512), "Qwen3-VL-8B language model as Qwen-Image 2.1's "
                "text encoder (36 x 4096, 32 x 128 query heads over 8 key heads, SwiGLU 12288), one 300-token "
                "prompt, bf16", "Qwen-Image 2.1 text encode s/prompt (300 tokens); prompts/s")
    if name == "qwen3":
        return (Qwen3TextConfig(context_rows=512), "Qwen3-0.6B as Anima's text encoder (28 x 1024, 16 x 128 "
                "query heads over 8 key heads, SwiGLU 3072), one 300-token prompt, bf16",
                "Anima Qwen3 text encode s/prompt (300 tokens); prompts/s")
    return (LlmAdapterConfig(context_rows=512, source_rows=512), "Anima's LLM adapter (6 x 1024, 16 x 64 "
            "heads, GELU 4096): 300 T5 ids cross-attending to 300 Qwen3 rows, bf16",
            "Anima LLM adapter s/prompt (300 ids); prompts/s")


PROMPT_ROWS = 300


def run_text(args):
    """Text towers: e2e = nd_text_encode from host ids to host hidden states;
    value = the device time of the same forward (event pairs per launch)."""
    import numpy as np
    import torch
    from naivediffusion_b200.denoiser import CudaDenoiser, Device, synthetic_weights_device

    rank, world, local = env_rank()
    if rank != 0:
        return 0  # one prompt per call: replicas only, rank 0 reports
    torch.cuda.set_device(local)
    cfg, workload, metric = _text_config(args.config)
    dev = Device(local)
    den = CudaDenoiser(dev, cfg.desc())
    for name, t in synthetic_weights_device(cfg, seed=0):
        den.set_weight(name, t)
    den.finalize()
    rng = np.random.default_rng(0)
    ids = rng.integers(0, cfg.vocab, PROMPT_ROWS).astype(np.int32)
    src = rng.standard_normal((PROMPT_ROWS, cfg.width)).astype(np.float32) if args.config == "adapter" else None
    for _ in range(max(3, args.warmup)):
        y = den.text_encode(ids, source=src)
    clocks = Clocks(local)
    clocks.start()
    step_s = []
    for _ in range(args.steps):
        t1 = time.perf_counter()
        y = den.text_encode(ids, source=src)
        step_s.append(time.perf_counter() - t1)
    clk = clocks.stop()
    prof = den.profile(steps=max(1, args.steps))
    dev_ms = sum(p["ms"] for p in prof)
    gemm = [p for p in prof if p["name"].startswith("gemm")]
    g_ms, g_fl = sum(p["ms"] for p in gemm), sum(p["flops"] for p in gemm)
    peaks = measured_peaks()
    e2e_ms = statistics.median(step_s) * 1e3
    line = {
        "metric": metric, "value": 1e3 / dev_ms, "unit": "prompts/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) weights on device, random ids)",
        "config": {"workload": workload, "global_batch": 1, "prompt_rows": PROMPT_ROWS},
        "e2e": {"value": 1e3 / e2e_ms, "unit": "prompts/s", "ms_per_step_median": e2e_ms,
                "h2d_bytes_per_step": int(ids.nbytes + (src.nbytes if src is not None else 0)),
                "d2h_bytes_per_step": int(y.nbytes)},
        "gpu_launches": sum(p["launches"] for p in prof),
        "roofline": {"bound": "tensor", "kernel": "gemm_sm100_kernel (tcgen05, all GEMM launches of a prompt)",
                     "achieved": g_fl / (g_ms / 1e3) / 1e12, "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": g_fl / (g_ms / 1e3) / 1e12 / peaks["bf16"], "traffic": None,
                     "peak_source": f"{peaks['source']} bf16 burst",
                     "note": "300 rows per GEMM: weight-streaming (HBM) territory, see gemm_bytes"},
        "kernels": [{k: (round(v, 4) if isinstance(v, float) else v) for k, v in p.items()} for p in prof],
        "clocks": clk, "output_finite": bool(np.isfinite(y).all()),
    }
    print(json.dumps(line), flush=True)
    den.close()
    dev.close()
    return 0


def run_vae_tiled(args):
    """The SDXL VAE's tiled decode of a 1024 x 1024 image, the reference's
    default decode (64-cell tiles overlapping by 8: 3 x 3 tiles of 512 x 512
    pixels, decoded as one batch of 9, then crossfaded). value: device time of
    one decode on device-resident latents; e2e: TiledVaeDecoder.run from a
    host latent to a host image."""
    import numpy as np
    import torch
    from naivediffusion_b200.denoiser import Device, VaeDecoderConfig, synthetic_weights_device
    from naivediffusion_b200.tiled_vae import open_tiled_decoder

    rank, world, local = env_rank()
    if rank != 0:
        return 0  # one image per call: replicas only, rank 0 reports
    torch.cuda.set_device(local)
    cfg = VaeDecoderConfig()
    dev = Device(local)
    weights = dict(synthetic_weights_device(cfg, seed=0))
    dec = open_tiled_decoder(dev, cfg, weights, 1024, 1024)
    del weights
    g = torch.Generator(device="cuda").manual_seed(1000)
    latent = torch.randn(1, 4, 128, 128, device="cuda", generator=g)
    for _ in range(max(3, args.warmup)):
        img = dec.run_device(latent)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        img = dec.run_device(latent)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    lat_h = latent.cpu().numpy()
    y = dec.run(lat_h)
    step_s = []
    for _ in range(args.steps):
        t1 = time.perf_counter()
        y = dec.run(lat_h)
        step_s.append(time.perf_counter() - t1)
    same = bool(np.array_equal(y, img.cpu().numpy()))
    prof = dec.model.profile(steps=3)
    conv = [p for p in prof if p["name"].startswith("gemm") or p["name"] == "conv3x3"]
    c_ms, c_fl = sum(p["ms"] for p in conv), sum(p["flops"] for p in conv)
    peaks = measured_peaks()
    e2e_ms = statistics.median(step_s) * 1e3
    line = {
        "metric": "SDXL VAE tiled decode s/image @1024×1024 fp16 (the reference's default decode); images/s",
        "value": 1e3 / ms, "unit": "images/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,0.02) weights on device, N(0,1) latent)",
        "config": {"workload": f"SDXL VAE decoder, 4x128x128 latent -> 3x1024x1024 image in {dec.tile_count} tiles "
                   f"of {dec.tile_side}x{dec.tile_side} (rows {dec.rows}, columns {dec.cols} in latent cells), "
                   "one batch", "global_batch": 1, "tiles": dec.tile_count},
        "e2e": {"value": 1e3 / e2e_ms, "unit": "images/s", "ms_per_step_median": e2e_ms,
                "h2d_bytes_per_step": int(lat_h.nbytes), "d2h_bytes_per_step": int(y.nbytes)},
        "e2e_matches_device_path": same,
        "gpu_launches": sum(p["launches"] for p in prof) + 2,
        "roofline": {"bound": "tensor", "kernel": "gemm_sm100_kernel (conv3x3 implicit GEMM + 1x1 / attention GEMMs)",
                     "achieved": c_fl / (c_ms / 1e3) / 1e12, "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": c_fl / (c_ms / 1e3) / 1e12 / peaks["bf16"], "traffic": None,
                     "peak_source": f"{peaks['source']} bf16 burst (fp16 dense taken as equal)"},
        "kernels": [{k: (round(v, 4) if isinstance(v, float) else v) for k, v in p.items()} for p in prof],
        "clocks": clk, "output_finite": bool(np.isfinite(y).all()),
    }
    print(json.dumps(line), flush=True)
    dec.close()
    dev.close()
    return 0


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from dataclasses import replace

    from naivediffusion_b200.denoiser import CudaDenoiser, Device, synthetic_weights_device
    from naivediffusion_b200.multigpu import CfgPair, gather_latents, max_over_ranks

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    cfg, workload, dtype, metric = _configs()[args.config]
    pair = None
    if args.cfg_pairs:
        # Two ranks per image, one CFG branch each (batch-1 denoisers), one
        # exchange of the predictions per step inside the pair.
        if getattr(cfg, "batch", 1) != 2 or world < 2 or world % 2:
            raise SystemExit("--cfg-pairs needs a two-branch configuration (cfg2, cfg5) and an even rank count")
        pair = CfgPair(rank, world)
        cfg = replace(cfg, batch=1)
    images = world // 2 if pair else world
    dev = Device(local)
    den = CudaDenoiser(dev, cfg.desc())
    for name, t in synthetic_weights_device(cfg, seed=0):
        den.set_weight(name, t)
    den.finalize()
    torch.cuda.synchronize()

    # One explicit stream for the inputs, the library's launches and the
    # timing events (a null stream handle would mean the library's own
    # stream, which the events below would not be ordered with).
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    if pair:
        # both ranks of a pair draw the image's two-branch inputs from the
        # image's seed and keep their own branch
        full, _, _, _ = _configs()[args.config]
        latent, cond, timestep = _inputs(full, pair.image)
        latent = latent[pair.branch:pair.branch + 1].contiguous()
        cond = {k: v[pair.branch:pair.branch + 1].contiguous() for k, v in cond.items()}
    else:
        latent, cond, timestep = _inputs(cfg, rank)
    out = torch.empty(den.output_shape(tuple(latent.shape)), device="cuda")
    both = torch.empty((2,) + tuple(out.shape[1:]), device="cuda") if pair else None
    sigma = 0.75

    def step_device():
        den.predict_device(latent, timestep, sigma, cond, out, stream=stream.cuda_stream)
        if pair:
            pair.exchange(out, both)  # [uncond, cond] on both ranks of the pair

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    # ---- device-resident step (the kernels' number)
    for _ in range(max(3, args.warmup)):
        step_device()
    barrier()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_device()
    gathered = gather_latents(out, world)  # the replicas' one collective (world > 1)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    total_ms = max_over_ranks(e0.elapsed_time(e1), device="cuda")
    ms_per_step = total_ms / args.steps
    value = images * args.steps / (total_ms / 1e3)
    finite = bool(all(torch.isfinite(g).all().item() for g in gathered))
    pair_same = None
    if pair:
        # the two ranks of a pair hold the same [uncond, cond] stack
        stacks = gather_latents(both, world)
        pair_same = all(torch.equal(stacks[2 * i], stacks[2 * i + 1]) for i in range(world // 2))
    # which GPUs the ranks drove (by UUID), as NCCL saw the job
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    if world > 1:
        uuids = [None] * world
        dist.all_gather_object(uuids, uuid)
    else:
        uuids = [uuid]

    # ---- end to end through the host C ABI (pinned host buffers)
    lat_h = torch.empty(latent.shape, dtype=torch.float32, pin_memory=True)
    lat_h.copy_(latent.cpu())
    cond_h = {}
    for k, v in cond.items():
        h = torch.empty(v.shape, dtype=torch.float32, pin_memory=True)
        h.copy_(v.cpu())
        cond_h[k] = h.numpy()
    out_h = torch.empty(tuple(out.shape), dtype=torch.float32, pin_memory=True)
    lat_np, y = lat_h.numpy(), out_h.numpy()
    pair_io = None
    if pair:
        # the exchange needs the prediction on the device: pinned host -> device,
        # exchange, both branches back to pinned host memory
        pair_io = (torch.empty(tuple(out.shape), device="cuda"),
                   torch.empty(tuple(both.shape), dtype=torch.float32, pin_memory=True))

    def step_host():
        den.predict(lat_np, timestep, sigma, cond_h, out=y)
        if pair:
            dev_y, both_h = pair_io
            dev_y.copy_(out_h, non_blocking=True)
            pair.exchange(dev_y, both)
            both_h.copy_(both)

    step_host()
    barrier()
    step_s = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        t1 = time.perf_counter()
        step_host()
        step_s.append(time.perf_counter() - t1)
    e2e_s = max_over_ranks(time.perf_counter() - t0, device="cuda")
    e2e_value = images * args.steps / e2e_s
    same = bool(np.allclose(y, out.cpu().numpy(), rtol=0, atol=0))
    h2d = int(lat_np.nbytes + sum(v.nbytes for v in cond_h.values())) + (int(y.nbytes) if pair else 0)
    d2h = int(y.nbytes) + (int(pair_io[1].numpy().nbytes) if pair else 0)

    # ---- per-kernel-class profile (a captured step with an event pair around every launch)
    prof = den.profile(steps=3)
    launches = sum(p["launches"] for p in prof)
    peaks = measured_peaks()
    tensor_classes = [p for p in prof if p["name"].startswith("gemm") or p["name"] == "conv3x3"]
    g_ms = sum(p["ms"] for p in tensor_classes)
    g_fl = sum(p["flops"] for p in tensor_classes)
    g_n = sum(p["launches"] for p in tensor_classes)
    achieved = g_fl / (g_ms / 1e3) / 1e12
    step_flops = cfg.flops_per_step() if hasattr(cfg, "flops_per_step") else sum(p["flops"] for p in prof)
    long_step = ms_per_step > 50.0
    peak = peaks["bf16_sustained"] if long_step else peaks["bf16"]
    traffic = None
    tpath = ROOT / "profiles" / "gemm_traffic.json"
    if args.config == "cfg3" and tpath.exists():
        traffic = json.loads(tpath.read_text()).get("dram_bytes_per_launch")
    kernel = "gemm2_sm100_kernel (tcgen05 CTA pairs; gemm_sm100_kernel for the small GEMMs; all GEMM launches of a step)"
    if args.config in ("cfg5", "vae", "wan21", "wan22"):
        kernel = ("gemm2_sm100_kernel / gemm_sm100_kernel (tcgen05: conv3x3 implicit GEMMs and the linear layers; "
                  "CTA pairs with 256- or 160-wide tiles over >= 1024 rows)")
    elif args.config == "cfg4":
        kernel = "gemm2_w8_sm100_kernel (tcgen05 CTA pairs, int8 weights widened in the mainloop)"
    elif args.config == "cfg1":
        kernel = ("gemm_sm100_kernel on bf16 hi|lo pairs (3 MMA passes per logical product; "
                  "achieved counts the logical fp32 FLOPs)")

    line = {
        "metric": metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded N(0,0.02) weights generated on device, N(0,1) latent and conditioning)",
        "config": {"workload": workload, "global_batch": images * (2 if pair else getattr(cfg, "batch", 1)),
                   "parallelism": (f"CFG pairs x{images} (two GPUs per image, one branch each, one exchange of "
                                   "the predictions per step)" if pair else
                                   f"replicas x{world} (one image per GPU)"),
                   "l2": "no flush: each step streams its weights and activations, far above the 126 MB L2"},
        "ranks": {"world": world, "backend": dist.get_backend() if world > 1 else None,
                  "gpus_active": len(set(uuids))},
        "e2e": {"value": e2e_value, "unit": UNIT,
                "ms_per_step_median": statistics.median(step_s) * 1e3,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "tensor", "kernel": kernel,
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peaks['source']} bf16 " + ("sustained (kernel timed inside a long step)"
                                                                   if long_step else "burst (short step)"),
                     "launches_per_step": g_n},
        "step_tflops": step_flops / (ms_per_step / 1e3) / 1e12,
        "step_frac_of_peak": step_flops / (ms_per_step / 1e3) / 1e12 / peaks["bf16"],
        "kernels": [{k: (round(v, 4) if isinstance(v, float) else v) for k, v in p.items()} for p in prof],
        "clocks": clk,
        "output_finite": finite, "e2e_matches_device_path": same,
    }
    if args.config in ("cfg3", "cfg4"):
        line["config"]["seq_len"] = cfg.tokens
    if pair:
        line["image_latency_ms"] = ms_per_step
        line["pairs_bit_identical"] = pair_same
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        got = cpu_sample(args.config, cfg, 3, 60.0)
        if got is not None:
            times, scale, sample = got
            host = host_cpu()
            line["cpu_baseline"] = {"value": 1.0 / (statistics.median(times) * scale), "unit": UNIT,
                                    "cores": host["omp_threads"], "kind": "port", "sample": sample,
                                    "samples_s": [round(t, 3) for t in times], **host}
    if rank == 0:
        print(json.dumps(line), flush=True)
    den.close()
    dev.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["cfg3", "cfg1", "cfg2", "cfg4", "cfg5", "vae", "vae_tiled", "qwen21", "wan21",
                                         "wan22", *TEXT_CONFIGS], default="cfg3",
                    help="benchmark configuration (default cfg3, the headline)")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle sample")
    ap.add_argument("--cfg-pairs", action="store_true",
                    help="two-branch configurations (cfg2, cfg5): two ranks per image, one CFG branch each")
    args = ap.parse_args()
    if args.impl == "reference":
        if args.config in TEXT_CONFIGS:
            print(json.dumps({"impl": "reference", "unavailable": f"{args.config}: the text towers are not a "
                              "benchmark configuration; no bounded CPU sample is timed"}))
            return 0
        if args.config == "vae_tiled":
            print(json.dumps({"impl": "reference", "unavailable": "vae_tiled has no bounded CPU sample of the decode"}))
            return 0
        return run_reference(args)
    if args.config in TEXT_CONFIGS:
        return run_text(args)
    if args.config == "vae_tiled":
        return run_vae_tiled(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
