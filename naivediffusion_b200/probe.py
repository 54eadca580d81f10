"""Operator probes: one kernel at one shape, timed with CUDA events.

    python -m naivediffusion_b200.probe attention [--tokens 4096 --heads 16 --head-dim 128]
    python -m naivediffusion_b200.probe quant     [--rows 4096 --width 1280]
    python -m naivediffusion_b200.probe gemm      --m 5632 --n 3072 --k 12288 [--epilogue residual_gate]
    python -m naivediffusion_b200.probe conv      --batch 2 --size 128 --cin 320 --cout 320 [--stride 1]
    python -m naivediffusion_b200.probe groupnorm --batch 2 --pixels 16384 --channels 320
    python -m naivediffusion_b200.probe modulate  --rows 5632 --width 3072
    python -m naivediffusion_b200.probe gemv      --n 368640 --k 3072

`attention` and `quant` are the counterparts of the reference's `attnprobe`
(NaiveDiffusion.Cli/AttentionProbe.cs: 4096 tokens x 16 x 128, TFLOPS =
4 H N^2 d / t) and `quantprobe` (NaiveDiffusion.Cli/QuantProbe.cs: fp16 vs int8
GEMM at [4096 x 1280] . [1280 -> 1280 / 5120], pass if the int8 error is below
2e-2 of max|y|). Each prints one JSON line: the device time per launch and
the achieved TFLOP/s or GB/s (algorithmic work / time). Inputs stay resident
in HBM; --iters launches are timed back to back after --warmup.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch

from . import _lib, ops


def _time(fn, warmup: int, iters: int) -> float:
    """Milliseconds per call, CUDA events on the current (explicit) stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / max(1, iters)


def _emit(kind: str, ms: float, flops: float = 0.0, nbytes: float = 0.0, **extra) -> None:
    line = {"probe": kind, "ms": ms}
    if flops:
        line["tflops"] = flops / (ms / 1e3) / 1e12
    if nbytes:
        line["gbs"] = nbytes / (ms / 1e3) / 1e9
    line.update(extra)
    print(json.dumps(line), flush=True)


def probe_attention(a) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    n, h, d = a.tokens, a.heads, a.head_dim
    dt = torch.float16 if a.f16 else torch.bfloat16
    qkv = torch.randn(n, 3 * h * d, device="cuda", generator=g).to(dt)
    q, k, v = qkv[:, :h * d], qkv[:, h * d:2 * h * d], qkv[:, 2 * h * d:]
    out = torch.empty(n, h * d, device="cuda", dtype=dt)
    ms = _time(lambda: ops.attention(q, k, v, h, out=out, head_dim=d), a.warmup, a.iters)
    _emit("attention", ms, 4.0 * h * n * n * d, tokens=n, heads=h, head_dim=d)


def probe_quant(a) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(a.rows, a.width, device="cuda", generator=g).bfloat16()
    for n_out in (a.width, 4 * a.width):
        w = (torch.randn(n_out, a.width, device="cuda", generator=g) * 0.02).bfloat16()
        q, s = ops.quantize(w, quant_group=32, scale_dtype=torch.float16)
        y16 = ops.linear(x, w)
        y8 = ops.linear(x, q, scales=s, quant_group=32)
        ms16 = _time(lambda: ops.linear(x, w), a.warmup, a.iters)
        ms8 = _time(lambda: ops.linear(x, q, scales=s, quant_group=32), a.warmup, a.iters)
        err = float((y8.float() - y16.float()).abs().max() / y16.float().abs().max())
        fl = 2.0 * a.rows * n_out * a.width
        print(json.dumps({"probe": "quant", "shape": [a.rows, a.width, n_out], "bf16_ms": ms16,
                          "int8_ms": ms8, "bf16_tflops": fl / ms16 / 1e9, "int8_tflops": fl / ms8 / 1e9,
                          "int8_rel_err": err, "pass": err < 2e-2}), flush=True)


_EPI = {"store": _lib.ND_EPI_STORE, "gelu_tanh": _lib.ND_EPI_GELU_TANH, "residual_gate": _lib.ND_EPI_RESIDUAL_GATE,
        "qk": _lib.ND_EPI_QK_NORM_ROPE, "swiglu": _lib.ND_EPI_SWIGLU, "geglu": _lib.ND_EPI_GEGLU}


def probe_gemm(a) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(a.m, a.k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(a.n, a.k, device="cuda", generator=g) * 0.02).bfloat16()
    b = torch.randn(a.n, device="cuda", generator=g) * 0.1
    epi = _EPI[a.epilogue]
    kw = {}
    if epi == _lib.ND_EPI_RESIDUAL_GATE:
        kw = dict(residual=torch.zeros(a.m, a.n, device="cuda"), gate=torch.ones(a.n, device="cuda") * 1e-3)
    elif epi == _lib.ND_EPI_QK_NORM_ROPE:
        kw = dict(qk_norm=torch.ones(2, 128, device="cuda"), rope_cos=torch.ones(a.m, 64, device="cuda"),
                  rope_sin=torch.zeros(a.m, 64, device="cuda"), qk_cols=2 * (a.n // 3))
    if a.int8:
        q, s = ops.quantize(w, quant_group=0, scale_dtype=torch.float32)
        fn = lambda: ops.linear(x, q, b, epilogue=epi, scales=s, quant_group=0, **kw)  # noqa: E731
    else:
        fn = lambda: ops.linear(x, w, b, epilogue=epi, **kw)  # noqa: E731
    ms = _time(fn, a.warmup, a.iters)
    _emit("gemm", ms, 2.0 * a.m * a.n * a.k, m=a.m, n=a.n, k=a.k, epilogue=a.epilogue, int8=a.int8)


def probe_conv(a) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(a.batch, a.size, a.size, a.cin, device="cuda", generator=g).half()
    w = (torch.randn(a.cout, 3, 3, (a.cin + 63) // 64 * 64, device="cuda", generator=g) * 0.02).half()
    b = torch.randn(a.cout, device="cuda", generator=g) * 0.1
    ho = (a.size - 1) // a.stride + 1
    ms = _time(lambda: ops.conv2d(x, w, b, stride=a.stride), a.warmup, a.iters)
    _emit("conv3x3", ms, 2.0 * a.batch * ho * ho * a.cout * 9 * a.cin, batch=a.batch, size=a.size,
          cin=a.cin, cout=a.cout, stride=a.stride)


def probe_groupnorm(a) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(a.batch, a.pixels, a.channels, device="cuda", generator=g).half()
    w = torch.ones(a.channels, device="cuda")
    b = torch.zeros(a.channels, device="cuda")
    ms = _time(lambda: ops.group_norm(x, 32, w, b, silu=True), a.warmup, a.iters)
    _emit("groupnorm", ms, nbytes=2.0 * 2 * x.numel(), batch=a.batch, pixels=a.pixels, channels=a.channels)


def probe_modulate(a) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(a.rows, a.width, device="cuda", generator=g)
    sh = torch.randn(a.width, device="cuda", generator=g)
    sc = torch.randn(a.width, device="cuda", generator=g)
    out = torch.empty(a.rows, a.width, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ops.modulate(x, sh, sc, out=out), a.warmup, a.iters)
    _emit("modulate", ms, nbytes=6.0 * a.rows * a.width, rows=a.rows, width=a.width)


def probe_gemv(a) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    w = (torch.randn(a.n, a.k, device="cuda", generator=g) * 0.02).bfloat16()
    x = torch.randn(1, a.k, device="cuda", generator=g)
    ms = _time(lambda: ops.gemv(w, x), a.warmup, a.iters)
    _emit("gemv", ms, 2.0 * a.n * a.k, nbytes=2.0 * a.n * a.k, n=a.n, k=a.k)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="probe", required=True)
    p = sub.add_parser("attention")
    p.add_argument("--tokens", type=int, default=4096)
    p.add_argument("--heads", type=int, default=16)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--f16", action="store_true")
    p = sub.add_parser("quant")
    p.add_argument("--rows", type=int, default=4096)
    p.add_argument("--width", type=int, default=1280)
    p = sub.add_parser("gemm")
    p.add_argument("--m", type=int, default=5632)
    p.add_argument("--n", type=int, default=3072)
    p.add_argument("--k", type=int, default=12288)
    p.add_argument("--epilogue", choices=sorted(_EPI), default="residual_gate")
    p.add_argument("--int8", action="store_true", help="int8 weight-only, per-channel fp32 scales")
    p = sub.add_parser("conv")
    p.add_argument("--batch", type=int, default=2)
    p.add_argument("--size", type=int, default=128)
    p.add_argument("--cin", type=int, default=320)
    p.add_argument("--cout", type=int, default=320)
    p.add_argument("--stride", type=int, default=1)
    p = sub.add_parser("groupnorm")
    p.add_argument("--batch", type=int, default=2)
    p.add_argument("--pixels", type=int, default=16384)
    p.add_argument("--channels", type=int, default=320)
    p = sub.add_parser("modulate")
    p.add_argument("--rows", type=int, default=5632)
    p.add_argument("--width", type=int, default=3072)
    p = sub.add_parser("gemv")
    p.add_argument("--n", type=int, default=368640)
    p.add_argument("--k", type=int, default=3072)
    for sp in sub.choices.values():
        sp.add_argument("--warmup", type=int, default=5)
        sp.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    torch.cuda.set_stream(torch.cuda.Stream())
    {"attention": probe_attention, "quant": probe_quant, "gemm": probe_gemm, "conv": probe_conv,
     "groupnorm": probe_groupnorm, "modulate": probe_modulate, "gemv": probe_gemv}[a.probe](a)
    return 0


if __name__ == "__main__":
    sys.exit(main())
