"""Parity at the benchmark configurations' real widths: one block of each
benchmarked model at its full width, token count and batch, and the joint
attention at the cfg3 shape, through the C ABI against the CPU oracle.

The reference's own check is of this form: a whole operator at a production
shape against a CPU loop over the same inputs (NaiveDiffusion.Cli/SmokeTest.cs:43-64;
the attention probe's 4096 x 16 x 128 case, NaiveDiffusion.Cli/AttentionProbe.cs:20-80).
The smaller-width step tests elsewhere cover the wiring; these cover the
kernels at the tile counts, head counts, row-group splits and key-tile
counts the benchmark runs (cfg3: 5376 + 256 rows, 24 heads, 44 key tiles
per query tile; cfg2: 4096 rows x batch 2; cfg5: 128 x 128 latent, widths
320 / 640 / 1280).

Tolerance (the task's bar for 16-bit compute), written in each test:
max|d| / max|ref| <= 2e-2 and cosine >= 0.999. The oracle computes in fp32
from the same 16-bit-rounded weights (int8: from the dequantized weights,
which the device reproduces bit for bit).
"""
import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import _lib
from naivediffusion_b200.denoiser import (AnimaConfig, CudaDenoiser, Device, MMDiTConfig, QwenImageConfig,
                                          UNetConfig, build_denoiser, synthetic_weights)

pytestmark = pytest.mark.gpu

REL, COS = 2e-2, 0.999


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def check(y, ref, what):
    r, c = rel(y, ref), cos(y, ref)
    print(f"{what}: max rel {r:.3e}, cosine {c:.7f}")
    assert y.shape == ref.shape, (what, y.shape, ref.shape)
    assert np.isfinite(y).all(), what
    assert r <= REL and c >= COS, f"{what}: max rel {r:.3e}, cosine {c:.6f}"


@pytest.fixture(scope="module")
def device(cuda):
    d = Device(0)
    yield d
    d.close()


# ---------------------------------------------------------------- cfg3 / cfg4

CFG3_BLOCK = MMDiTConfig(blocks=1)  # 3072 wide, 24 x 128 heads, MLP 12288, 5376 + 256 rows


@pytest.fixture(scope="module")
def cfg3_case():
    w = dict(synthetic_weights(CFG3_BLOCK, seed=0))
    rng = np.random.default_rng(0)
    lat = rng.standard_normal((1, 16, 128, 168)).astype(np.float32)
    ctx = rng.standard_normal((1, 256, 3584)).astype(np.float32)
    return w, lat, ctx


def test_cfg3_block_full_width(device, cfg3_case):
    """One dual-stream block of the cfg3 model at its real shape (the text
    stream's rows start at 5376, inside the same GEMM launches), plus the
    embeddings and the final layer, against the oracle."""
    w, lat, ctx = cfg3_case
    with build_denoiser(device, CFG3_BLOCK, w) as d:
        y = d.predict(lat, 0.0, 0.7, {"context": ctx})
    check(y, O.mmdit_forward(w, CFG3_BLOCK, lat, ctx[0], 0.7), "cfg3 block")


def test_cfg3_block_full_width_key_count(device, cfg3_case):
    """The same block with the text rows padded: only the first 40 text rows
    are keys (QwenImageConditioning's key_length), with the rotary tables of a
    40-token prompt."""
    w, lat, ctx = cfg3_case
    cfg = CFG3_BLOCK
    cs, sn = O.qwen_rope_tables(64, 84, 40, cfg.context_rows)
    keys = cfg.image_tokens + 40
    cond = {"context": ctx, "cos": cs, "sin": sn, "key_length": np.array([keys], np.int32)}
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.4, cond)
    check(y, O.mmdit_forward(w, cfg, lat, ctx[0], 0.4, cs, sn, key_len=keys), "cfg3 block, key count")


@pytest.mark.parametrize("group,scale_dtype", [(0, _lib.ND_F32), (32, _lib.ND_F16)],
                         ids=["per-channel-f32", "g32-f16"])
def test_cfg4_int8_block_full_width(device, cfg3_case, group, scale_dtype):
    """cfg4: the cfg3 block with int8 weights quantized on the device from the
    seeded bf16 weights (per output channel with fp32 scales, the benchmark
    configuration; and the reference's G = 32 fp16 scales), against the
    oracle run on the dequantized weights."""
    w, lat, ctx = cfg3_case
    cfg = MMDiTConfig(blocks=1, weight_dtype=_lib.ND_I8, quant_group=group, quant_scale_dtype=scale_dtype)
    deq = {}
    quantized = 0
    for name, a in w.items():
        if a.ndim == 2 and cfg.quantized(*a.shape):
            g = group or a.shape[1]
            q, s = O.quantize(a, group=g, scale_f16=scale_dtype == _lib.ND_F16)
            deq[name] = O.round_bf16(O.dequantize(q, s, group=g))
            quantized += 1
        else:
            deq[name] = a
    assert quantized >= 2 * 6  # both streams' q/k/v/out/up/down (+ modulation)
    d = CudaDenoiser(device, cfg.desc())
    try:
        for name, a in w.items():
            d.set_weight(name, a)
        d.finalize()
        y = d.predict(lat, 0.0, 0.55, {"context": ctx})
    finally:
        d.close()
    check(y, O.mmdit_forward(deq, cfg, lat, ctx[0], 0.55), f"cfg4 block ({group}, {scale_dtype})")


@pytest.mark.parametrize("key_limit", [0, 5376 + 40], ids=["all-keys", "key-count"])
def test_attention_cfg3_shape(cuda, key_limit):
    """nd_op_attention at the cfg3 joint shape: 5632 queries x 5632 keys x 24
    heads of 128 (44 key tiles per query tile), with and without a key-count
    limit that ends inside a key tile."""
    from naivediffusion_b200 import ops
    rows, heads = 5632, 24
    g = torch.Generator(device="cuda").manual_seed(1234 + key_limit)
    q = (torch.randn(rows, heads * 128, device="cuda", generator=g) * 1.5).bfloat16()
    k = (torch.randn(rows, heads * 128, device="cuda", generator=g) * 1.5).bfloat16()
    v = torch.randn(rows, heads * 128, device="cuda", generator=g).bfloat16()
    y = ops.attention(q, k, v, heads, key_limit=key_limit)
    ops.sync()
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref = O.attention(f(q), f(k), f(v), heads, key_len=key_limit)
    check(f(y), ref, f"attention 5632 x 24, key limit {key_limit}")


# ---------------------------------------------------------------------- cfg2

def test_cfg2_anima_block_full_width(device):
    """One Anima block of cfg2 at its real shape: 2048 wide, 16 heads, 4096
    image tokens (3-D RoPE), cross-attention to 256 x 1024 text rows, exact
    GELU MLP 8192, low-rank adaLN 256, batch 2 (the CFG branches)."""
    cfg = AnimaConfig(blocks=1)
    w = dict(synthetic_weights(cfg, seed=2))
    rng = np.random.default_rng(2)
    lat = rng.standard_normal((2, 16, 128, 128)).astype(np.float32)
    ctx = rng.standard_normal((2, 256, 1024)).astype(np.float32)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.6, {"context": ctx})
    check(y, O.anima_forward(w, cfg, lat, ctx, 0.6), "cfg2 block")


# ---------------------------------------------------------------------- cfg5

def test_cfg5_unet_full_width(device):
    """The SDXL UNet of cfg5 at its real widths (320 / 640 / 1280, heads 5 /
    10 / 20 of 64), two resnets per level (so every skip-concat width of the
    real up path), the 128 x 128 latent, 77 x 2048 context, 2816-wide add
    embedding, batch 2, fp16; one transformer block per attention level
    instead of 2 / 10 (the same shapes, repeated, in the real model)."""
    cfg = UNetConfig(depth=(0, 1, 1), resnets=2)
    w = dict(synthetic_weights(cfg, seed=3))
    rng = np.random.default_rng(3)
    lat = rng.standard_normal((2, 4, 128, 128)).astype(np.float32)
    add = rng.standard_normal((2, 2816)).astype(np.float32)
    ctx = rng.standard_normal((2, 77, 2048)).astype(np.float32)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 481.0, 0.0, {"context": ctx, "add": add})
    check(y, O.unet_forward(w, cfg, lat, 481.0, add, ctx), "cfg5 UNet")


# ------------------------------------------------------- Qwen-Image 2.1 (f3)

def test_qwen_image_block_full_width(device):
    """One block of the reference's own Qwen-Image 2.1 single-stream DiT at its
    released shape (4096 wide, 32 x 128 heads, SwiGLU 12288, 64-channel
    latent at patch 1: 4096 image rows + 256 text rows, 4096-wide text
    states), fp16 compute, with 40 real text rows under the causal text table
    and the key count, against the oracle's composition of the reference's
    step (which turns adjacent feature pairs on the file's weight order)."""
    cfg = QwenImageConfig(blocks=1)
    w = dict(synthetic_weights(cfg, seed=4))
    rng = np.random.default_rng(4)
    real = 40
    lat = rng.standard_normal((1, cfg.latent_channels, cfg.latent_height, cfg.latent_width)).astype(np.float32)
    ctx = np.zeros((1, cfg.context_rows, cfg.context_width), np.float32)
    ctx[0, :real] = rng.standard_normal((real, cfg.context_width))
    n_img = cfg.latent_height * cfg.latent_width
    cond = {"context": ctx, "key_length": np.array([n_img + real], np.int32),
            "text_mask": O.causal_table(real, cfg.context_rows)}
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.7, cond)
    check(y, O.qwen_image_forward(w, cfg, lat, ctx[0], 0.7, key_len=n_img + real), "Qwen-Image 2.1 block")
