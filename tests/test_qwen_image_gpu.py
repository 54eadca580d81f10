"""Qwen-Image 2.1's single-stream DiT (family ND_FAMILY_QWEN_IMAGE) against the
oracle's composition of the reference's step (oracle.qwen_image_forward),
which turns adjacent feature pairs on the file's own weight order, so the
device's pairs-to-halves permutation is checked, not repeated.

Tolerances: bf16 / fp16 compute max|d| / max|ref| <= 2e-2 and cosine >= 0.999;
fp32 compute <= 1e-4; int8 weights against the oracle run on the dequantized
weights, the 16-bit bar.
"""
import numpy as np
import pytest

import oracle as O
from naivediffusion_b200 import _lib
from naivediffusion_b200.denoiser import (CudaDenoiser, Device, QwenImageConfig, build_denoiser,
                                          synthetic_weights)

pytestmark = pytest.mark.gpu

SMALL = dict(width=256, heads=2, blocks=2, mlp_width=384, context_rows=40, context_width=128,
             latent_height=16, latent_width=12, time_width=64)


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def device(cuda):
    d = Device(0)
    yield d
    d.close()


def _inputs(cfg, seed, real):
    rng = np.random.default_rng(seed)
    lat = rng.standard_normal((1, cfg.latent_channels, cfg.latent_height, cfg.latent_width)).astype(np.float32)
    ctx = np.zeros((1, cfg.context_rows, cfg.context_width), np.float32)
    ctx[0, :real] = rng.standard_normal((real, cfg.context_width))  # zero padding past the real rows
    n_img = cfg.latent_height * cfg.latent_width
    cond = {"context": ctx, "key_length": np.array([n_img + real], np.int32),
            "text_mask": O.causal_table(real, cfg.context_rows)}
    return lat, ctx, cond


@pytest.mark.parametrize("compute", [_lib.ND_BF16, _lib.ND_F16])
@pytest.mark.parametrize("real", [29, 40])
def test_qwen_image_step_matches_oracle(device, compute, real):
    cfg = QwenImageConfig(**SMALL, compute=compute)
    w = dict(synthetic_weights(cfg, seed=3))
    lat, ctx, cond = _inputs(cfg, 3, real)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.7, cond)
        y2 = d.predict(lat, 0.0, 0.7, cond)
    ref = O.qwen_image_forward(w, cfg, lat, ctx[0], 0.7, key_len=cfg.image_tokens + real)
    assert y.shape == lat.shape
    assert np.array_equal(y, y2)
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999


def test_qwen_image_fp32_within_1e4(device):
    cfg = QwenImageConfig(**SMALL, compute=_lib.ND_F32)
    w = dict(synthetic_weights(cfg, seed=4))
    lat, ctx, cond = _inputs(cfg, 4, 33)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.35, cond)
    ref = O.qwen_image_forward(w, cfg, lat, ctx[0], 0.35, key_len=cfg.image_tokens + 33)
    assert rel(y, ref) < 1e-4, rel(y, ref)


def test_qwen_image_wider_model(device):
    """Eight heads, the released model's SwiGLU ratio, 768 image tokens."""
    cfg = QwenImageConfig(width=1024, heads=8, blocks=2, mlp_width=3072, context_rows=96, context_width=256,
                          latent_height=32, latent_width=24, time_width=256, compute=_lib.ND_BF16)
    w = dict(synthetic_weights(cfg, seed=8))
    lat, ctx, cond = _inputs(cfg, 8, 77)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.9, cond)
    ref = O.qwen_image_forward(w, cfg, lat, ctx[0], 0.9, key_len=cfg.image_tokens + 77)
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999


def test_split_gate_and_up_equal_the_fused_tensor(device):
    """img_mlp.gate_layer + img_mlp.proj land in the two halves of the fused
    gate_up storage: the same step, bit for bit."""
    fused = QwenImageConfig(**SMALL)
    split = QwenImageConfig(**SMALL, fused_gate_up=False)
    w = dict(synthetic_weights(fused, seed=6))
    F = fused.mlp_width
    ws = {}
    for n, a in w.items():
        if n.endswith("img_mlp.gate_up.weight"):
            p = n[: -len("gate_up.weight")]
            ws[p + "gate_layer.weight"] = np.ascontiguousarray(a[:F])
            ws[p + "proj.weight"] = np.ascontiguousarray(a[F:])
        else:
            ws[n] = a
    lat, _ctx, cond = _inputs(fused, 6, 40)
    with build_denoiser(device, fused, w) as d:
        a = d.predict(lat, 0.0, 0.5, cond)
    with build_denoiser(device, split, ws) as d:
        b = d.predict(lat, 0.0, 0.5, cond)
    assert np.array_equal(a, b)


def test_default_tables_are_the_conditioners(device):
    """Without cos / sin the family builds the conditioner's tables for the
    branch's real text length (QwenImageConditioning), so passing them equals
    leaving them out."""
    cfg = QwenImageConfig(**SMALL)
    w = dict(synthetic_weights(cfg, seed=2))
    lat, _ctx, cond = _inputs(cfg, 2, 21)
    c, s = O.qwen_rope_tables(cfg.latent_height, cfg.latent_width, 21, cfg.context_rows)
    with build_denoiser(device, cfg, w) as d:
        a = d.predict(lat, 0.0, 0.5, cond)
        b = d.predict(lat, 0.0, 0.5, {**cond, "cos": c, "sin": s})
        full = d.predict(lat, 0.0, 0.5, {"context": cond["context"]})   # every row real
        a2 = d.predict(lat, 0.0, 0.5, cond)
    assert np.array_equal(a, b)
    assert np.array_equal(a, a2)
    assert not np.array_equal(a, full)


def test_conditioning_errors(device):
    cfg = QwenImageConfig(**SMALL)
    w = dict(synthetic_weights(cfg, seed=1))
    lat, _ctx, cond = _inputs(cfg, 1, 30)
    with build_denoiser(device, cfg, w) as d:
        bad = O.causal_table(31, cfg.context_rows)
        with pytest.raises(Exception, match="text_mask"):
            d.predict(lat, 0.0, 0.5, {**cond, "text_mask": bad})
        with pytest.raises(Exception, match="key_length"):
            d.predict(lat, 0.0, 0.5, {**cond, "key_length": np.array([cfg.image_tokens], np.int32)})
        with pytest.raises(Exception, match="context"):
            d.predict(lat, 0.0, 0.5, {"key_length": cond["key_length"]})


def test_missing_feed_forward_is_reported(device):
    cfg = QwenImageConfig(**{**SMALL, "blocks": 1})
    w = dict(synthetic_weights(cfg, seed=1))
    d = CudaDenoiser(device, cfg.desc())
    try:
        for n, a in w.items():
            if not n.endswith("gate_up.weight"):
                d.set_weight(n, a)
        with pytest.raises(Exception, match="gate_up"):
            d.finalize()
    finally:
        d.close()


@pytest.mark.parametrize("group,scale_dtype", [(32, _lib.ND_F16), (0, _lib.ND_F32)])
def test_qwen_image_int8(device, group, scale_dtype):
    cfg = QwenImageConfig(**SMALL, compute=_lib.ND_BF16, weight_dtype=_lib.ND_I8, quant_group=group,
                          quant_scale_dtype=scale_dtype)
    w = dict(synthetic_weights(cfg, seed=7))
    deq, nq = {}, 0
    for name, a in w.items():
        if a.ndim == 2 and cfg.quantized(*a.shape):
            g = group or a.shape[1]
            q, s = O.quantize(a, group=g, scale_f16=scale_dtype == _lib.ND_F16)
            deq[name] = O.round_bf16(O.dequantize(q, s, group=g))
            nq += 1
        else:
            deq[name] = a
    assert nq >= 2 * 5
    lat, ctx, cond = _inputs(cfg, 7, 35)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.6, cond)
    ref = O.qwen_image_forward(deq, cfg, lat, ctx[0], 0.6, key_len=cfg.image_tokens + 35)
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999
