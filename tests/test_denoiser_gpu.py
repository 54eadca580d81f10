"""The denoiser plug-in end to end (nd_denoiser_* through the C ABI) against
the CPU oracle's composed forward step, on seeded synthetic weights.

Tolerance: bf16 compute, so max|d| / max|ref| <= 2e-2 and cosine >= 0.999
over the predicted latent (the task's bf16 bar); the oracle is fp32 with the
same bf16-rounded weights.
"""
import numpy as np
import pytest

import oracle as O
from naivediffusion_b200 import _lib
from naivediffusion_b200.denoiser import (CudaDenoiser, Device, MMDiTConfig, build_denoiser,
                                          synthetic_weights)

pytestmark = pytest.mark.gpu

SMALL = dict(width=256, heads=2, blocks=2, mlp_width=512, context_rows=64, context_width=64,
             latent_height=16, latent_width=32)


def rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())


def cos(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def device(cuda):
    d = Device(0)
    yield d
    d.close()


def _inputs(cfg, seed=0):
    rng = np.random.default_rng(seed)
    lat = rng.standard_normal((1, cfg.latent_channels, cfg.latent_height, cfg.latent_width)).astype(np.float32)
    ctx = rng.standard_normal((1, cfg.context_rows, cfg.context_width)).astype(np.float32)
    return lat, ctx


@pytest.mark.parametrize("blocks,heads,width", [(2, 2, 256), (1, 4, 512)])
def test_mmdit_step_matches_oracle(device, blocks, heads, width):
    cfg = MMDiTConfig(**{**SMALL, "blocks": blocks, "heads": heads, "width": width})
    w = dict(synthetic_weights(cfg, seed=blocks))
    lat, ctx = _inputs(cfg, seed=blocks)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 500.0, 0.5, {"context": ctx})
    ref = O.mmdit_forward(w, cfg, lat, ctx[0], 0.5)
    assert y.shape == lat.shape
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999


def test_mmdit_repeat_is_bit_identical_and_tracks_inputs(device):
    """Replays of the captured step are deterministic (SmokeTest's first- vs
    second-dispatch check, NaiveDiffusion.Cli/SmokeTest.cs:631-645), and a new
    sigma / latent flows through the captured graph."""
    cfg = MMDiTConfig(**SMALL)
    w = dict(synthetic_weights(cfg, seed=3))
    lat, ctx = _inputs(cfg, seed=3)
    with build_denoiser(device, cfg, w) as d:
        a = d.predict(lat, 0.0, 0.9, {"context": ctx})
        b = d.predict(lat, 0.0, 0.9, {"context": ctx})
        c = d.predict(lat * 0.5, 0.0, 0.2, {"context": ctx})
        assert d.graph_count == 1
        m = d.memory()
        assert m.streamed_bytes == 0 and m.resident_bytes == m.persistent_bytes > 0
    np.testing.assert_array_equal(a, b)
    ref = O.mmdit_forward(w, cfg, lat * 0.5, ctx[0], 0.2)
    assert rel(c, ref) < 2e-2 and cos(c, ref) > 0.999


def test_mmdit_conditioning_tables_and_key_count(device):
    """Caller-supplied rotary tables (another branch's text length) and a
    key-count mask over padded text rows (QwenImageConditioning's key_length)."""
    cfg = MMDiTConfig(**SMALL)
    w = dict(synthetic_weights(cfg, seed=4))
    lat, ctx = _inputs(cfg, seed=4)
    cs, sn = O.qwen_rope_tables(cfg.latent_height // 2, cfg.latent_width // 2, 40, cfg.context_rows)
    keys = cfg.image_tokens + 40
    cond = {"context": ctx, "cos": cs, "sin": sn, "key_length": np.array([keys], np.int32)}
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.3, cond)
        y_default = d.predict(lat, 0.0, 0.3, {"context": ctx})
    ref = O.mmdit_forward(w, cfg, lat, ctx[0], 0.3, cs, sn, key_len=keys)
    assert rel(y, ref) < 2e-2 and cos(y, ref) > 0.999
    ref_d = O.mmdit_forward(w, cfg, lat, ctx[0], 0.3)
    assert rel(y_default, ref_d) < 2e-2


def test_plugin_errors(device):
    cfg = MMDiTConfig(**SMALL)
    d = CudaDenoiser(device, cfg.desc())
    try:
        names = d.weight_info()
        assert len(names) == 13 + cfg.blocks * 32
        with pytest.raises(_lib.NdError) as e:
            d.finalize()
        assert e.value.code == _lib.ND_ERR_MISSING_WEIGHT
        with pytest.raises(_lib.NdError) as e:
            d.set_weight("img_in.weight", np.zeros((3, 3), np.float32))
        assert e.value.code == _lib.ND_ERR_INVALID
        with pytest.raises(_lib.NdError) as e:
            d.set_weight("no.such.tensor", np.zeros((3, 3), np.float32))
        assert e.value.code == _lib.ND_ERR_INVALID
        lat, ctx = _inputs(cfg)
        with pytest.raises(_lib.NdError) as e:
            d.predict(lat, 0.0, 0.5, {"context": ctx})
        assert e.value.code == _lib.ND_ERR_STATE
    finally:
        d.close()
    bad = cfg.desc()
    bad.heads = 3
    with pytest.raises(_lib.NdError) as e:
        CudaDenoiser(device, bad)
    assert e.value.code == _lib.ND_ERR_INVALID


ANIMA_SMALL = dict(width=256, heads=2, blocks=2, mlp_width=1024, adaln_rank=64, context_rows=96,
                   context_width=128, latent_height=32, latent_width=16, batch=2)


@pytest.mark.parametrize("batch", [1, 2])
def test_anima_step_matches_oracle(device, batch):
    """The Anima DiT step (self-attention with 3-D RoPE, cross-attention to the
    text rows, low-rank adaLN, exact GELU) against the oracle's AnimaDit."""
    from naivediffusion_b200.denoiser import AnimaConfig
    cfg = AnimaConfig(**{**ANIMA_SMALL, "batch": batch})
    w = dict(synthetic_weights(cfg, seed=11))
    rng = np.random.default_rng(11)
    lat = rng.standard_normal((batch, 16, cfg.latent_height, cfg.latent_width)).astype(np.float32)
    ctx = rng.standard_normal((batch, cfg.context_rows, cfg.context_width)).astype(np.float32)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.6, {"context": ctx})
    ref = O.anima_forward(w, cfg, lat, ctx, 0.6)
    assert y.shape == lat.shape
    assert rel(y, ref) < 2e-2 and cos(y, ref) > 0.999, (rel(y, ref), cos(y, ref))


def test_profile_times_every_kernel_class(device):
    """nd_denoiser_profile replays a captured step with an event pair around
    every launch: every class gets a positive device time, and the launch
    count matches between two calls."""
    cfg = MMDiTConfig(**SMALL)
    w = dict(synthetic_weights(cfg, seed=2))
    lat, ctx = _inputs(cfg, seed=2)
    with build_denoiser(device, cfg, w) as d:
        d.predict(lat, 500.0, 0.5, {"context": ctx})
        p1 = d.profile(steps=2)
        p2 = d.profile(steps=1)
        y = d.predict(lat, 500.0, 0.5, {"context": ctx})  # the plug-in still works afterwards
    assert {p["name"] for p in p1} >= {"gemm.qkv", "attention", "gemm.out", "modulate", "gemm.up", "gemm.down"}
    assert all(p["ms"] > 0 for p in p1), p1
    assert [p["launches"] for p in p1] == [p["launches"] for p in p2]
    assert np.isfinite(y).all()
