"""The Wan VAE decoders (families ND_FAMILY_VAE_WAN21 / ND_FAMILY_VAE_WAN22,
Vae/WanVae.cs and Vae/Wan22Vae.cs on one frame) against the oracle's
restatement (oracle.wan_vae_decode). fp16 compute: max|d| / max|ref| <= 2e-2
and cosine >= 0.999 on the decoded image."""
import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import ops
from naivediffusion_b200.denoiser import Device, WanVaeConfig, build_denoiser, synthetic_weights

pytestmark = pytest.mark.gpu


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


@pytest.mark.parametrize("kw", [
    dict(version=21, width=96, latent_channels=16, latent_height=16, latent_width=16),            # Wan 2.1 widths
    dict(version=21, width=64, latent_channels=16, latent_height=16, latent_width=32, batch=2),
    dict(version=22, width=72, latent_channels=64, latent_height=8, latent_width=16),
    dict(version=22, width=144, latent_channels=64, latent_height=8, latent_width=16),            # Qwen-Image 2.1's widths
])
def test_wan_decode_matches_oracle(device, kw):
    cfg = WanVaeConfig(**kw)
    w = dict(synthetic_weights(cfg, seed=cfg.width))
    lat = np.random.default_rng(cfg.width).standard_normal(
        (cfg.batch, cfg.latent_channels, cfg.latent_height, cfg.latent_width)).astype(np.float32)
    out = np.empty((cfg.batch, 3, cfg.image_height, cfg.image_width), np.float32)
    with build_denoiser(device, cfg, w) as d:
        img = d.predict(lat, 0.0, 0.0, {}, out=out)
        again = d.predict(lat, 0.0, 0.0, {}, out=np.empty_like(out))
    ref = O.wan_vae_decode(w, cfg, lat)
    assert img.shape == ref.shape
    assert np.array_equal(img, again)
    assert rel(img, ref) < 2e-2, rel(img, ref)
    assert cos(img, ref) > 0.999


def test_wan_rejects_conditioning(device):
    cfg = WanVaeConfig(width=64, latent_height=16, latent_width=16)
    w = dict(synthetic_weights(cfg, seed=1))
    lat = np.zeros((1, 16, 16, 16), np.float32)
    with build_denoiser(device, cfg, w) as d:
        with pytest.raises(Exception, match="conditioning"):
            d.predict(lat, 0.0, 0.0, {"context": np.zeros((1, 4), np.float32)},
                      out=np.empty((1, 3, 128, 128), np.float32))


@pytest.mark.parametrize("c", [96, 144, 1152])
def test_channel_rms_silu_matches_oracle(cuda, c):
    g = torch.Generator().manual_seed(c)
    x = (torch.randn(1000, c, generator=g) * 2).half()
    gamma = 1 + 0.1 * torch.randn(c, generator=g)
    y = ops.rmsnorm(x.cuda(), gamma.cuda(), eps=1e-24 / c, silu=True)
    torch.cuda.synchronize()
    ref = O.silu(O.rmsnorm(x.float().numpy(), gamma.numpy(), 1e-24 / c))
    assert rel(y.float().cpu().numpy(), ref) < 4e-3
