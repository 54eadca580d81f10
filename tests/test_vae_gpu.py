"""The AutoencoderKL decoder (family ND_FAMILY_VAE_KL) against the oracle's
restatement of AutoencoderKl.Decoder. fp16 compute: max|d| / max|ref| <= 2e-2
and cosine >= 0.999 on the decoded image."""
import numpy as np
import pytest

import oracle as O
from naivediffusion_b200.denoiser import Device, VaeDecoderConfig, build_denoiser, synthetic_weights

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


@pytest.mark.parametrize("latent,mult,lpb,batch", [
    (16, (1, 2, 2), 1, 1),     # 64 x 64 image
    (32, (1, 2, 2), 1, 2),     # 128 x 128, two latents
    (64, (1, 1, 2), 1, 1),     # 256 x 256: rows wider than one conv tile
])
def test_vae_decode_matches_oracle(device, latent, mult, lpb, batch):
    cfg = VaeDecoderConfig(width=64, mult=mult, layers_per_block=lpb, latent_height=latent, latent_width=latent,
                           batch=batch)
    w = dict(synthetic_weights(cfg, seed=latent))
    lat = np.random.default_rng(latent).standard_normal((batch, 4, latent, latent)).astype(np.float32)
    with build_denoiser(device, cfg, w) as d:
        img = d.predict(lat, 0.0, 0.0, {}, out=np.empty((batch, 3, cfg.image_height, cfg.image_width), np.float32))
        again = d.predict(lat, 0.0, 0.0, {}, out=np.empty_like(img))
    ref = O.vae_decode(w, cfg, lat)
    assert img.shape == ref.shape
    assert np.array_equal(img, again)
    assert rel(img, ref) < 2e-2, rel(img, ref)
    assert cos(img, ref) > 0.999


def test_vae_rejects_conditioning(device):
    cfg = VaeDecoderConfig(width=64, mult=(1, 2), layers_per_block=1, latent_height=16, latent_width=16)
    w = dict(synthetic_weights(cfg, seed=1))
    lat = np.zeros((1, 4, 16, 16), np.float32)
    with build_denoiser(device, cfg, w) as d:
        with pytest.raises(Exception, match="conditioning"):
            d.predict(lat, 0.0, 0.0, {"context": np.zeros((1, 4), np.float32)},
                      out=np.empty((1, 3, 32, 32), np.float32))
