"""The tiled VAE decode on the GPU (nd_op_tile_gather, nd_op_tile_blend and
TiledVaeDecoder) against the oracle's restatement of TiledVaeDecoder.Run
(Vae/TiledVae.cs:136-159).

The gather and the blend are bit-exact (same float operations in the same
order). A whole tiled decode is compared with the oracle's fp32 decoder run
tile by tile at the decoder's tolerance (fp16: max|d| / max|ref| <= 2e-2,
cosine >= 0.999), and with the GPU's own decoded tiles blended by the oracle
bit-exactly.
"""
import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import ops
from naivediffusion_b200.denoiser import Device, VaeDecoderConfig, WanVaeConfig, build_denoiser, synthetic_weights
from naivediffusion_b200.tiled_vae import TiledVaeDecoder, crossfade, open_tiled_decoder, tile_starts

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


@pytest.mark.parametrize("h,w,side,overlap", [(96, 160, 64, 8), (200, 200, 64, 8), (72, 64, 64, 8),
                                              (24, 40, 16, 4), (64, 64, 64, 8)])
def test_tile_blend_is_bit_exact(cuda, h, w, side, overlap):
    rows, cols = tile_starts(h, side, overlap), tile_starts(w, side, overlap)
    g = torch.Generator().manual_seed(h * w + side)
    tiles = torch.randn(len(rows) * len(cols), 3, side, side, generator=g)
    v = torch.from_numpy(crossfade(rows, side)).cuda()
    hz = torch.from_numpy(crossfade(cols, side)).cuda()
    out = ops.tile_blend(tiles.cuda(), rows, cols, v, hz, h, w)
    ops.sync()
    ref = O.vae_tile_blend(tiles.numpy(), rows, cols, h, w)
    assert np.array_equal(out.cpu().numpy(), ref)


def test_tile_gather(cuda):
    c, h, w, t = 4, 24, 40, 16
    rows, cols = tile_starts(h, t, 4), tile_starts(w, t, 4)
    lat = torch.randn(c, h, w)
    tiles = ops.tile_gather(lat.cuda(), rows, cols, t)
    ops.sync()
    ref = torch.stack([lat[:, r:r + t, q:q + t] for r in rows for q in cols])
    assert torch.equal(tiles.cpu(), ref)


def test_tile_ops_reject_tiles_outside_the_image(cuda):
    lat = torch.zeros(4, 24, 40, device="cuda")
    with pytest.raises(Exception, match="outside"):
        ops.tile_gather(lat, [0, 9], [0], 16)
    tiles = torch.zeros(2, 3, 16, 16, device="cuda")
    ramp = torch.ones(16, device="cuda")
    with pytest.raises(Exception, match="outside"):
        ops.tile_blend(tiles, [0], [0, 30], ramp, ramp, 24, 40)


def _kl(tile, batch=1):
    return VaeDecoderConfig(width=64, mult=(1, 2, 2), layers_per_block=1, latent_height=tile, latent_width=tile,
                            batch=batch)


def test_tiled_kl_decode_matches_oracle(device):
    """A 24 x 40 latent in 16-cell tiles overlapping by 4: 2 x 3 tiles, one batch of 6."""
    cfg = _kl(16)
    w = dict(synthetic_weights(cfg, seed=21))
    lat = np.random.default_rng(21).standard_normal((1, 4, 24, 40)).astype(np.float32)
    with open_tiled_decoder(device, cfg, w, 96, 160, tile=16, overlap=4) as dec:
        assert (dec.rows, dec.cols, dec.tile_side) == ([0, 8], [0, 12, 24], 64)
        img = dec.run(lat)
        again = dec.run(lat)
        tiles = dec.decode_tiles(torch.from_numpy(lat[0]).cuda()).cpu().numpy()
    assert img.shape == (1, 3, 96, 160)
    assert np.array_equal(img, again)
    # the GPU's own tiles through the oracle's blend: bit-identical
    assert np.array_equal(img[0], O.vae_tile_blend(tiles, [0, 32], [0, 48, 96], 96, 160))
    ref = O.vae_tiled_decode(lambda piece: O.vae_decode(w, cfg, piece[None])[0], lat, 4, tile=16, overlap=4)
    assert rel(img, ref) < 2e-2, rel(img, ref)
    assert cos(img, ref) > 0.999


def test_one_tile_decodes_as_the_whole_image(device):
    """TiledVae: an image of one tile or less goes through as the whole-image graph would."""
    cfg = _kl(16)
    w = dict(synthetic_weights(cfg, seed=22))
    lat = np.random.default_rng(22).standard_normal((1, 4, 16, 16)).astype(np.float32)
    with open_tiled_decoder(device, cfg, w, 64, 64) as dec:
        assert dec.tile_count == 1
        img = dec.run(lat)
    with build_denoiser(device, cfg, w) as d:
        whole = d.predict(lat, 0.0, 0.0, {}, out=np.empty((1, 3, 64, 64), np.float32))
    assert np.array_equal(img, whole)


def test_tiled_wan21_decode_matches_oracle(device):
    """Anima's Wan 2.1 decoder (8x) over a 24 x 24 latent in 16-cell tiles: one batch of 4."""
    cfg = WanVaeConfig(version=21, width=64, latent_channels=16, latent_height=16, latent_width=16)
    w = dict(synthetic_weights(cfg, seed=23))
    lat = np.random.default_rng(23).standard_normal((1, 16, 24, 24)).astype(np.float32)
    with open_tiled_decoder(device, cfg, w, 192, 192, tile=16, overlap=4) as dec:
        assert dec.tile_count == 4
        img = dec.run(lat)
    ref = O.vae_tiled_decode(lambda piece: O.wan_vae_decode(w, cfg, piece[None])[0], lat, 8, tile=16, overlap=4)
    assert rel(img, ref) < 2e-2, rel(img, ref)
    assert cos(img, ref) > 0.999


def test_tiled_decoder_rejects_a_wrong_latent(device):
    cfg = _kl(16)
    w = dict(synthetic_weights(cfg, seed=24))
    with open_tiled_decoder(device, cfg, w, 96, 160, tile=16, overlap=4) as dec:
        with pytest.raises(ValueError):
            dec.run(np.zeros((1, 4, 16, 16), np.float32))
