"""The tiled VAE decode's host half (tile grid, crossfade, window) against
the reference's own tests of it (tests/NaiveDiffusion.Tests/VaeTilingTests.cs),
for both the product's host code and the oracle's restatement, and the two
against each other over a sweep (identical lists, bit-identical ramps)."""
import numpy as np
import pytest

import oracle as O
from naivediffusion_b200 import tiled_vae as T


@pytest.mark.parametrize("starts", [T.tile_starts, O.vae_tile_starts])
def test_an_image_of_one_tile_or_less_is_one_tile_at_the_origin(starts):
    assert starts(64, 64, 8) == [0]
    assert starts(32, 64, 8) == [0]


@pytest.mark.parametrize("starts", [T.tile_starts, O.vae_tile_starts])
def test_a_1024_image_is_three_tiles_overlapping_by_half(starts):
    assert starts(128, 64, 8) == [0, 32, 64]
    assert starts(128, 64, 16) == [0, 32, 64]   # the overlap only sets the count
    assert starts(96, 64, 8) == [0, 32]
    assert starts(256, 64, 8) == [0, 48, 96, 144, 192]


@pytest.mark.parametrize("starts", [T.tile_starts, O.vae_tile_starts])
def test_every_tile_ends_inside_the_image(starts):
    for extent in (64, 72, 100, 128, 200, 256, 257):
        s = starts(extent, 64, 8)
        assert s[0] == 0
        assert s[-1] + 64 <= extent, extent
        assert s == sorted(s)


@pytest.mark.parametrize("crossfade", [T.crossfade, O.vae_crossfade])
def test_two_ramps_meeting_sum_to_one_and_a_single_tile_is_all_ones(crossfade):
    assert np.all(crossfade([0], 8) == 1.0)
    ramp = crossfade([0, 4], 8)
    for i in range(4):
        assert abs(float(ramp[4 + i]) + float(ramp[i]) - 1.0) <= 1e-6, i
    assert ramp[0] < ramp[3]
    assert ramp[7] < ramp[4]


@pytest.mark.parametrize("window,crossfade", [(T.window, T.crossfade), (O.vae_window, O.vae_crossfade)])
def test_the_window_is_the_product_of_the_two_axes(window, crossfade):
    w = window([0, 4], [0], 8)
    v = crossfade([0, 4], 8)
    for y in range(8):
        for x in range(8):
            assert abs(float(w[y, x]) - float(v[y])) <= 1e-6


def test_product_host_half_matches_the_oracle():
    for extent in range(1, 300, 7):
        for tile in (8, 16, 40, 64):
            for overlap in (0, 2, 8, 16):
                if overlap >= tile:
                    continue
                a = T.tile_starts(extent, tile, overlap)
                assert a == O.vae_tile_starts(extent, tile, overlap), (extent, tile, overlap)
                if a[-1] + tile <= extent:
                    assert np.array_equal(T.crossfade(a, tile), O.vae_crossfade(a, tile))
    # starts closer than half a tile: the two ends' ramps overwrite each other in the middle
    s = T.tile_starts(72, 64, 8)
    assert s == [0, 8]
    assert np.array_equal(T.crossfade(s, 64), O.vae_crossfade(s, 64))
    assert np.array_equal(T.window([0, 4], [0, 4], 8), O.vae_window([0, 4], [0, 4], 8))


def test_blend_of_constant_tiles_is_constant():
    """Crossfades meeting sum to one, and the border ramps are divided back out."""
    rows, cols = O.vae_tile_starts(96, 64, 8), O.vae_tile_starts(160, 64, 8)
    tiles = np.full((len(rows) * len(cols), 3, 64, 64), 0.75, np.float32)
    img = O.vae_tile_blend(tiles, rows, cols, 96, 160)
    assert np.allclose(img, 0.75, rtol=0, atol=1e-6)


def test_tile_ops_check_their_tensors_before_any_launch():
    """The C ABI sees plain pointers: the wrappers refuse a tile count, a ramp
    or an output that does not match the grid (CPU tensors; nothing launches)."""
    import torch
    from naivediffusion_b200 import ops
    ramp = torch.ones(16)
    with pytest.raises(ValueError, match="square tiles"):
        ops.tile_blend(torch.zeros(5, 3, 16, 16), [0, 8], [0, 12, 24], ramp, ramp, 24, 40)
    with pytest.raises(ValueError, match="ramps"):
        ops.tile_blend(torch.zeros(6, 3, 16, 16), [0, 8], [0, 12, 24], torch.ones(8), ramp, 24, 40)
    with pytest.raises(ValueError, match="out must be"):
        ops.tile_blend(torch.zeros(6, 3, 16, 16), [0, 8], [0, 12, 24], ramp, ramp, 24, 40,
                       out=torch.zeros(3, 24, 39))
    with pytest.raises(ValueError, match="float32"):
        ops.tile_gather(torch.zeros(4, 24, 40, dtype=torch.float16), [0, 8], [0, 12, 24], 16)
