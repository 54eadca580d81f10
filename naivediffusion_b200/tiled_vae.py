"""Tiled VAE decode: the reference's default decode path
(GenerationOptions.TileVae = true, src/NaiveDiffusion/Pipeline/GenerationOptions.cs:79;
VaeLatentCodec.OpenDecoder, Vae/VaeLatentCodec.cs:71-88).

The host half is the reference's (Vae/VaeTiling.cs, Vae/TiledVae.cs:21-59):
the tile side, the evenly spread tile origins and the crossfade ramps. The
device half differs in schedule, not in result: instead of running one
tile-sized graph once per tile, every tile is gathered into one batch and
decoded by ONE decoder created for the tile's size with batch = the tile
count. A batch item is normalised over its own pixels only, which is exactly
what a tile run alone sees, so the decoded tiles are the reference's; the
crossfade then runs on the device in the reference's float operations
(nd_op_tile_gather / nd_op_tile_blend).
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from . import ops

TILE_LATENT = 64   # TiledVae.TileLatent (Vae/TiledVae.cs:24): tile side in latent cells
TILE_OVERLAP = 8   # TiledVae.TileOverlap (:25)


def tile_starts(extent: int, tile: int, overlap: int) -> list[int]:
    """VaeTiling.TileStarts (Vae/VaeTiling.cs:12-25): enough equal tiles to
    keep every overlap at least `overlap` wide, spread evenly from 0 to
    extent - tile (rounded half to even, as Math.Round)."""
    if extent <= tile:
        return [0]
    count = ((extent - overlap) + (tile - overlap) - 1) // (tile - overlap)
    span = extent - tile
    # i * span / (count - 1): Python's int / int is the correctly rounded
    # quotient, as the reference's double division of the exact operands.
    return [int(round(i * span / (count - 1))) for i in range(count)]


def crossfade(starts: list[int], tile: int) -> np.ndarray:
    """VaeTiling.Crossfade (Vae/VaeTiling.cs:29-49): ones, with a linear ramp
    (i + 1) / (overlap + 1) at both ends across what neighbours share."""
    weight = np.ones(tile, np.float32)
    if len(starts) > 1:
        step = min(starts[i] - starts[i - 1] for i in range(1, len(starts)))
        overlap = tile - step
        for i in range(overlap):
            ramp = np.float32(i + 1) / np.float32(overlap + 1)
            weight[i] = ramp
            weight[tile - 1 - i] = ramp
    return weight


def window(rows: list[int], cols: list[int], side: int) -> np.ndarray:
    """VaeTiling.Window (Vae/VaeTiling.cs:55-68): the two axes' ramps multiplied."""
    return np.outer(crossfade(rows, side), crossfade(cols, side)).astype(np.float32)


def scale_factor(cfg) -> int:
    """Pixels per latent cell of a decoder config (VaeDecoderConfig or WanVaeConfig)."""
    if hasattr(cfg, "scale"):
        return int(cfg.scale)
    return 1 << (len(cfg.mult) - 1)


class TiledVaeDecoder:
    """TiledVaeDecoder (Vae/TiledVae.cs:124-160) over the library's decoders.

    build(tile, batch) returns a finalized decoder (CudaDenoiser) for a
    [batch, C, tile, tile] latent: see `decoder_builder`. height / width are
    the image's, in pixels."""

    def __init__(self, build, latent_channels: int, scale: int, height: int, width: int,
                 tile: int = TILE_LATENT, overlap: int = TILE_OVERLAP):
        self.latent_channels = latent_channels
        self.scale = scale
        self.height = height
        self.width = width
        # TiledVae's constructor (Vae/TiledVae.cs:43-55)
        self.tile = min(tile, min(height, width) // scale)
        overlap = min(overlap, self.tile // 2)
        self.rows = tile_starts(height // scale, self.tile, overlap)
        self.cols = tile_starts(width // scale, self.tile, overlap)
        self.model = build(self.tile, len(self.rows) * len(self.cols))
        dev = torch.device("cuda", self.model.device.ordinal)
        side = self.tile_side
        self._rows_px = [r * scale for r in self.rows]
        self._cols_px = [c * scale for c in self.cols]
        self._vertical = torch.from_numpy(crossfade(self._rows_px, side)).to(dev)
        self._horizontal = torch.from_numpy(crossfade(self._cols_px, side)).to(dev)
        self._device = dev
        self._decoded = None
        # Gather, decode and blend are ordered on one stream of the decoder's
        # own: a null stream handle would send the decode to the library's
        # device stream, unordered against torch's default stream.
        self._stream = torch.cuda.Stream(device=dev)

    @property
    def tile_side(self) -> int:
        """The tile's side in pixels."""
        return self.tile * self.scale

    @property
    def tile_count(self) -> int:
        return len(self.rows) * len(self.cols)

    def _decode(self, latent: torch.Tensor) -> torch.Tensor:
        # on self._stream
        tiles = ops.tile_gather(latent.contiguous(), self.rows, self.cols, self.tile)
        side = self.tile_side
        if self._decoded is None:
            self._decoded = torch.empty(self.tile_count, 3, side, side, device=self._device, dtype=torch.float32)
        self.model.predict_device(tiles, 0.0, 0.0, {}, self._decoded, self._stream.cuda_stream)
        return self._decoded

    def decode_tiles(self, latent: torch.Tensor) -> torch.Tensor:
        """Every tile of one latent [C, h, w] (CUDA, fp32) decoded as one batch:
        [tiles, 3, side, side], tiles in row-then-column order (ordered after
        and before torch's current stream's work)."""
        caller = torch.cuda.current_stream(self._device)
        self._stream.wait_stream(caller)
        with torch.cuda.stream(self._stream):
            decoded = self._decode(latent)
        caller.wait_stream(self._stream)
        return decoded

    def blend(self, decoded: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """The decoded tiles crossfaded into [3, height, width], on torch's current stream."""
        return ops.tile_blend(decoded, self._rows_px, self._cols_px, self._vertical, self._horizontal,
                              self.height, self.width, out)

    def run_device(self, latent: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """One unscaled latent [1, C, h, w] (CUDA) -> image [1, 3, H, W] (CUDA),
        ordered after and before torch's current stream's work."""
        if tuple(latent.shape) != (1, self.latent_channels, self.height // self.scale, self.width // self.scale):
            raise ValueError(f"latent must be [1, {self.latent_channels}, {self.height // self.scale}, "
                             f"{self.width // self.scale}], got {tuple(latent.shape)}")
        if out is not None and (tuple(out.shape) != (1, 3, self.height, self.width) or out.dtype != torch.float32
                                or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous float32 [1, 3, {self.height}, {self.width}] tensor")
        caller = torch.cuda.current_stream(self._device)
        self._stream.wait_stream(caller)
        with torch.cuda.stream(self._stream):
            img = self.blend(self._decode(latent[0].float()), None if out is None else out[0])
        caller.wait_stream(self._stream)
        img.record_stream(caller)
        return img.unsqueeze(0) if out is None else out

    def run(self, latent: np.ndarray) -> np.ndarray:
        """The same contract as the whole-image decoder (TiledVaeDecoder.Run):
        one unscaled latent [1, C, H/f, W/f] in, one image [1, 3, H, W] out."""
        x = torch.from_numpy(np.ascontiguousarray(latent, np.float32)).to(self._device)
        img = self.run_device(x)
        return img.cpu().numpy()

    def close(self) -> None:
        if self.model is not None:
            self.model.close()
            self.model = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def decoder_builder(device, cfg, weights):
    """build(tile, batch) for TiledVaeDecoder: the decoder config `cfg` at a
    tile x tile latent with `batch` items, the same weights."""
    from .denoiser import build_denoiser

    def build(tile: int, batch: int):
        return build_denoiser(device, dataclasses.replace(cfg, latent_height=tile, latent_width=tile, batch=batch),
                              weights)
    return build


def open_tiled_decoder(device, cfg, weights, height: int, width: int, tile: int = TILE_LATENT,
                       overlap: int = TILE_OVERLAP) -> TiledVaeDecoder:
    """VaeLatentCodec.OpenDecoder with TileVae on: the decoder of `cfg`
    (VaeDecoderConfig or WanVaeConfig; its own latent size and batch are
    ignored) tiled over a height x width image."""
    return TiledVaeDecoder(decoder_builder(device, cfg, weights), cfg.latent_channels, scale_factor(cfg), height,
                           width, tile, overlap)
