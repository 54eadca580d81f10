"""Host-side multi-GPU plumbing for the denoiser step (one process per GPU).

The path shards by image: every rank holds the full weights and denoises its
own images (the CFG branches of an image stay on one rank, stacked as batch
rows); nothing crosses GPUs during a step. The one collective is the gather
of the predicted latents to rank 0 at the end (SamplingLoop hands one latent
per image back to the pipeline). Timing across ranks is the maximum of the
per-rank device times. torch.distributed carries it: NCCL over NVLink on
GPUs, gloo on CPU (the tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def image_shard(n_images: int, rank: int, world: int) -> range:
    """The images rank `rank` denoises: contiguous blocks, sizes differing by
    at most one (images [start, stop) of the job)."""
    if n_images < 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError("image_shard: bad job shape")
    base, extra = divmod(n_images, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def gather_latents(latent: torch.Tensor, world: int) -> list[torch.Tensor]:
    """Every rank's prediction (same shape on every rank), in rank order.
    One all_gather; the tensors stay on the collective's device."""
    if world == 1:
        return [latent]
    out = [torch.empty_like(latent) for _ in range(world)]
    dist.all_gather(out, latent.contiguous())
    return out


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """The largest of the ranks' values (the job's time is its slowest rank's)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
