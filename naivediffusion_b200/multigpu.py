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


# ------------------------------------------------------------ CFG-parallel pairs
#
# The alternative partitioning for the two-branch (classifier-free guidance)
# configurations: two ranks per image, one branch each. Both hold the full
# weights in a batch-1 denoiser; per step each predicts its own branch, one
# all_gather inside the pair stacks the two predictions as [uncond, cond]
# (GuidanceStrategy.Combine, Pipeline/GuidanceStrategy.cs:34-47, needs both),
# and both ranks take the same sampler step on the same inputs, so their
# latents stay bit-identical without a second exchange. For the stochastic
# samplers (Euler a, DPM++ 2M SDE) "the same inputs" includes the noise: both
# ranks of a pair must draw it from the image's seed (the image index and
# step), never from a per-rank one, or the two copies of the latent drift
# apart after the first noisy step. At cfg2's latent that
# is 1 MB per step over NVLink against a step of tens of milliseconds: the
# image's latency halves where the replicas layout keeps one image per GPU.


class CfgPair:
    """This rank's place in a CFG-parallel pair: ranks (2i, 2i + 1) denoise
    image i, the even one the unconditional branch (0), the odd one the
    conditional branch (1). Every rank must construct it (the pair groups are
    created collectively, in the same order on every rank)."""

    def __init__(self, rank: int, world: int):
        if world < 2 or world % 2:
            raise ValueError("CfgPair: an even number of ranks, two per image")
        if not 0 <= rank < world:
            raise ValueError("CfgPair: rank outside the job")
        self.rank = rank
        self.image = rank // 2
        self.branch = rank % 2
        self.group = None  # two ranks: the default group is the pair
        if world > 2:
            groups = [dist.new_group([2 * i, 2 * i + 1]) for i in range(world // 2)]
            self.group = groups[self.image]

    def exchange(self, mine: torch.Tensor, both: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's prediction [1, ...] -> both branches' [2, ...] (uncond,
        cond), identical on the two ranks of the pair."""
        if mine.shape[0] != 1:
            raise ValueError("CfgPair.exchange: one branch per rank ([1, ...])")
        if both is None:
            both = torch.empty((2,) + tuple(mine.shape[1:]), dtype=mine.dtype, device=mine.device)
        elif (tuple(both.shape) != (2,) + tuple(mine.shape[1:]) or both.dtype != mine.dtype
              or not both.is_contiguous() or both.device != mine.device):
            raise ValueError("CfgPair.exchange: `both` must be a contiguous [2, ...] tensor of the prediction's "
                             "dtype on its device")
        # into the two contiguous halves of `both`, in pair order: uncond, cond
        dist.all_gather([both[0], both[1]], mine[0].contiguous(), group=self.group)
        return both
