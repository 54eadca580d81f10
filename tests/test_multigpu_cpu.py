"""The multi-GPU host logic (image sharding, the latent gather, the max-over-
ranks timing) as world_size-2 gloo process groups on the CPU, plus the
failure paths: a rank that raises, and a rank that never joins, end the job
with an error on the host instead of a hang."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from naivediffusion_b200.multigpu import CfgPair, gather_latents, image_shard, max_over_ranks


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _gather_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        n_images = 5
        mine = image_shard(n_images, rank, world)
        # each rank "predicts" its images: latent[i] filled with the image index
        preds = torch.stack([torch.full((4, 8, 8), float(i)) for i in mine])
        # ranks may hold different counts: pad to the largest shard for the gather
        most = len(image_shard(n_images, 0, world))
        pad = torch.full((most, 4, 8, 8), -1.0)
        pad[:len(mine)] = preds
        got = gather_latents(pad, world)
        slowest = max_over_ranks(10.0 + rank)
        if rank == 0:
            images = [t for r, g in enumerate(got) for t in g[:len(image_shard(n_images, r, world))]]
            q.put(("ok", [float(t[0, 0, 0]) for t in images], slowest))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(("error", traceback.format_exc(), None))


def test_image_shard_covers_every_image_once():
    for n in range(0, 20):
        for world in (1, 2, 3, 8):
            seen = [i for r in range(world) for i in image_shard(n, r, world)]
            assert seen == list(range(n))
            sizes = [len(image_shard(n, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        image_shard(4, 2, 2)


def test_gather_and_max_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    status, images, slowest = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert status == "ok", images
    assert images == [0.0, 1.0, 2.0, 3.0, 4.0]
    assert slowest == 11.0


def _failing_worker(rank, world, port, q, mode):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            if mode == "raise":
                raise RuntimeError("rank 1 failed before its step")
            return  # "exit": leaves without joining the collective
        t = torch.ones(3)
        dist.all_reduce(t)  # rank 0 waits for a peer that is gone
        q.put(("no error", None))
    except Exception as e:  # noqa: BLE001
        q.put(("error", f"rank {rank}: {type(e).__name__}"))


@pytest.mark.parametrize("mode", ["raise", "exit"])
def test_a_lost_rank_ends_the_collective_with_an_error(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        while len(results) < (2 if mode == "raise" else 1):
            results.append(q.get(timeout=90))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(r[0] == "error" for r in results), results
    assert any(r[1].startswith("rank 0") for r in results), results


# ---------------------------------------------------------------- CFG-parallel pairs
#
# A stand-in denoiser and solver step (deterministic torch float ops) replace
# the GPU ones: what is tested is the pairing, the order of the exchanged
# branches and that the two ranks of a pair stay bit-identical.

SIGMAS = [1.0, 0.7, 0.4, 0.0]
GUIDANCE = 4.0


def _start(image):
    return torch.randn(1, 4, 8, 8, generator=torch.Generator().manual_seed(100 + image))


def _context(image, branch):
    return torch.randn(1, 4, 8, 8, generator=torch.Generator().manual_seed(200 + 10 * image + branch))


def _predict(model_in, context):
    return torch.tanh(model_in * 0.5 + context)


def _solver_step(both, sample, step):
    uncond, cond = both[0:1], both[1:2]
    denoised = uncond + GUIDANCE * (cond - uncond)
    return sample + (SIGMAS[step + 1] - SIGMAS[step]) * denoised


def _one_image_on_one_rank(image):
    sample = _start(image)
    ctx = torch.cat([_context(image, 0), _context(image, 1)])
    for step in range(len(SIGMAS) - 1):
        both = _predict(sample.expand(2, -1, -1, -1), ctx)
        sample = _solver_step(both, sample, step)
    return sample


def _cfg_pair_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        pair = CfgPair(rank, world)
        sample = _start(pair.image)
        ctx = _context(pair.image, pair.branch)
        both = torch.empty(2, 4, 8, 8)
        for step in range(len(SIGMAS) - 1):
            mine = _predict(sample, ctx)                 # this rank's branch only
            pair.exchange(mine, both)                    # [uncond, cond] on both ranks
            sample = _solver_step(both, sample, step)
        q.put(("ok", rank, pair.image, pair.branch, sample))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(("error", rank, traceback.format_exc(), None, None))


@pytest.mark.parametrize("world", [2, 4])
def test_cfg_parallel_pairs_match_one_rank_per_image(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cfg_pair_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in results), [r[2] for r in results if r[0] != "ok"]
    for _, rank, image, branch, sample in results:
        assert (image, branch) == (rank // 2, rank % 2)
        assert torch.equal(sample, _one_image_on_one_rank(image)), (rank, image)


def test_cfg_pair_needs_an_even_job():
    with pytest.raises(ValueError):
        CfgPair(0, 3)
    with pytest.raises(ValueError):
        CfgPair(4, 4)
