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


def _noise(seed, step):
    return torch.randn(1, 4, 8, 8, generator=torch.Generator().manual_seed(300 + 10 * seed + step))


def _solver_step(both, sample, step, noise=None):
    """A deterministic Euler-like step, or with `noise` an ancestral one (the
    shape of Euler a: a deterministic move plus fresh noise scaled by the
    step)."""
    uncond, cond = both[0:1], both[1:2]
    denoised = uncond + GUIDANCE * (cond - uncond)
    out = sample + (SIGMAS[step + 1] - SIGMAS[step]) * denoised
    if noise is not None:
        out = out + 0.3 * SIGMAS[step + 1] * noise
    return out


def _one_image_on_one_rank(image, stochastic=False):
    sample = _start(image)
    ctx = torch.cat([_context(image, 0), _context(image, 1)])
    for step in range(len(SIGMAS) - 1):
        both = _predict(sample.expand(2, -1, -1, -1), ctx)
        sample = _solver_step(both, sample, step, _noise(image, step) if stochastic else None)
    return sample


def _cfg_pair_worker(rank, world, port, q, noise_seed):
    """noise_seed: None (deterministic step), "image" (both ranks of a pair
    draw the noise from the image's seed, as CfgPair requires) or "rank" (a
    per-rank seed: the mistake the requirement guards against)."""
    try:
        _init(rank, world, port)
        pair = CfgPair(rank, world)
        sample = _start(pair.image)
        ctx = _context(pair.image, pair.branch)
        both = torch.empty(2, 4, 8, 8)
        for step in range(len(SIGMAS) - 1):
            mine = _predict(sample, ctx)                 # this rank's branch only
            pair.exchange(mine, both)                    # [uncond, cond] on both ranks
            noise = None
            if noise_seed == "image":
                noise = _noise(pair.image, step)
            elif noise_seed == "rank":
                noise = _noise(100 + rank, step)
            sample = _solver_step(both, sample, step, noise)
        q.put(("ok", rank, pair.image, pair.branch, sample))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(("error", rank, traceback.format_exc(), None, None))


def _run_pairs(world, noise_seed):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cfg_pair_worker, args=(r, world, port, q, noise_seed)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in results), [r[2] for r in results if r[0] != "ok"]
    return sorted(results, key=lambda r: r[1])


@pytest.mark.parametrize("world", [2, 4])
def test_cfg_parallel_pairs_match_one_rank_per_image(world):
    for _, rank, image, branch, sample in _run_pairs(world, None):
        assert (image, branch) == (rank // 2, rank % 2)
        assert torch.equal(sample, _one_image_on_one_rank(image)), (rank, image)


def test_cfg_pairs_with_a_stochastic_step_need_the_image_seed():
    """With an ancestral (noisy) step the two ranks of a pair stay
    bit-identical, and equal to one rank per image, when both draw the noise
    from the image's seed; with per-rank seeds they drift apart."""
    for _, rank, image, _, sample in _run_pairs(2, "image"):
        assert torch.equal(sample, _one_image_on_one_rank(image, stochastic=True)), rank
    r = _run_pairs(2, "rank")
    assert not torch.equal(r[0][4], r[1][4])


def _exchange_checks_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        pair = CfgPair(rank, world)
        mine = torch.ones(1, 4, 8, 8) * rank
        errors = 0
        for bad in (torch.empty(2, 8, 8, 4).permute(0, 3, 1, 2),   # right shape, not contiguous
                    torch.empty(2, 4, 8, 8, dtype=torch.float64),    # wrong dtype
                    torch.empty(3, 4, 8, 8)):                        # wrong shape
            try:
                pair.exchange(mine, bad)
            except ValueError:
                errors += 1
        both = pair.exchange(mine)
        q.put(("ok", rank, errors, both[:, 0, 0, 0].tolist()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(("error", rank, traceback.format_exc(), None))


def test_cfg_pair_exchange_rejects_unusable_outputs():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_checks_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in results), [r[2] for r in results if r[0] != "ok"]
    for _, _, errors, got in results:
        assert errors == 3 and got == [0.0, 1.0]


def test_cfg_pair_needs_an_even_job():
    with pytest.raises(ValueError):
        CfgPair(0, 3)
    with pytest.raises(ValueError):
        CfgPair(4, 4)
