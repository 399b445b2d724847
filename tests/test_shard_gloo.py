"""Multi-process (gloo, world_size 2 and 3, CPU) tests of the image sharding + latent gather."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zimage_b200.shard import gather_images, image_seeds, shard_range


def test_shard_range_covers_all():
    for n in (1, 5, 16):
        for w in (1, 2, 3, 4, 8):
            got = [shard_range(n, w, r) for r in range(w)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(got[i][1] == got[i + 1][0] for i in range(w - 1))
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fake_step(seed: int) -> torch.Tensor:
    """Stand-in for one image's latents: deterministic in the image seed only."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(4, 8, 8, generator=g)


def _worker(rank, world, port, n_images, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        seeds = image_seeds(n_images)
        a, b = shard_range(n_images, world, rank)
        local = torch.stack([_fake_step(s) for s in seeds[a:b]]) if b > a else torch.zeros(0, 4, 8, 8)
        full = gather_images(local, n_images)
        out[rank] = full
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_images", [(2, 16), (3, 16), (2, 3)])
def test_gather_matches_single_process(world, n_images):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_images, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = torch.stack([_fake_step(s) for s in image_seeds(n_images)])
    for r in range(world):
        assert torch.equal(out[r], want)


def _failing_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        if rank == 1:
            raise SystemExit(3)  # a rank leaves before the gather
        gather_images(torch.zeros(1, 2), 2)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_gather_fails_loudly_when_a_rank_leaves():
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode != 0  # the surviving rank's collective errors out (bounded timeout)
