"""Multi-GPU decomposition of the bench (CPU): R x S grids of row/column-band
shards.  BAG only combines blocks at equal offsets, so the recursion on rank
(i, j)'s compact shards (row band i of every block-row of A, column band j of
every block-column of B) must equal the full BAG product restricted to those
rows and columns -- bit for bit with sequential-fmaf leaves."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import bench
from oracle import bag_oracle as O


def _inputs(n, seed=0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, n), dtype=np.float32),
            rng.standard_normal((n, n), dtype=np.float32))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_grid_covers_every_index_once(world):
    n, depth = 256, 2
    gr, gc = bench.shard_grid(world)
    assert gr * gc == world
    for g in (gr, gc):
        owned = np.concatenate([bench.band_rows(n, depth, g, r) for r in range(g)])
        assert np.array_equal(np.sort(owned), np.arange(n))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_restriction_is_exact(world):
    n, depth = 128, 2
    a, b = _inputs(n)
    full = O.bag_product(a, b, depth, "minimal", leaf="fmaf")
    gr, gc = bench.shard_grid(world)
    for rank in range(world):
        rows = bench.band_rows(n, depth, gr, rank // gc)
        cols = bench.band_rows(n, depth, gc, rank % gc)
        part = O.bag_product(np.ascontiguousarray(a[rows]), np.ascontiguousarray(b[:, cols]), depth,
                             "minimal", leaf="fmaf")
        assert np.array_equal(part, full[np.ix_(rows, cols)]), rank


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, depth, out_path):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a, b = _inputs(n)
    gr, gc = bench.shard_grid(world)
    rows = bench.band_rows(n, depth, gr, rank // gc)
    cols = bench.band_rows(n, depth, gc, rank % gc)
    part = O.bag_product(np.ascontiguousarray(a[rows]), np.ascontiguousarray(b[:, cols]), depth,
                         "minimal", leaf="fmaf")
    parts = [torch.empty(part.shape, dtype=torch.float32) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(part))
    if rank == 0:
        c = np.empty((n, n), dtype=np.float32)
        for r, p in enumerate(parts):
            rr = bench.band_rows(n, depth, gr, r // gc)
            cc = bench.band_rows(n, depth, gc, r % gc)
            c[np.ix_(rr, cc)] = p.numpy()
        np.save(out_path, c)
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_gloo_reassemble_the_full_product(tmp_path):
    import torch.multiprocessing as mp
    n, depth, world = 128, 2, 2
    out = str(tmp_path / "c.npy")
    mp.spawn(_rank_main, args=(world, _free_port(), n, depth, out), nprocs=world, join=True)
    a, b = _inputs(n)
    assert np.array_equal(np.load(out), O.bag_product(a, b, depth, "minimal", leaf="fmaf"))
