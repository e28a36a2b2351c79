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


def _gather_main(rank, world, port, n, depth, out_dir):
    """One rank of the bench's e2e input path: upload only this rank's pieces,
    all-gather inside the row and column groups, compare with the shards."""
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a, b = _inputs(n, seed=5)
    gr, gc = bench.shard_grid(world)
    rows = bench.band_rows(n, depth, gr, rank // gc)
    cols = bench.band_rows(n, depth, gc, rank % gc)
    a_shard, b_shard = np.ascontiguousarray(a[rows]), np.ascontiguousarray(b[:, cols])
    pc = bench.upload_pieces(rows.size, n, gr, gc, rank)
    rgs = [dist.new_group([i * gc + j for j in range(gc)]) for i in range(gr)]
    cgs = [dist.new_group([i * gc + j for i in range(gr)]) for j in range(gc)]
    assert pc["row_group"] == [rank // gc * gc + j for j in range(gc)]
    assert pc["col_group"] == [i * gc + rank % gc for i in range(gr)]
    a_piece = torch.from_numpy(np.ascontiguousarray(a_shard[slice(*pc["a_rows"])]))
    b_piece = torch.from_numpy(np.ascontiguousarray(b_shard[slice(*pc["b_rows"])]))
    a_parts = [torch.empty_like(a_piece) for _ in range(gc)]
    b_parts = [torch.empty_like(b_piece) for _ in range(gr)]
    dist.all_gather(a_parts, a_piece, group=rgs[rank // gc])
    dist.all_gather(b_parts, b_piece, group=cgs[rank % gc])
    ok = (np.array_equal(torch.cat(a_parts).numpy(), a_shard)
          and np.array_equal(torch.cat(b_parts).numpy(), b_shard))
    uploaded = a_piece.numel() + b_piece.numel()
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([int(ok), uploaded]))
    dist.barrier()
    dist.destroy_process_group()


def test_e2e_pieces_gather_into_the_shards_and_upload_each_byte_once(tmp_path):
    """world 4 = 2 x 2 grid over gloo: every rank's shards are rebuilt from the
    group all-gathers, and the ranks upload A and B exactly once in total."""
    import torch.multiprocessing as mp
    n, depth, world = 128, 2, 4
    mp.spawn(_gather_main, args=(world, _free_port(), n, depth, str(tmp_path)), nprocs=world,
             join=True)
    res = [np.load(tmp_path / f"r{r}.npy") for r in range(world)]
    assert all(int(r[0]) == 1 for r in res)
    assert sum(int(r[1]) for r in res) == 2 * n * n
