"""Tensor-parallel sharding on the host: gloo ranks on CPU, oracle arithmetic.

Column-parallel shards (blocks of output rows) concatenate to the full
product; row-parallel shards (blocks of whole groups along K) sum to it.
The sum runs as a world-size-2 (and 4) gloo all_reduce, the way the GPU path
sums partials over NCCL or NVLink peer memory.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import q4_oracle as O
from siliconfer_b200 import quant as Q
from siliconfer_b200.tensor_parallel import shard_bounds, shard_column, shard_row


def test_shard_bounds_even_and_uneven():
    assert [shard_bounds(28672, 8, r, 128) for r in range(8)] == [(r * 3584, (r + 1) * 3584) for r in range(8)]
    # 7B down_proj: 86 groups over 4 ranks -> 22, 22, 21, 21 groups
    b = [shard_bounds(11008, 4, r, 128) for r in range(4)]
    assert [(hi - lo) // 128 for lo, hi in b] == [22, 22, 21, 21]
    assert b[0][0] == 0 and b[-1][1] == 11008 and all(b[i][1] == b[i + 1][0] for i in range(3))
    with pytest.raises(ValueError):
        shard_bounds(100, 2, 0, 128)
    with pytest.raises(ValueError):
        shard_bounds(256, 4, 0, 128)


@pytest.mark.parametrize("asym", [False, True])
def test_shards_reassemble_the_packed_triple(asym):
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.02, (96, 1024)).astype(np.float32)
    trip = Q.pack_weights_asym(w, 128) if asym else (*Q.pack_weights_sym(w, 128), None)
    p, s, z = trip
    cols = [shard_column(p, s, z, r, 3) for r in range(3)]
    assert np.array_equal(np.concatenate([c[0] for c in cols]), p)
    assert np.array_equal(np.concatenate([c[1] for c in cols]), s)
    rows = [shard_row(p, s, z, 128, r, 3) for r in range(3)]
    assert np.array_equal(np.concatenate([r[0] for r in rows], axis=1), p)
    assert np.array_equal(np.concatenate([r[1] for r in rows], axis=1), s)
    if asym:
        assert np.array_equal(np.concatenate([r[2] for r in rows], axis=1), z)
        assert np.array_equal(np.concatenate([c[2] for c in cols]), z)


def test_column_shards_keep_heads_whole():
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.02, (8 * 64, 256)).astype(np.float32)   # 8 heads of 64 rows
    p, s = Q.pack_weights_sym(w, 128)
    for world in (1, 2, 4, 8):
        blocks = [shard_column(p, s, None, r, world, unit=64) for r in range(world)]
        assert all(b[0].shape[0] == 8 // world * 64 for b in blocks)
        assert np.array_equal(np.concatenate([b[0] for b in blocks]), p)
    with pytest.raises(ValueError, match="heads"):
        shard_column(p, s, None, 0, 3, unit=64)       # 8 heads over 3 ranks
    with pytest.raises(ValueError, match="heads"):
        shard_column(p[:100], s[:100], None, 0, 2, unit=64)   # not whole heads


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, asym, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)
        n, k, gs, t = 64, 1024, 128, 3
        w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
        x = rng.normal(0, 1, (t, k)).astype(np.float32)
        p, s, z = Q.pack_weights_asym(w, gs) if asym else (*Q.pack_weights_sym(w, gs), None)
        full = O.gemm(p, s, z, x, gs)
        # row-parallel: partial over this rank's groups, summed over ranks
        ps, ss, zs, (k0, k1) = shard_row(p, s, z, gs, rank, world)
        part = torch.from_numpy(O.gemm(ps, ss, zs, np.ascontiguousarray(x[:, k0:k1]), gs).astype(np.float64))
        dist.all_reduce(part)
        err_row = O.normwise_rel_err(part.numpy().astype(np.float32), full)
        # column-parallel: this rank's rows, gathered
        pc, sc, zc, _ = shard_column(p, s, z, rank, world)
        mine = torch.from_numpy(O.gemm(pc, sc, zc, x, gs))
        lo, hi = shard_bounds(n, world, rank)
        parts = [torch.empty((t, b - a)) for a, b in (shard_bounds(n, world, r) for r in range(world))]
        dist.all_gather(parts, mine)
        err_col = float(np.max(np.abs(torch.cat(parts, dim=1).numpy() - full)))
        q.put((rank, err_row, err_col, (lo, hi)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("asym", [False, True])
def test_row_and_column_parallel_match_unsharded_gloo(world, asym):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, asym, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    for rank, err_row, err_col, _ in res:
        assert err_row <= 1e-6, (rank, err_row)
        assert err_col == 0.0, (rank, err_col)
