"""Multi-rank exchange logic of the row-sharded scan, on CPU with gloo (world sizes 2 and 3).

The per-rank scan is the oracle (the GPU kernel's stand-in on CPU) and the
column merge a numpy restatement; the test checks the partition, the
certificate all-reduce, the column-list exchange (all-to-all by column block,
merge by the block's owner, all-gather of the merged blocks; every rank's copy)
and the candidate gather to rank 0 against a single-process oracle scan of the
whole problem; world size 3 gives uneven blocks.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(q=37, n=29, d=6, seed=5):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (x[rng.integers(0, q, n)] + 0.4 * rng.normal(size=(n, d))).astype(np.float32)
    a = (x.astype(np.float64) ** 2).sum(1)
    b = (y.astype(np.float64) ** 2).sum(1)
    f = 0.5 * a + rng.normal(size=q) * 3
    g = 0.5 * b + rng.normal(size=n) * 3
    return x, y, a, b, f, g


def _numpy_merge(vals, idx, k):
    parts, rows, width = vals.shape
    ov = np.full((rows, k), -np.inf)
    oi = np.full((rows, k), -1, dtype=np.int32)
    for r in range(rows):
        items = [(-vals[p, r, s], int(idx[p, r, s])) for p in range(parts) for s in range(width) if idx[p, r, s] >= 0]
        items.sort()
        for s, (v, i) in enumerate(items[:k]):
            ov[r, s], oi[r, s] = -v, i
    return torch.from_numpy(ov), torch.from_numpy(oi)


def _worker(rank, world, port, k, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "tests"))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        import __graft_entry__ as entry
        hb = entry.load_package()
        from hello_ot_b200.sharded import ShardedPricingScan, row_partition

        x, y, a, b, f, g = _problem()

        def local_scan(xs, ys, as_, bs, qb, dbb, kk):
            rv, ri, cv, ci, st = oracle.scan("raw", xs.numpy(), ys.numpy(), qb.numpy(), dbb.numpy(), as_.numpy(),
                                             bs.numpy(), dot_scale=2.0, rk=kk, ck=kk)
            return (torch.from_numpy(rv), torch.from_numpy(ri.astype(np.int32)), torch.from_numpy(cv),
                    torch.from_numpy(ci.astype(np.int32)), torch.from_numpy(st))

        def merge(v, i, kk):
            return _numpy_merge(v.numpy(), i.numpy(), kk)

        lo, hi = row_partition(len(x), world, rank)
        T = torch.from_numpy
        res = ShardedPricingScan(local_scan=local_scan, merge=merge).scan(
            T(x[lo:hi]), T(y), T(a[lo:hi]), T(b), T(f[lo:hi]), T(g), k, row_offset=lo)
        if rank == 0:
            np.savez(out_path, rows=res.rows.numpy(), cols=res.cols.numpy(), stats=res.stats.numpy(),
                     cv=res.col_vals.numpy(), ci=res.col_idx.numpy())
        else:
            assert res.rows is None and res.cols is None
            np.savez(f"{out_path}.{rank}.npz", cv=res.col_vals.numpy(), ci=res.col_idx.numpy(),
                     stats=res.stats.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_scan_matches_single_process(oracle, tmp_path, world):
    k = 3
    out = tmp_path / "res.npz"
    mp.spawn(_worker, args=(world, _free_port(), k, str(out)), nprocs=world, join=True)
    got = np.load(out)
    x, y, a, b, f, g = _problem()
    rv, ri, cv, ci, st = oracle.scan("raw", x, y, f - a, g - b, a, b, dot_scale=2.0, rk=k, ck=k)
    from parity import flatten
    rows, cols = flatten(rv, ri, cv, ci)
    assert np.array_equal(got["rows"], rows) and np.array_equal(got["cols"], cols)
    assert np.array_equal(got["ci"], ci) and np.array_equal(got["cv"], cv)
    np.testing.assert_allclose(got["stats"], st, rtol=1e-12)
    for r in range(1, world):  # every rank holds the same merged column lists and certificate
        other = np.load(f"{out}.{r}.npz")
        assert np.array_equal(other["ci"], ci) and np.array_equal(other["cv"], cv)
        np.testing.assert_allclose(other["stats"], st, rtol=1e-12)


def _pairs_worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "tests"))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        import __graft_entry__ as entry
        entry.load_package()
        from hello_ot_b200.sharded import ShardedPairCosts, row_partition

        x, y, a, b, _, _ = _problem()
        rng = np.random.default_rng(11)
        rows = rng.integers(0, len(x), 200)
        cols = rng.integers(0, len(y), 200)

        names = {0: "l1", 1: "linf", 2: "l2", 3: "raw"}

        def local_costs(kind, xs, ys, r, c, as_, bs, dot_scale):
            return torch.from_numpy(oracle.pair_costs(names[kind], xs.numpy(), ys.numpy(), r.numpy(), c.numpy(),
                                                      as_.numpy(), bs.numpy(), dot_scale=dot_scale))

        lo, hi = row_partition(len(x), world, rank)
        T = torch.from_numpy
        got = ShardedPairCosts(local_costs=local_costs).costs(T(rows), T(cols), T(x[lo:hi]), T(y), row_offset=lo,
                                                             a_block=T(a[lo:hi]), b=T(b))
        if rank == 0:
            np.savez(out_path, costs=got.numpy(), rows=rows, cols=cols)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_pair_costs_match_single_process(oracle, tmp_path, world):
    out = tmp_path / "pairs.npz"
    mp.spawn(_pairs_worker, args=(world, _free_port(), str(out)), nprocs=world, join=True)
    got = np.load(out)
    x, y, a, b, _, _ = _problem()
    want = oracle.pair_costs("raw", x, y, got["rows"], got["cols"], a, b, dot_scale=2.0)
    assert np.array_equal(got["costs"], want)


def test_row_partition_covers_rows(hb):
    from hello_ot_b200.sharded import row_partition
    for total in (1, 7, 100, 1_048_576):
        for world in (1, 2, 3, 8):
            spans = [row_partition(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(s[1] - s[0] for s in spans) - min(s[1] - s[0] for s in spans) <= 1
