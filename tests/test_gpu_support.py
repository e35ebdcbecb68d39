"""Active-support filter on the GPU through the C ABI: integer work, so the new
pairs must equal the reference's (fixtures) and the oracle's exactly."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("support_*.npz")))
def test_support_filter_golden(hb, cuda, path):
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    nr, nc, found, new = hb.filter_new_candidate_pairs(torch.as_tensor(z["active_keys"], device=cuda),
                                                       int(z["n_source"]), int(z["n_target"]), z["rows"], z["cols"])
    assert found == int(z["found"]) and new == int(z["new_count"])
    assert np.array_equal(nr.cpu().numpy(), z["new_rows"]) and np.array_equal(nc.cpu().numpy(), z["new_cols"])


@pytest.mark.parametrize("ns,nt,size,cand,sorted_", [(1, 1, 0, 5, False), (3000, 2000, 50000, 200000, False),
                                                     (3000, 2000, 50000, 200000, True), (70000, 90000, 10 ** 6,
                                                                                         3 * 10 ** 6, False)])
def test_support_filter_matches_oracle(hb, cuda, oracle, ns, nt, size, cand, sorted_):
    rng = np.random.default_rng(ns + cand)
    keys = rng.choice(ns * nt, size=size, replace=False).astype(np.int64)
    if sorted_:
        keys.sort()
    rows = np.concatenate([(keys[: size // 2] // nt), rng.integers(0, ns, cand)]).astype(np.int32)
    cols = np.concatenate([(keys[: size // 2] % nt), rng.integers(0, nt, cand)]).astype(np.int32)
    got = hb.filter_new_candidate_pairs(torch.as_tensor(keys, device=cuda), ns, nt, rows, cols, active_sorted=sorted_)
    ref = oracle.filter_new_pairs(keys, rows, cols, nt)
    assert got[2] == ref[2] and got[3] == ref[3]
    assert np.array_equal(got[0].cpu().numpy(), ref[0]) and np.array_equal(got[1].cpu().numpy(), ref[1])


def test_support_filter_edges(hb, cuda):
    keys = torch.tensor([3, 7], dtype=torch.int64, device=cuda)
    nr, nc, found, new = hb.filter_new_candidate_pairs(keys, 4, 4, np.zeros(0, np.int32), np.zeros(0, np.int32))
    assert (found, new) == (0, 0) and nr.numel() == 0
    # every candidate already present
    nr, nc, found, new = hb.filter_new_candidate_pairs(keys, 4, 4, [0, 1, 1], [3, 3, 3])
    assert (found, new) == (3, 0)
    with pytest.raises(ValueError):  # column out of range
        hb.filter_new_candidate_pairs(keys, 4, 4, [0], [4])


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("prune_*.npz")))
def test_prune_select_golden(hb, cuda, path):
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    pos = hb.select_prune_positions(z["rows"], z["cols"], z["costs"], z["x"], z["creation"], z["duals"],
                                    int(z["n_source"]), int(z["n_target"]), int(z["num"]), int(z["current"]))
    assert np.array_equal(pos, z["positions"])


@pytest.mark.parametrize("e,frac,ties", [(10, 0.3, False), (200000, 0.4, True), (3_000_000, 0.2, False)])
def test_prune_select_matches_oracle(hb, cuda, oracle, e, frac, ties):
    rng = np.random.default_rng(e)
    ns, nt = 5000, 4000
    rows = rng.integers(0, ns, e).astype(np.int32)
    cols = rng.integers(0, nt, e).astype(np.int32)
    costs = rng.random(e) * 3
    if ties:  # many exactly equal reduced costs, incl. signed zeros and non-finite values
        costs = np.round(costs)
        costs[:50] = np.inf
        costs[50:60] = np.nan
    x = np.where(rng.random(e) < 0.3, rng.random(e), 0.0)
    x[:5] = -0.0
    creation = rng.integers(-2, 6, e).astype(np.int32)
    duals = np.zeros(ns + nt) if ties else rng.normal(size=ns + nt)
    num = int(frac * e)
    ref, nrem = oracle.prune_select(rows, cols, costs, x, creation, duals, ns, num, 5)
    if ref is None:
        with pytest.raises(RuntimeError, match="invariant violated"):
            hb.select_prune_positions(rows, cols, costs, x, creation, duals, ns, nt, num, 5)
        return
    got = hb.select_prune_positions(rows, cols, costs, x, creation, duals, ns, nt, num, 5)
    assert np.array_equal(got, ref)


def test_prune_select_too_few(hb, cuda):
    with pytest.raises(RuntimeError, match="invariant violated"):
        hb.select_prune_positions([0, 1], [0, 1], [1.0, 2.0], [1.0, 0.0], [0, 0], np.zeros(4), 2, 2, 2, 5)
