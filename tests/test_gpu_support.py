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
