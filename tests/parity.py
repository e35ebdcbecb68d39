"""Shared parity checks: top-k lists and certificates against exact fp64 scores.

The reference computes the ℓ2² dot products in fp32 (cuBLAS SGEMM on the GPU,
torch.mm on the CPU) and norm distances in fp32; this build computes them on
tcgen05 tensor cores (3-term fp16 split) or fp32 CUDA cores.  None of these agree
bit for bit, so candidate lists are compared against the exact fp64 scores of
the oracle with a stated per-pair error bound ``eps``: an index set must match
exactly wherever the exact score gap at the selection boundary exceeds
``2*eps``, every reported value must lie within ``eps`` of its exact score, and
every reported index must be a possible member of the exact top-k.
"""
from __future__ import annotations

import numpy as np

U32 = 2.0 ** -24  # unit roundoff of fp32
U64 = 2.0 ** -53


def l2sq_error_bound(x, y, rows, cols, scale, biases, accum_terms=None):
    """Error bound of an fp32-class score σ = (s<x,y> + qb) + dbb for pairs.

    |dot_fp32 - dot| <= (d+2) u Σ_k |x_k y_k| (sequential fp32 summation, the
    worst case of any summation order, plus the final rounding); the fp64
    additions add a few ulps of the largest operand.  ``biases`` is a tuple of
    arrays (indexed like rows/cols) whose magnitudes enter the fp64 rounding.
    """
    x = np.asarray(x, np.float64)
    y = np.asarray(y, np.float64)
    d = x.shape[1] if accum_terms is None else accum_terms
    absdot = np.einsum("ij,ij->i", np.abs(x[rows]), np.abs(y[cols]))
    mag = sum(np.abs(b) for b in biases) + scale * absdot
    return scale * (d + 2) * U32 * absdot + 16 * U64 * mag


def norm_error_bound(kind, x, y, rows, cols, f, g):
    x = np.asarray(x, np.float64)
    y = np.asarray(y, np.float64)
    diff = np.abs(x[rows] - y[cols])
    d = x.shape[1]
    if kind == "l1":
        dist = diff.sum(1)
        e = (d + 2) * U32 * dist
    elif kind == "linf":
        dist = diff.max(1)
        e = 2 * U32 * dist
    else:
        dist = np.sqrt((diff ** 2).sum(1))
        e = (d + 4) * U32 * dist
    return e + 16 * U64 * (np.abs(f[rows]) + np.abs(g[cols]) + dist)


def check_topk(test_v, test_i, exact_v, exact_i, pair_score, pair_eps, *, min_clear=0.5, label=""):
    """Compare one direction's top-k lists.

    test_v/test_i: (rows, k) from the implementation under test (-1 = missing).
    exact_v/exact_i: (rows, k+1) exact fp64 top-(k+1) from the oracle.
    pair_score(r, idx) -> exact scores; pair_eps(r, idx) -> error bounds.
    Returns the fraction of rows whose boundary was clear (compared exactly).
    """
    test_v = np.asarray(test_v)
    test_i = np.asarray(test_i).astype(np.int64)
    rows, k = test_i.shape
    assert exact_i.shape[0] == rows
    valid = test_i >= 0
    r_idx = np.repeat(np.arange(rows), k).reshape(rows, k)
    s = np.full(test_v.shape, -np.inf)
    e = np.zeros(test_v.shape)
    if valid.any():
        s[valid] = pair_score(r_idx[valid], test_i[valid])
        e[valid] = pair_eps(r_idx[valid], test_i[valid])
    # every reported value is its pair's score within eps
    assert np.all(np.abs(test_v[valid] - s[valid]) <= e[valid]), f"{label}: reported values off their scores"
    # missing slots agree with the exact list
    ex_missing = exact_i[:, :k] < 0
    assert np.array_equal(~valid, ex_missing), f"{label}: missing-slot pattern differs"
    # no duplicates
    for r in range(rows):
        ids = test_i[r][valid[r]]
        assert len(set(ids.tolist())) == ids.size, f"{label}: duplicate index in row {r}"
    emax = np.where(valid, e, 0).max(axis=1) if k else np.zeros(rows)
    kth = exact_v[:, k - 1]
    # every reported index could belong to the exact top-k
    ok = (~valid) | (s >= kth[:, None] - 2 * emax[:, None] - 1e-300)
    assert np.all(ok), f"{label}: an index outside the exact top-k band"
    nxt = exact_v[:, k] if exact_v.shape[1] > k else np.full(rows, -np.inf)
    clear = (kth - nxt) > 2 * emax + 0.0
    clear &= ~ex_missing.any(axis=1)
    for r in np.nonzero(clear)[0]:
        assert set(test_i[r].tolist()) == set(exact_i[r, :k].tolist()), f"{label}: row {r} set differs"
    if rows:
        assert clear.mean() >= min_clear or ex_missing.any(), f"{label}: only {clear.mean():.2f} rows clear"
    return float(clear.mean()) if rows else 1.0


def flatten(rv, ri, cv, ci, theta=0.0):
    """Candidate pairs in the reference order: query rows (row-major, slot order)
    then database columns (bilinear_topk.py:393-448, cpp_scan.py:169-171)."""
    rv, ri, cv, ci = map(np.asarray, (rv, ri, cv, ci))
    rm = (rv > theta) & (ri >= 0)
    cm = (cv > theta) & (ci >= 0)
    r_rows = np.repeat(np.arange(rv.shape[0]), rv.shape[1]).reshape(rv.shape)[rm]
    c_cols = np.repeat(np.arange(cv.shape[0]), cv.shape[1]).reshape(cv.shape)[cm]
    rows = np.concatenate((r_rows, ci[cm])).astype(np.int64)
    cols = np.concatenate((ri[rm], c_cols)).astype(np.int64)
    return rows, cols


def check_stats(test, exact, score, cost, eps, eps_cost=None, rel=0.0, label=""):
    """test/exact: [num, den, max_pos, max_abs_cost, count]; score/cost: exact fp64
    score and cost of every pair; eps / eps_cost: per-pair error bounds of the
    score / cost as the implementation under test evaluates them; rel: relative
    rounding of its partial sums.  Each sum may move by the sum of its terms'
    bounds, the count by the pairs within eps of 0."""
    test = np.asarray(test, np.float64)
    exact = np.asarray(exact, np.float64)
    s, c, e = (np.asarray(v, np.float64) for v in (score, cost, eps))
    ec = e if eps_cost is None else np.asarray(eps_cost, np.float64)
    tiny = 1e-12 * (1 + abs(exact[1]))
    pos = s > -e
    num_tol = float(np.sum((2 * np.abs(s) * e + e * e)[pos])) + rel * float(np.sum(np.maximum(s, 0) ** 2)) + tiny
    den_tol = float(np.sum(2 * np.abs(c) * ec + ec * ec)) + rel * exact[1] + 1e-12 * exact[1] + tiny
    assert abs(test[1] - exact[1]) <= den_tol, f"{label}: den {test[1]} vs {exact[1]} (tol {den_tol})"
    assert abs(test[0] - exact[0]) <= num_tol, f"{label}: num {test[0]} vs {exact[0]} (tol {num_tol})"
    assert abs(test[2] - exact[2]) <= e.max() + tiny, f"{label}: max+ {test[2]} vs {exact[2]}"
    assert abs(test[3] - exact[3]) <= ec.max() + tiny, f"{label}: max|c| {test[3]} vs {exact[3]}"
    assert abs(test[4] - exact[4]) <= int(np.sum(np.abs(s) <= e)), f"{label}: count {test[4]} vs {exact[4]}"
