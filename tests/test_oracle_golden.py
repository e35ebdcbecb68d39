"""Pin the oracle against the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py from the reference
package and its C++ backend compiled from the reference sources.  These tests
need no GPU and no reference checkout.
"""
from pathlib import Path

import numpy as np
import pytest

from parity import check_stats, check_topk, flatten, l2sq_error_bound, norm_error_bound

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    with np.load(GOLDEN / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("scan_l2sq_*.npz")))
def test_l2sq_scan_oracle_matches_reference(oracle, path):
    z = _load(path)
    x, y, a, b, f, g, k = z["x"], z["y"], z["a"], z["b"], z["f"], z["g"], int(z["k"])
    q, n = len(x), len(y)
    rk, ck = min(k, n), min(k, q)
    qb, dbb = f - a, g - b
    rv, ri, cv, ci, stats = oracle.scan("raw", x, y, qb, dbb, a, b, dot_scale=2.0,
                                        rk=min(rk + 1, n), ck=min(ck + 1, q))
    if rv.shape[1] == rk:  # no (k+1)-th column available: pad with -inf
        rv = np.pad(rv, ((0, 0), (0, 1)), constant_values=-np.inf)
        ri = np.pad(ri, ((0, 0), (0, 1)), constant_values=-1)
    if cv.shape[1] == ck:
        cv = np.pad(cv, ((0, 0), (0, 1)), constant_values=-np.inf)
        ci = np.pad(ci, ((0, 0), (0, 1)), constant_values=-1)

    def score(r, c):
        return oracle.pair_scores("raw", x, y, qb, dbb, a, b, r, c, dot_scale=2.0)[0]

    def eps(r, c):
        return l2sq_error_bound(x, y, r, c, 2.0, (a[r], b[c], f[r], g[c]))

    check_topk(z["rv"], z["ri"], rv, ri, score, eps, label=path + ":rows")
    check_topk(z["cv"], z["ci"], cv, ci, lambda r, c: score(c, r), lambda r, c: eps(c, r), label=path + ":cols")
    all_r, all_c = np.divmod(np.arange(q * n), n)
    s, c = oracle.pair_scores("raw", x, y, qb, dbb, a, b, all_r, all_c, dot_scale=2.0)
    check_stats(z["stats"], stats, s, c, eps(all_r, all_c), label=path)
    # candidate flattening order of the reference CPU scan
    rows, cols = flatten(z["rv"], z["ri"], z["cv"], z["ci"])
    assert np.array_equal(rows, z["rows"]) and np.array_equal(cols, z["cols"])


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("scan_*.npz")
                                        if not p.name.startswith("scan_l2sq_")))
def test_norm_scan_oracle_matches_reference(oracle, path):
    z = _load(path)
    kind, x, y, f, g, k = str(z["kind"]), z["x"], z["y"], z["f"], z["g"], int(z["k"])
    q, n = len(x), len(y)
    rk, ck = min(k, n), min(k, q)
    rv, ri, cv, ci, stats = oracle.scan(kind, x, y, f, g, rk=rk, ck=ck)
    rows, cols = flatten(rv, ri, cv, ci)
    ours = set(zip(rows.tolist(), cols.tolist()))
    ref = set(zip(z["rows"].tolist(), z["cols"].tolist()))
    diff = np.array(sorted(ours ^ ref), dtype=np.int64).reshape(-1, 2)
    if diff.size:
        s, _ = oracle.pair_scores(kind, x, y, f, g, None, None, diff[:, 0], diff[:, 1])
        e = norm_error_bound(kind, x, y, diff[:, 0], diff[:, 1], f, g)
        # a pair may only differ when its score is within the error band of the θ=0 cut
        # or of its row's / column's k-th score
        full_r, _, full_c, _, _ = oracle.scan(kind, x, y, f, g, rk=rk, ck=ck)
        near = (np.abs(s) <= 2 * e) | (np.abs(s - full_r[diff[:, 0], rk - 1]) <= 2 * e) \
            | (np.abs(s - full_c[diff[:, 1], ck - 1]) <= 2 * e)
        assert near.all(), f"{path}: {int((~near).sum())} unexplained candidate differences"
    all_r, all_c = np.divmod(np.arange(q * n), n)
    s, c = oracle.pair_scores(kind, x, y, f, g, None, None, all_r, all_c)
    check_stats(z["stats"], stats, s, c, norm_error_bound(kind, x, y, all_r, all_c, f, g), label=path)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("pdlp_*.npz")))
def test_pdlp_oracle_matches_reference(oracle, path):
    z = _load(path)
    x0 = z["x0"] if z["x0"].size else None
    y0 = z["y0"] if z["y0"].size else None
    args = (z["rows"], z["cols"], z["costs"], z["source_mass"], z["target_mass"], x0, y0)
    # 40 iterations, evaluation every 5, tolerance 0: same operation order as the
    # single-thread reference, so the iterates agree bit for bit
    r = oracle.pdlp(*args, frequency=5, iteration_limit=40, tolerance=0.0)
    assert r["iterations"] == 40 and r["termination_reason"] == "ITERATION_LIMIT"
    assert np.array_equal(r["x"], z["cpp40_x"]) and np.array_equal(r["y"], z["cpp40_y"])
    assert r["restarts"] == int(z["cpp40_meta"][1])
    # and within round-off of the Torch restatement
    np.testing.assert_allclose(r["x"], z["torch40_x"], atol=2e-11, rtol=2e-10)
    np.testing.assert_allclose(r["y"], z["torch40_y"], atol=2e-11, rtol=2e-10)
    # converged solve
    r = oracle.pdlp(*args, frequency=20, iteration_limit=200000, tolerance=1e-7)
    meta = z["cpp_meta"]
    assert r["termination_reason"] == str(z["cpp_reason"]) == "OPTIMAL"
    assert r["iterations"] == int(meta[0]) and r["restarts"] == int(meta[1])
    assert np.array_equal(r["x"], z["cpp_x"]) and np.array_equal(r["y"], z["cpp_y"])
    assert r["obj_val"] == meta[2]


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("pairs_*.npz")))
def test_pair_costs_oracle_matches_reference(oracle, path):
    z = _load(path)
    x, y, rows, cols = z["x"], z["y"], z["rows"], z["cols"]
    out = oracle.pair_costs("raw", x, y, rows, cols, z["a"], z["b"], dot_scale=2.0)
    # the reference evaluates a+b-2<x,y> entirely in fp32
    e = l2sq_error_bound(x, y, rows, cols, 2.0, (z["a"][rows], z["b"][cols]))
    e += 4 * 2.0 ** -24 * (np.abs(z["a"][rows]) + np.abs(z["b"][cols]) + np.abs(out))
    assert np.all(np.abs(out - z["lowrank"]) <= e)
    for kind in ("l1", "l2", "linf"):
        got = oracle.pair_costs(kind, x, y, rows, cols)
        np.testing.assert_allclose(got, z[kind], rtol=1e-13, atol=0)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("directional_*.npz")))
def test_directional_oracle_matches_reference(oracle, path):
    """The reference's directional assignment (known side = target): each source row's
    best k of g_j - c_ij.  The oracle's row lists (no source bias) give the same pairs
    except inside the fp32 error band, and the same top-1 scores within it."""
    z = _load(path)
    x, y, g, k = z["x"], z["y"], z["g"], int(z["k"])
    q, n = len(x), len(y)
    rk = min(k, n)
    if str(z["family"]) == "inner_product":
        a, b = z["a"], z["b"]
        rowb, colb, kind = -a, g - b, "raw"
        rv, ri, _, _, _ = oracle.scan(kind, x, y, rowb, colb, a, b, dot_scale=2.0, rk=min(rk + 1, n), ck=0)
        score = lambda r, c: oracle.pair_scores(kind, x, y, rowb, colb, a, b, r, c, dot_scale=2.0)[0]  # noqa: E731
        # the reference evaluates g - ((a + b) - 2 fp32(x y^T)): fp32 dot error plus fp64 rounding
        bound = lambda r, c: l2sq_error_bound(x, y, r, c, 2.0, (a[r], b[c], g[c])) + 1e-12 * (a[r] + b[c])  # noqa: E731
    else:
        kind = str(z["cost"])
        rowb, colb = np.full(q, -0.0), g
        rv, ri, _, _, _ = oracle.scan(kind, x, y, rowb, colb, rk=min(rk + 1, n), ck=0, exact=False)
        score = lambda r, c: oracle.pair_scores(kind, x, y, rowb, colb, None, None, r, c)[0]  # noqa: E731
        bound = lambda r, c: norm_error_bound(kind, x, y, r, c, rowb, colb)  # noqa: E731
    # top-1 value and index of every row
    r_all = np.arange(q)
    e1 = bound(r_all, z["top1_indices"])
    assert np.all(np.abs(rv[:, 0] - z["top1_values"]) <= 2 * e1 + 1e-300)
    same = ri[:, 0] == z["top1_indices"]
    gap = rv[:, 0] - (rv[:, 1] if rv.shape[1] > 1 else -np.inf)
    assert np.all(same | (gap <= 2 * e1)), f"{path}: top-1 index differs outside the error band"
    # the candidate pairs: each row's top-k set
    ref = set(zip(z["rows"].tolist(), z["cols"].tolist()))
    ours = {(r, int(c)) for r in range(q) for c in ri[r, :rk] if c >= 0}
    diff = np.array(sorted(ours ^ ref), dtype=np.int64).reshape(-1, 2)
    if diff.size:
        s = score(diff[:, 0], diff[:, 1])
        e = bound(diff[:, 0], diff[:, 1])
        kth = rv[diff[:, 0], rk - 1]
        assert np.all(np.abs(s - kth) <= 2 * e + 1e-300), f"{path}: candidate differences outside the error band"


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("support_*.npz")))
def test_support_filter_oracle_matches_reference(oracle, path):
    z = _load(path)
    nr, nc, found, new = oracle.filter_new_pairs(z["active_keys"], z["rows"], z["cols"], int(z["n_target"]))
    assert found == int(z["found"]) and new == int(z["new_count"])
    assert np.array_equal(nr, z["new_rows"]) and np.array_equal(nc, z["new_cols"])


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("prune_*.npz")))
def test_prune_oracle_matches_reference(oracle, path):
    z = _load(path)
    pos, _ = oracle.prune_select(z["rows"], z["cols"], z["costs"], z["x"], z["creation"], z["duals"],
                                 int(z["n_source"]), int(z["num"]), int(z["current"]))
    assert np.array_equal(pos, z["positions"])


def test_perturbation_noise_matches_reference(oracle, hb):
    """Index-hash noise bit for bit against the reference's NumPy form, and the
    coefficients the host layer derives from the seed."""
    z = _load("perturb.npz")
    seed = int(z["seed"])
    from hello_ot_b200.perturb import index_hash_coefficients  # host logic, no GPU
    assert tuple(z["coeffs"].tolist()) == index_hash_coefficients(seed)
    got = oracle.noise(z["src"], z["tgt"], 1.0, seed, 1, z["coeffs"])
    assert np.array_equal(got, z["noise"].astype(np.float64))
    # perturbed metric pair costs: fp64 distance + sigma * noise
    for kind in ("l1", "l2", "linf"):
        base = oracle.pair_costs(kind, z["x"], z["y"], z["rows"], z["cols"])
        pert = base + oracle.noise(z["si"][z["rows"]], z["ti"][z["cols"]], 0.05, seed, 1, z["coeffs"])
        np.testing.assert_allclose(pert, z[f"pairs_{kind}"], rtol=1e-13, atol=0)
