"""Scans on the baseline's end-to-end configurations and the product scan entry point.

* config 2 (ℓ2, n = m = 32768, d = 3): the whole scan against the oracle's fp32 model,
  both directions: lists identical bit for bit, certificate to summation order;
* config 3 (ℓ1, n = m = 262144, d = 128, 16-component mixtures): 32 sampled rows and 32
  sampled columns against the oracle's fp32 model, bit for bit;
* raw_lowrank_bidir_feasibility_pricing_scan, the function the reference's refinement
  loop calls (src/hello_ot/kernels/bilinear_topk.py:207), on the reference-generated
  fixtures: the candidate pairs equal the reference's except pairs inside the fp32 band of
  the reference's own dots, the certificate within fp32-class rounding.
Duals: N(0, 1) x the median pair cost (65536 sampled pairs), as config 5 specifies for
the isolated scans.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import bench

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _duals(oracle, kind, x, y, seed):
    rng = np.random.default_rng(seed)
    r, c = rng.integers(0, len(x), 65536), rng.integers(0, len(y), 65536)
    med = float(np.median(oracle.pair_costs(kind, x, y, r, c)))
    return rng.normal(size=len(x)) * med, rng.normal(size=len(y)) * med


@pytest.mark.parametrize("k", [2, 8])
def test_config2_l2_scan_full_vs_oracle(hb, cuda, oracle, k):
    x, y, _, _, cost = bench.solve_config("C2")
    assert cost == "l2"
    f, g = _duals(oracle, "l2", x, y, seed=5)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    rv, ri, cv, ci, stats = (t.cpu().numpy() for t in hb.norm_scan(T(x, torch.float32), T(y, torch.float32),
                                                                    T(f, torch.float64), T(g, torch.float64), k, "l2"))
    ev, ei, fv, fi, es = oracle.scan("l2", x, y, f, g, rk=k, ck=k, exact=False)
    assert np.array_equal(ri, ei) and np.array_equal(ci, fi)
    assert np.array_equal(rv, ev) and np.array_equal(cv, fv)
    assert stats[2] == es[2] and stats[3] == es[3] and stats[4] == es[4]
    np.testing.assert_allclose(stats[:2], es[:2], rtol=1e-12)


def test_config3_l1_scan_sampled_rows_and_columns(hb, cuda, oracle):
    x, y, _, _, cost = bench.solve_config("C3")
    assert cost == "l1"
    k = 8
    f, g = _duals(oracle, "l1", x, y, seed=6)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    rv, ri, cv, ci, _ = (t.cpu().numpy() for t in hb.norm_scan(T(x, torch.float32), T(y, torch.float32),
                                                                T(f, torch.float64), T(g, torch.float64), k, "l1"))
    rng = np.random.default_rng(7)
    rows = np.sort(rng.choice(len(x), 32, replace=False))
    cols = np.sort(rng.choice(len(y), 32, replace=False))
    ev, ei, _, _, _ = oracle.scan("l1", x[rows], y, f[rows], g, rk=k, ck=0, exact=False)
    _, _, fv, fi, _ = oracle.scan("l1", x, y[cols], f, g[cols], rk=0, ck=k, exact=False)
    assert np.array_equal(ri[rows], ei) and np.array_equal(rv[rows], ev)
    assert np.array_equal(ci[cols], fi) and np.array_equal(cv[cols], fv)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("scan_l2sq_*.npz")))
@pytest.mark.parametrize("exact", [True, False])
def test_product_pricing_scan_matches_reference(hb, cuda, oracle, path, exact):
    with np.load(GOLDEN / path) as z:
        z = {key: z[key] for key in z.files}
    k = int(z["k"])
    res = hb.raw_lowrank_bidir_feasibility_pricing_scan(z["x"], z["y"], z["a"], z["b"], z["f"], z["g"], topk=k,
                                                        dot_scale=2.0, exact=exact)
    assert res.rows.dtype == np.int64 and res.cols.dtype == np.int64
    ours = set(zip(res.rows.tolist(), res.cols.tolist()))
    ref = set(zip(z["rows"].tolist(), z["cols"].tolist()))
    assert len(ours ^ ref) <= max(2, len(ref) // 100), f"{len(ours ^ ref)} candidate differences"
    assert res.dual_feasibility == pytest.approx(float(z["dual_feasibility"]), rel=1e-5)
    if exact:  # every candidate is an exact fp64 top-k member with a positive exact score
        score = oracle.pair_scores("raw", z["x"], z["y"], z["f"] - z["a"], z["g"] - z["b"], z["a"], z["b"],
                                   res.rows, res.cols, dot_scale=2.0)[0]
        assert np.all(score > -1e-9 * (1.0 + np.abs(z["f"]).max() + np.abs(z["g"]).max()))


def test_product_pricing_scan_fp64_precision(hb, cuda):
    """compute_precision="fp64" on features holding fp32 values (given as fp64 arrays) gives the
    exact fp64 lists: the same candidates and certificate as the fp32 features with exact=True."""
    path = sorted(GOLDEN.glob("scan_l2sq_*.npz"))[0]
    with np.load(path) as z:
        z = {key: z[key] for key in z.files}
    k = int(z["k"])
    args = (z["a"], z["b"], z["f"], z["g"])
    ref = hb.raw_lowrank_bidir_feasibility_pricing_scan(z["x"], z["y"], *args, topk=k, dot_scale=2.0, exact=True)
    got = hb.raw_lowrank_bidir_feasibility_pricing_scan(z["x"].astype(np.float64), z["y"].astype(np.float64), *args,
                                                        topk=k, dot_scale=2.0, compute_precision="fp64", exact=False)
    assert np.array_equal(got.rows, ref.rows) and np.array_equal(got.cols, ref.cols)
    assert got.dual_feasibility == ref.dual_feasibility
    assert got.diagnostics["fp64_recheck"] and got.diagnostics["cost_compute_precision"] == "fp64"

