"""Full-size checks (the baseline's config 5: m = n = 1,048,576, d = 256, k = 8).

At this size the exact top-k of every row cannot be recomputed in a test, so
the scan is checked through properties that do not depend on the size:
  * sampled rows and columns: the reported lists equal the exact fp64 top-k
    (torch fp64 on the GPU as exact arithmetic) wherever the boundary gap
    exceeds twice the stated error bound, and every value is within the bound;
  * row/column consistency: a pair that beats a column's k-th entry by more than
    the bound appears in that column's list;
  * the cost terms of the certificate do not depend on the duals (bitwise).
The PDHG is compared with the reference's own C++ solver (multithreaded) on a
medium support.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
N, D, K = 1_048_576, 256, 8
U32 = 2.0 ** -24


@pytest.fixture(scope="module")
def c5(cuda):
    g = torch.Generator(device=cuda)
    g.manual_seed(2024)
    x = torch.randn(N, D, device=cuda, generator=g)
    y = torch.randn(N, D, device=cuda, generator=g)
    a, b = (x.double() ** 2).sum(1), (y.double() ** 2).sum(1)
    f = torch.randn(N, device=cuda, dtype=torch.float64, generator=g) * 512
    gd = torch.randn(N, device=cuda, dtype=torch.float64, generator=g) * 512
    return x, y, a, b, f, gd


def _exact_rows(x, y, a, b, f, g, idx):
    """Exact fp64 scores of rows idx against every column (chunked)."""
    xs = x[idx].double()
    out = []
    for c0 in range(0, y.shape[0], 262144):
        dot = 2.0 * (xs @ y[c0:c0 + 262144].double().T)
        out.append((dot + (f - a)[idx, None]) + (g - b)[None, c0:c0 + 262144])
    return torch.cat(out, dim=1)


def _bound_rows(x, y, idx, cols):
    """3-term fp16 split + fp32-accumulation bound s (2^-19 + 2 (d+2) u) sum |x y| per pair,
    plus the fp16-subnormal floor s 2^-38 (max|x| sum|y_k| + max|y| sum|x_k|)."""
    ax = x[idx].abs().double()
    sabs = torch.stack([(ax[i] * y[cols[i]].abs().double()).sum(-1) for i in range(len(idx))])
    mx, my = float(x.abs().max()), float(y.abs().max())
    floor = torch.stack([mx * y[cols[i]].abs().double().sum(-1) + my * ax[i].sum() for i in range(len(idx))])
    return 2.0 * ((2.0 ** -19 + 2 * (D + 2) * U32) * sabs + 2.0 ** -38 * floor) + 1e-9


def test_l2sq_full_size_properties(hb, c5):
    x, y, a, b, f, g = c5
    rv, ri, cv, ci, stats = hb.l2sq_scan(x, y, a, b, f - a, g - b, K, dot_scale=2.0)
    torch.cuda.synchronize()
    # structure: sorted lists of valid, distinct indices
    assert bool((ri >= 0).all()) and bool((ri < N).all()) and bool((ci >= 0).all()) and bool((ci < N).all())
    assert bool((rv[:, :-1] >= rv[:, 1:]).all()) and bool((cv[:, :-1] >= cv[:, 1:]).all())
    # sampled rows against the exact top-k
    gen = torch.Generator().manual_seed(7)
    rows = torch.randint(0, N, (48,), generator=gen).to(x.device)
    exact = _exact_rows(x, y, a, b, f, g, rows)
    ev, ei = exact.topk(K + 1, dim=1)
    e = _bound_rows(x, y, rows, ri[rows].long())
    assert bool(((rv[rows] - exact.gather(1, ri[rows].long())).abs() <= e).all()), "row values off their scores"
    emax = e.max(dim=1).values
    clear = (ev[:, K - 1] - ev[:, K]) > 2 * emax
    for r in torch.nonzero(clear)[:, 0].tolist():
        assert set(ri[rows[r]].tolist()) == set(ei[r, :K].tolist())
    assert clear.float().mean() > 0.5
    # sampled columns, through the transposed problem
    cols = torch.randint(0, N, (48,), generator=gen).to(x.device)
    exact_c = _exact_rows(y, x, b, a, g, f, cols)  # score is symmetric in (x, f) <-> (y, g)
    cv_e, ci_e = exact_c.topk(K + 1, dim=1)
    ec = _bound_rows(y, x, cols, ci[cols].long())
    assert bool(((cv[cols] - exact_c.gather(1, ci[cols].long())).abs() <= ec).all()), "column values off"
    clear_c = (cv_e[:, K - 1] - cv_e[:, K]) > 2 * ec.max(dim=1).values
    for c in torch.nonzero(clear_c)[:, 0].tolist():
        assert set(ci[cols[c]].tolist()) == set(ci_e[c, :K].tolist())
    # row/column consistency: each row's best pair beats or ties into its column's list
    j = ri[:, 0].long()
    beats = rv[:, 0] > cv[j, K - 1] + 1e-6 * rv[:, 0].abs()
    i_all = torch.arange(N, device=x.device)
    present = (ci[j] == i_all[:, None].int()).any(dim=1)
    assert bool(present[beats].all()), "a row's best pair is missing from its column's list"


def test_l2sq_full_size_cost_terms_ignore_duals(hb, c5):
    x, y, a, b, f, g = c5
    s1 = hb.l2sq_scan(x, y, a, b, f - a, g - b, K, dot_scale=2.0)[4].cpu()
    s2 = hb.l2sq_scan(x, y, a, b, 0.5 * f - a, -g - b, K, dot_scale=2.0)[4].cpu()
    assert s1[1] == s2[1] and s1[3] == s2[3]


def test_pdlp_medium_support_matches_reference(hb, cuda, oracle):
    rng = np.random.default_rng(11)
    n = m = 3000
    extra = 12 * (n + m)
    rows = np.concatenate([np.arange(n), rng.integers(0, n, m), rng.integers(0, n, extra)])
    cols = np.concatenate([rng.integers(0, m, n), np.arange(m), rng.integers(0, m, extra)])
    key = np.unique(rows * m + cols)
    rows, cols = key // m, key % m
    cost = rng.random(rows.size) * 2
    a, b = np.full(n, 1.0 / n), np.full(m, 1.0 / m)
    lp = oracle.load_ref("lp")
    threads = os.cpu_count() or 1
    ref = lp.solve_once(rows, cols, cost, np.concatenate((a, b)), np.zeros(rows.size), np.zeros(n + m), n, threads,
                        200, 600.0, 2_000_000, 1e-6, 1e-6, 1e-6, False, False)
    got = hb.NativeRestrictedOTPDLP(device=cuda).solve_restricted(rows=rows, cols=cols, costs=cost, source_mass=a,
                                                                   target_mass=b, tolerance=1e-6)
    assert ref["termination_reason"] == got.termination_reason == "OPTIMAL"
    assert got.obj_val == pytest.approx(ref["obj_val"], rel=1e-6)
    assert got.primal_feas < 1e-6 and got.dual_feas < 1e-6 and got.gap < 1e-6
