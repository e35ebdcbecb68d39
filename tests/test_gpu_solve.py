"""End to end: the reference's ``hello_ot.solve(backend="native")`` on the B200 path.

The unmodified reference package (``baseline/_ref``) is bound to this library by
``hello_ot_b200.plugin.install`` and solves the baseline's configurations.  The
bar (the north star's): the final objective within 1e-6 relative of the
reference's own ``backend="cpp"`` solve (``tests/golden/solve_reference.json``,
made by ``make_solve_golden.py``; the reference's own relative gap is part of
its error, so the comparison allows the sum of both runs' reported gaps on top),
the full-space relative KKT error at most 1e-6, every scan, pair-cost, LP,
support and coarsest call routed to this package and none to the reference's
implementations; then the returned plan and duals are checked independently on
the CPU with the oracle: marginals, objective from fp64 costs, and the exact
full-space dual feasibility (a row sample for config 3).
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

import refpkg

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "solve_reference.json").read_text())
KKT_TOL = 1e-6
# the reported objective is the LP's primal objective; the returned plan keeps the entries above
# the reference's threshold, so sum(c * x) over it differs in the last digits (seen: 1.7e-9)
OBJ_RECOMPUTE_TOL = 1e-7


@pytest.fixture(scope="module")
def bound(hb, cuda):
    if not refpkg.available():
        pytest.skip("the reference package is not installed in baseline/_ref")
    hello_ot = refpkg.import_reference()
    from hello_ot_b200 import plugin
    plugin.install(hello_ot)
    yield hello_ot, plugin
    plugin.uninstall()


def _solve(bound, name, perturbation, n=None):
    hello_ot, plugin = bound
    from hello_ot.progress import final_metrics

    x, y, a, b, cost = refpkg.solve_config(name) if n is None else __import__("bench").solve_config(name, n=n)
    plugin.routes(reset=True)
    r = hello_ot.solve(x, y, source_mass=a, target_mass=b, cost=cost,
                       options=hello_ot.SolverOptions(backend="native", verbose="off",
                                                      cost_perturbation=perturbation))
    routes = plugin.routes()
    return (x, y, a, b, cost), r, final_metrics(r), routes


def _check_routes(routes):
    fallbacks = {k: v for k, v in routes.items() if k.startswith("reference:")}
    assert not fallbacks, f"reference implementations were called: {fallbacks}"
    assert sum(v for k, v in routes.items() if k.startswith("scan:")) > 0, routes
    assert sum(v for k, v in routes.items() if k.startswith("pair_costs:")) > 0, routes
    assert routes.get("lp:restricted_ot_pdhg", 0) > 0, routes
    assert routes.get("support:filter", 0) > 0, routes
    assert routes.get("coarsest:solve", 0) > 0, routes


def _oracle_check(oracle, inputs, r, *, sample_rows=None):
    """Plan marginals, objective and exact fp64 dual feasibility of the returned solution."""
    x, y, a, b, cost = inputs
    n, m = x.shape[0], y.shape[0]
    a = np.full(n, 1.0 / n) if a is None else np.asarray(a, np.float64)
    b = np.full(m, 1.0 / m) if b is None else np.asarray(b, np.float64)
    s = r.solution
    rows, cols, vals = s.rows, s.cols, s.values
    assert np.all(vals >= -1e-12)
    rs = np.bincount(rows, weights=vals, minlength=n)
    cs = np.bincount(cols, weights=vals, minlength=m)
    primal = math.sqrt(np.sum((rs - a) ** 2) + np.sum((cs - b) ** 2)) / (1 + math.sqrt(np.sum(a * a) + np.sum(b * b)))
    f, g = s.source_dual, s.target_dual
    if cost == "l2^2":
        xa = (x.astype(np.float64) ** 2).sum(1)
        yb = (y.astype(np.float64) ** 2).sum(1)
        kind, args = "raw", dict(nx=xa, ny=yb, dot_scale=2.0)
        rowb, colb = f - xa, g - yb
        c = oracle.pair_costs("raw", x, y, rows, cols, xa, yb, dot_scale=2.0)
    else:
        kind, args = cost, {}
        rowb, colb = f, g
        c = oracle.pair_costs(cost, x, y, rows, cols)
    objective = float(c @ vals)
    if sample_rows is None:
        stats = oracle.scan(kind, x, y, rowb, colb, rk=1, ck=1, **args)[4]
        dfeas = math.sqrt(stats[0]) / (1 + math.sqrt(stats[1]))
        max_violation = stats[2]
    else:  # a uniform row sample: its sums scaled by n / rows estimate the full-space terms
        pick = np.random.default_rng(0).choice(n, sample_rows, replace=False)
        sub = {k: (v[pick] if k == "nx" else v) for k, v in args.items()}
        stats = oracle.scan(kind, x[pick], y, rowb[pick], colb, rk=1, ck=1, **sub)[4]
        scale = n / sample_rows
        dfeas = math.sqrt(stats[0] * scale) / (1 + math.sqrt(stats[1] * scale))
        max_violation = stats[2]
    dual_objective = float(a @ f + b @ g)
    gap = abs(objective - dual_objective) / (1 + abs(objective) + abs(dual_objective))
    return dict(primal=primal, objective=objective, dual_feasibility=dfeas, max_violation=max_violation,
                gap=gap, cost_scale=float(np.abs(c).max()))


@pytest.mark.parametrize("perturbation", ["off", "auto"])
@pytest.mark.parametrize("name", ["C1", "C2"])
def test_solve_matches_reference_cpp(bound, oracle, name, perturbation):
    inputs, r, (pfeas, dfeas, gap, kkt), routes = _solve(bound, name, perturbation)
    _check_routes(routes)
    ref = GOLDEN[f"{name}/{perturbation}"]
    assert kkt is not None and kkt <= KKT_TOL, (pfeas, dfeas, gap)
    rel = abs(r.objective - ref["objective"]) / abs(ref["objective"])
    assert rel <= 1e-6 + abs(gap) + abs(ref["gap"]), (r.objective, ref["objective"], rel)
    chk = _oracle_check(oracle, inputs, r)
    assert chk["primal"] <= 2 * KKT_TOL, chk
    assert abs(chk["objective"] - r.objective) <= OBJ_RECOMPUTE_TOL * abs(r.objective), chk
    assert chk["dual_feasibility"] <= 2 * KKT_TOL, chk
    assert chk["gap"] <= 2 * KKT_TOL, chk


def test_solve_config3_kkt(bound, oracle):
    """Config 3 (ℓ1, 262144², d = 128): the reference's CPU backend cannot solve it here, so
    the bar is the relative KKT error and the oracle's independent checks (exact fp64 costs
    of the plan, marginals, duality gap, and the full-space dual feasibility estimated
    from 64 random full rows)."""
    inputs, r, (pfeas, dfeas, gap, kkt), routes = _solve(bound, "C3", "off")
    _check_routes(routes)
    assert kkt is not None and kkt <= KKT_TOL, (pfeas, dfeas, gap)
    chk = _oracle_check(oracle, inputs, r, sample_rows=64)
    assert chk["primal"] <= 2 * KKT_TOL, chk
    assert abs(chk["objective"] - r.objective) <= OBJ_RECOMPUTE_TOL * abs(r.objective), chk
    assert chk["gap"] <= 2 * KKT_TOL, chk
    assert chk["dual_feasibility"] <= 2 * KKT_TOL, chk
