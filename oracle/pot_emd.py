"""Stand-in for POT's ``ot.emd`` (TEST INFRASTRUCTURE ONLY).

The reference solves each coarsest hierarchy level with POT
(``_solve_lowrank_leaf_with_pot_from_precomputed_cost``,
src/hello_ot/hierarchy/coarsest.py:50-154, which calls
``ot.emd(a, b, M, numItermax=10_000_000, log=True)``).  POT (PyPI ``pot``, a
dependency of the reference whose version is not pinned beyond ``>=0.9.7``) is
not installed in this image, so the reference's own CPU runs (``backend="cpp"``)
that produce the solve objectives the tests compare against use this module in
its place: the same balanced transport LP, solved exactly by SciPy's HiGHS
simplex, returning a vertex plan and the equality-constraint duals (u, v) with
``log = {"cost", "u", "v", "warning", "result_code"}``.  The duals are centred
as POT's ``center_ot_dual`` does (u + c, v - c with c = (b.v - a.u)/(sum a +
sum b)).  When the LP has several optimal vertices or duals HiGHS may pick
another one than POT's network simplex; the optimal cost is the same.

Only tests/, the golden-fixture scripts and bench.py's reference (CPU) arm use
it; the product package never does.
"""
from __future__ import annotations

import sys
import types

import numpy as np


def emd(a, b, M, numItermax=10_000_000, log=False, center_dual=True, **_unused):
    import scipy.sparse as sp
    from scipy.optimize import linprog

    a = np.asarray(a, dtype=np.float64).reshape(-1)
    b = np.asarray(b, dtype=np.float64).reshape(-1)
    M = np.asarray(M, dtype=np.float64)
    n, m = M.shape
    if a.size != n or b.size != m:
        raise ValueError("mass vectors do not match the cost matrix")
    var = np.arange(n * m)
    rows = sp.csr_matrix((np.ones(n * m), (var // m, var)), shape=(n, n * m))
    cols = sp.csr_matrix((np.ones(n * m), (var % m, var)), shape=(m, n * m))
    res = linprog(M.reshape(-1), A_eq=sp.vstack([rows, cols]).tocsr(), b_eq=np.concatenate([a, b]),
                  bounds=(0, None), method="highs")
    if res.status != 0:
        raise RuntimeError(f"emd stand-in: HiGHS status {res.status}: {res.message}")
    plan = res.x.reshape(n, m)
    if not log:
        return plan
    duals = np.asarray(res.eqlin.marginals, dtype=np.float64)
    u, v = duals[:n].copy(), duals[n:].copy()
    if center_dual:
        c = (b.dot(v) - a.dot(u)) / (a.sum() + b.sum())
        u += c
        v -= c
    return plan, {"cost": float(res.fun), "u": u, "v": v, "warning": None, "result_code": 1}


def install() -> types.ModuleType:
    """Register this stand-in as the module ``ot`` (only when POT is absent)."""
    try:
        import ot  # noqa: F401
        return sys.modules["ot"]
    except ImportError:
        pass
    module = types.ModuleType("ot")
    module.emd = emd
    module.__doc__ = "ot.emd stand-in (oracle/pot_emd.py): SciPy HiGHS on the dense transport LP"
    sys.modules["ot"] = module
    return module
