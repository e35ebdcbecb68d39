"""Generate the golden fixtures in this folder from the reference implementation.

Run with HELLO_REF naming a checkout of the reference project, after
``make -C oracle ref REF=$HELLO_REF``:

    HELLO_REF=<reference checkout> python tests/golden/make_golden.py

It imports the reference's Python package with its C++ CPU backend
(``oracle/_ref/hello_ot_cpp``, compiled from the reference sources) and records
its outputs on small seeded inputs.  The fixtures pin the oracle
(tests/test_oracle_golden.py) and, on the GPU, the CUDA path.  The GPU box
never runs this script: only the committed ``.npz`` files travel.

Reference entry points recorded:
  * ℓ2² scan:  hello_ot.kernels.cpp_scan.fused_dot_tile / cpp_violation_scan
               (src/hello_ot/kernels/cpp_scan.py:9-21, 95-182)
  * norm scan: hello_ot.kernels.torch_scan.bidirectional_violation_scan
               (src/hello_ot/kernels/torch_scan.py:337)
  * PDLP:      CppRestrictedOTPDLP / TorchRestrictedOTPDLP
               (src/hello_ot/_internal/lp/{cpp,torch}_restricted_ot.py)
  * directional (initial) scans: hello_ot.kernels.torch_scan.directional_assignment
               (src/hello_ot/kernels/torch_scan.py:165-291), known side = target
  * pair costs: hello_ot.costs.pairs._cost_pairs_lowrank_batched (CPU branch,
               src/hello_ot/costs/pairs.py:296-307) and
               hello_ot.costs.metric.pair_costs_metric(compute_precision="fp64")
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("HELLO_REF"):
    raise SystemExit("set HELLO_REF to a checkout of the reference project")
REF = Path(os.environ["HELLO_REF"])
sys.path.insert(0, str(REF / "src"))
sys.path.insert(0, str(REPO / "oracle" / "_ref"))

import torch  # noqa: E402

torch.set_num_threads(1)

from hello_ot.kernels.cpp_scan import cpp_violation_scan, fused_dot_tile  # noqa: E402
from hello_ot.kernels.torch_scan import bidirectional_violation_scan, directional_assignment  # noqa: E402
from hello_ot._internal.lp.cpp_restricted_ot import CppRestrictedOTPDLP  # noqa: E402
from hello_ot._internal.lp.torch_restricted_ot import TorchRestrictedOTPDLP  # noqa: E402
from hello_ot.costs.pairs import _cost_pairs_lowrank_batched  # noqa: E402
from hello_ot.costs.metric import pair_costs_metric  # noqa: E402
from hello_ot.restricted_ot.active_support import ActiveSupport  # noqa: E402
from hello_ot.refinement.budgeted_pruning import DualGapCleaning  # noqa: E402
from hello_ot.costs.metric_perturbation import (_apply_metric_pair_perturbation, _index_hash_parameters,  # noqa: E402
                                                _metric_index_hash_noise_numpy)

SCAN_L2SQ = [  # (name, q, n, d, k, seed, dual scale)
    ("l2sq_a", 37, 53, 8, 3, 1, 1.0),
    ("l2sq_b", 64, 48, 33, 8, 2, 1.5),
    ("l2sq_c", 200, 150, 16, 2, 3, 1.0),
    ("l2sq_d", 5, 3, 4, 8, 4, 1.0),      # fewer columns than k
    ("l2sq_e", 96, 130, 64, 32, 5, 0.5),
    ("l2sq_f", 129, 257, 5, 1, 6, 1.0),  # ragged tile edges
]
SCAN_NORM = [  # (name, cost, q, n, d, k, seed)
    ("l1_a", "l1", 41, 29, 3, 2, 11),
    ("l1_b", "l1", 64, 80, 20, 8, 12),
    ("l2_a", "l2", 33, 47, 3, 4, 13),
    ("l2_b", "l2", 50, 70, 17, 1, 14),
    ("linf_a", "linf", 45, 38, 2, 3, 15),
    ("linf_b", "linf", 72, 60, 9, 16, 16),
]


def _points(rng, q, n, d):
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (x[rng.integers(0, q, size=n)] + 0.5 * rng.normal(size=(n, d))).astype(np.float32)
    return x, y


def l2sq_case(name, q, n, d, k, seed, dual_scale):
    rng = np.random.default_rng(seed)
    x, y = _points(rng, q, n, d)
    a = np.sum(x.astype(np.float64) ** 2, axis=1)
    b = np.sum(y.astype(np.float64) ** 2, axis=1)
    scale = float(np.median(a)) * dual_scale
    f = rng.normal(size=q) * scale * 0.3 + 0.5 * a
    g = rng.normal(size=n) * scale * 0.3 + 0.5 * b
    rk, ck = min(k, n), min(k, q)
    rv = torch.full((q, rk), -torch.inf, dtype=torch.float64)
    ri = torch.full((q, rk), -1, dtype=torch.int64)
    cv = torch.full((n, ck), -torch.inf, dtype=torch.float64)
    ci = torch.full((n, ck), -1, dtype=torch.int64)
    num, den, cnt, mx, cm = fused_dot_tile(torch.from_numpy(x), torch.from_numpy(y), torch.from_numpy(a),
                                          torch.from_numpy(b), torch.from_numpy(f), torch.from_numpy(g),
                                          rv, ri, cv, ci, 2.0, 0, 0, 0)
    flat = cpp_violation_scan(source_points=x, target_points=y, source_offset=a, target_offset=b,
                              source_dual=f, target_dual=g, score_family="inner_product", cost_type="lowrank",
                              dot_scale=2.0, topk=k, theta=0.0, device="cpu")
    np.savez_compressed(HERE / f"scan_{name}.npz", kind="l2^2", x=x, y=y, a=a, b=b, f=f, g=g, k=k, dot_scale=2.0,
                        rv=rv.numpy(), ri=ri.numpy(), cv=cv.numpy(), ci=ci.numpy(),
                        stats=np.array([num, den, mx, cm, cnt], dtype=np.float64),
                        rows=np.asarray(flat.rows), cols=np.asarray(flat.cols),
                        dual_feasibility=flat.dual_feasibility)


def norm_case(name, cost, q, n, d, k, seed):
    rng = np.random.default_rng(seed)
    x, y = _points(rng, q, n, d)
    x = np.abs(x) if cost == "l1" else x
    diff = np.abs(x[:, None, :].astype(np.float64) - y[None, :, :])
    med = float(np.median(diff.sum(2) if cost == "l1" else diff.max(2) if cost == "linf"
                          else np.sqrt((diff ** 2).sum(2))))
    f = rng.normal(size=q) * med * 0.4 + 0.5 * med
    g = rng.normal(size=n) * med * 0.4 + 0.5 * med
    res = bidirectional_violation_scan(source_points=x, target_points=y, source_offset=None, target_offset=None,
                                       source_dual=f, target_dual=g, score_family="norm_cost", cost_type=cost,
                                       dot_scale=1.0, topk=k, theta=0.0, device="cpu")
    dg = res.diagnostics
    np.savez_compressed(HERE / f"scan_{name}.npz", kind=cost, x=x, y=y, f=f, g=g, k=k,
                        rows=np.asarray(res.rows), cols=np.asarray(res.cols),
                        stats=np.array([dg["dual_feasibility_num_sq"], dg["dual_feasibility_den_sq"],
                                        dg["dual_feasibility_max_violation"], dg["dual_feasibility_cost_linf"],
                                        dg["dual_feasibility_positive_count"]], dtype=np.float64),
                        dual_feasibility=res.dual_feasibility)


DIRECTIONAL = [  # (name, family, cost, q, n, d, k, seed)
    ("l2sq_a", "inner_product", "lowrank", 70, 90, 12, 8, 41),
    ("l2sq_b", "inner_product", "lowrank", 33, 20, 40, 32, 42),   # k > n
    ("l1_a", "norm_cost", "l1", 64, 75, 3, 16, 43),
    ("l2_a", "norm_cost", "l2", 50, 41, 9, 4, 44),
    ("linf_a", "norm_cost", "linf", 48, 66, 2, 1, 45),
]


def directional_case(name, family, cost, q, n, d, k, seed):
    """Known side = target: each source row's best k of g_j - c_ij (the reference keeps
    the candidate pairs and the top-1 value / index of each row)."""
    from types import SimpleNamespace
    rng = np.random.default_rng(seed)
    x, y = _points(rng, q, n, d)
    a = np.sum(x.astype(np.float64) ** 2, axis=1)
    b = np.sum(y.astype(np.float64) ** 2, axis=1)
    g = rng.normal(size=n) * (float(np.median(a)) if family == "inner_product" else 2.0)
    f = np.zeros(q)
    state = SimpleNamespace(rows=np.zeros(0, np.int32), cols=np.zeros(0, np.int32), x_prev=np.zeros(0),
                            dual_uv=np.concatenate([f, g]), n_source=q, n_target=n)
    aug, _, _, cand = directional_assignment(
        state=state, source_points=x, target_points=y,
        source_offset=a if family == "inner_product" else None, target_offset=b if family == "inner_product" else None,
        score_family=family, cost_type=cost, dot_scale=2.0, known_side="target", topk=k, device="cpu")
    np.savez_compressed(HERE / f"directional_{name}.npz", family=family, cost=cost, x=x, y=y, a=a, b=b, g=g, k=k,
                        rows=np.asarray(aug.rows, np.int64), cols=np.asarray(aug.cols, np.int64),
                        top1_values=cand.values.numpy(), top1_indices=cand.indices.numpy())


def support_cases():
    """ActiveSupport.filter_new_candidate_pairs (active_support.py:483-506) on CPU."""
    rng = np.random.default_rng(51)
    for name, ns, nt, size, cand in (("a", 40, 30, 200, 500), ("b", 1000, 700, 20000, 30000), ("empty", 50, 60, 0, 300)):
        keys = rng.choice(ns * nt, size=size, replace=False)
        rows, cols = keys // nt, keys % nt
        sup = ActiveSupport(n_source=ns, n_target=nt, device="cpu")
        sup.initialize_from_arrays(rows=rows, cols=cols, costs=np.zeros(size), x_prev=np.zeros(size))
        # candidates: some already in the support, some repeated
        cr = np.concatenate([rows[: size // 3], rng.integers(0, ns, cand)])
        cc = np.concatenate([cols[: size // 3], rng.integers(0, nt, cand)])
        dup = rng.integers(0, cr.size, cand // 5)
        cr, cc = np.concatenate([cr, cr[dup]]), np.concatenate([cc, cc[dup]])
        nr, nc, found, new = sup.filter_new_candidate_pairs(cr, cc)
        np.savez_compressed(HERE / f"support_{name}.npz", n_source=ns, n_target=nt, active_keys=keys.astype(np.int64),
                            rows=cr.astype(np.int32), cols=cc.astype(np.int32), new_rows=nr.numpy(),
                            new_cols=nc.numpy(), found=found, new_count=new)


def prune_cases():
    """DualGapCleaning.select_indices_to_remove, protect-new mode (budgeted_pruning.py:177-201)."""
    rng = np.random.default_rng(61)
    for name, ns, nt, size, frac in (("a", 30, 40, 400, 0.2), ("b", 800, 600, 20000, 0.35)):
        keys = rng.choice(ns * nt, size=size, replace=False)
        rows, cols = keys // nt, keys % nt
        costs = rng.random(size) * 3
        x = np.where(rng.random(size) < 0.3, rng.random(size), 0.0)
        creation = rng.integers(-2, 6, size).astype(np.int32)  # -1 structural, -2 initial, 5 = current
        duals = rng.normal(size=ns + nt)
        costs[:7] = np.round(costs[:7])   # a few exactly tied reduced costs
        duals_t = duals.copy()
        sup = ActiveSupport(n_source=ns, n_target=nt, device="cpu")
        sup.initialize_from_arrays(rows=rows, cols=cols, costs=costs, x_prev=x, creation_iteration=creation)
        num = int(frac * size)
        out = DualGapCleaning().select_indices_to_remove(sup, num, duals=duals_t, n_source=ns, current_inner_iter=5)
        np.savez_compressed(HERE / f"prune_{name}.npz", n_source=ns, n_target=nt, rows=rows.astype(np.int32),
                            cols=cols.astype(np.int32), costs=costs, x=x, creation=creation, duals=duals,
                            num=num, current=5, positions=np.asarray(out, np.int32))


def perturb_cases():
    """Norm-cost perturbation (metric_perturbation.py): index-hash noise, its coefficients,
    perturbed metric pair costs, and a perturbed torch norm scan (torch_scan.py:488-503)."""
    rng = np.random.default_rng(71)
    seed = 1234
    src = np.concatenate([rng.integers(0, 5000, 400), rng.integers(0, 3_000_000, 400), [0, 2002, 2003, 4021]])
    tgt = np.concatenate([rng.integers(0, 5000, 400), rng.integers(0, 3_000_000, 400), [2010, 2011, 0, 4022]])
    coeffs = np.asarray(sum(_index_hash_parameters(seed), ()), np.int64)
    x = rng.normal(size=(70, 9)).astype(np.float32)
    y = rng.normal(size=(50, 9)).astype(np.float32)
    rows, cols = rng.integers(0, 70, 600), rng.integers(0, 50, 600)
    si, ti = rng.permutation(1_000_000)[:70], rng.permutation(1_000_000)[:50]
    out = {}
    for cost in ("l1", "l2", "linf"):
        base = np.asarray(pair_costs_metric(source_points=x, target_points=y, rows=rows, cols=cols, cost_type=cost,
                                            compute_precision="fp64"))
        out[f"pairs_{cost}"] = np.asarray(_apply_metric_pair_perturbation(
            base, rows, cols, {"mode": "full_cost_perturb", "sigma": 0.05, "seed": seed, "noise": "index_hash",
                               "source_global_index": si, "target_global_index": ti}))
    # a perturbed ℓ1 scan (the torch tile path adds the noise in the tile's dtype)
    med = 6.0
    f = rng.normal(size=70) * med * 0.4 + 0.5 * med
    g = rng.normal(size=50) * med * 0.4 + 0.5 * med
    pert = {"mode": "full_cost_perturb", "sigma": 0.3, "seed": seed, "noise": "index_hash",
            "source_global_index": si, "target_global_index": ti}
    res = bidirectional_violation_scan(source_points=x, target_points=y, source_offset=None, target_offset=None,
                                       source_dual=f, target_dual=g, score_family="norm_cost", cost_type="l1",
                                       dot_scale=1.0, topk=4, theta=0.0, device="cpu", perturbation=pert)
    np.savez_compressed(HERE / "perturb.npz", src=src, tgt=tgt, seed=seed, coeffs=coeffs,
                        noise=_metric_index_hash_noise_numpy(src, tgt, seed=seed), x=x, y=y, rows=rows, cols=cols,
                        si=si, ti=ti, f=f, g=g, scan_rows=np.asarray(res.rows), scan_cols=np.asarray(res.cols),
                        dual_feasibility=res.dual_feasibility, **out)


def pdlp_cases():
    cases = []
    rng = np.random.default_rng(12)
    r, c = np.indices((7, 5))
    cases.append(("dense7x5", r.ravel(), c.ravel(), rng.random(35), np.full(7, 1 / 7), np.full(5, 1 / 5), None, None))
    cases.append(("small2x2", np.array([0, 0, 1, 1]), np.array([0, 1, 0, 1]), np.array([0.0, 2.0, 1.0, 0.0]),
                  np.array([0.4, 0.6]), np.array([0.5, 0.5]), np.array([0.35, 0.05, 0.15, 0.45]), np.zeros(4)))
    rng = np.random.default_rng(21)
    ns, nt = 30, 40
    rows = np.concatenate([np.arange(ns), rng.integers(0, ns, 180)])
    cols = np.concatenate([rng.integers(0, nt, ns), rng.integers(0, nt, 180)])
    rows = np.concatenate([rows, rng.integers(0, ns, nt)])
    cols = np.concatenate([cols, np.arange(nt)])
    key = np.unique(rows * nt + cols)
    rows, cols = key // nt, key % nt
    perm = rng.permutation(rows.size)
    rows, cols = rows[perm], cols[perm]
    wa, wb = rng.uniform(0.5, 1.5, ns), rng.uniform(0.5, 1.5, nt)
    cost = rng.random(rows.size) * 3
    cases.append(("sparse30x40", rows, cols, cost, wa / wa.sum(), wb / wb.sum(), None, None))
    cases.append(("sparse30x40_warm", rows, cols, cost, wa / wa.sum(), wb / wb.sum(),
                  rng.random(rows.size) * 0.01, rng.normal(size=ns + nt) * 0.1))
    for name, rows, cols, cost, a, b, x0, y0 in cases:
        out = {}
        for label, solver, tol, limit in (("cpp40", CppRestrictedOTPDLP(num_threads=1, evaluation_frequency=5,
                                                                        iteration_limit=40), 0.0, 40),
                                          ("cpp", CppRestrictedOTPDLP(num_threads=1, evaluation_frequency=20,
                                                                      iteration_limit=200000), 1e-7, 200000),
                                          ("torch40", TorchRestrictedOTPDLP(evaluation_frequency=5,
                                                                            iteration_limit=40), 0.0, 40)):
            res = solver.solve_restricted(rows=rows, cols=cols, costs=cost, source_mass=a, target_mass=b,
                                          warm_start_primal=x0, warm_start_dual=y0, tolerance=tol)
            out[f"{label}_x"] = np.asarray(res.x)
            out[f"{label}_y"] = np.asarray(res.y)
            out[f"{label}_meta"] = np.array([res.iterations, res.solver_diag["restart_count"], res.obj_val,
                                             res.primal_feas, res.dual_feas, res.gap], dtype=np.float64)
            out[f"{label}_reason"] = np.array(res.termination_reason)
            out[f"{label}_limit"] = limit
        np.savez_compressed(HERE / f"pdlp_{name}.npz", rows=np.asarray(rows, np.int64), cols=np.asarray(cols, np.int64),
                            costs=np.asarray(cost, np.float64), source_mass=a, target_mass=b,
                            x0=np.zeros(0) if x0 is None else x0, y0=np.zeros(0) if y0 is None else y0, **out)


def pairs_cases():
    rng = np.random.default_rng(31)
    for d in (3, 16, 70):
        x = rng.normal(size=(60, d)).astype(np.float32)
        y = rng.normal(size=(45, d)).astype(np.float32)
        rows = rng.integers(0, 60, 500)
        cols = rng.integers(0, 45, 500)
        a = np.sum(x.astype(np.float64) ** 2, axis=1)
        b = np.sum(y.astype(np.float64) ** 2, axis=1)
        lowrank = _cost_pairs_lowrank_batched(dict(F=x, G=y, a=a, b=b, dot_scale=2.0), rows, cols)
        norms = {c: np.asarray(pair_costs_metric(source_points=x, target_points=y, rows=rows, cols=cols,
                                                 cost_type=c, compute_precision="fp64"))
                 for c in ("l1", "l2", "linf")}
        np.savez_compressed(HERE / f"pairs_d{d}.npz", x=x, y=y, a=a, b=b, rows=rows, cols=cols,
                            lowrank=np.asarray(lowrank), **norms)


if __name__ == "__main__":
    for case in SCAN_L2SQ:
        l2sq_case(*case)
    for case in SCAN_NORM:
        norm_case(*case)
    for case in DIRECTIONAL:
        directional_case(*case)
    support_cases()
    prune_cases()
    perturb_cases()
    pdlp_cases()
    pairs_cases()
    print("fixtures written to", HERE)
