"""Coarsest-level exact transport on the GPU.

``solve_leaf_from_cost`` stands in for the reference's POT leaf solve
(``_solve_lowrank_leaf_with_pot_from_precomputed_cost``,
src/hello_ot/hierarchy/coarsest.py:50-154, which calls ``ot.emd(a, b, M, log=True)``):
it solves the dense transport LP of a coarsest level (n, m <= a few thousand)
with the library's restarted Halpern PDHG on the complete support to a tight
relative KKT tolerance and returns the same fields: the plan entries above
1e-12 as a sparse warm start, the duals (u, v) with c_ij - u_i - v_j >= 0 up to
the tolerance, and the distance.  Unlike a network simplex the plan is an
interior optimum when the LP has several (the objective agrees to the
tolerance); the hierarchy only needs an optimal warm start and its duals.
"""
from __future__ import annotations

import time
from types import SimpleNamespace
from typing import Any, Dict

import numpy as np
import torch

from .pdlp import NativeRestrictedOTPDLP


def solve_leaf_from_cost(*, cost, source_mass, target_mass, tolerance: float = 1e-9, device="cuda",
                         **_unused) -> Dict[str, Any]:
    """Dense OT between source_mass (n) and target_mass (m) with cost (n x m)."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("solve_leaf_from_cost runs on CUDA devices only")
    c = torch.as_tensor(np.asarray(cost, dtype=np.float64) if not torch.is_tensor(cost) else cost,
                        dtype=torch.float64, device=dev)
    if c.dim() != 2:
        raise ValueError("cost must be an n x m matrix")
    n, m = c.shape
    a = torch.as_tensor(source_mass, dtype=torch.float64, device=dev).view(-1)
    b = torch.as_tensor(target_mass, dtype=torch.float64, device=dev).view(-1)
    if a.numel() != n or b.numel() != m:
        raise ValueError("mass vectors do not match the cost matrix")
    t0 = time.perf_counter()
    rows = torch.arange(n, device=dev, dtype=torch.int64).repeat_interleave(m)
    cols = torch.arange(m, device=dev, dtype=torch.int64).repeat(n)
    solver = NativeRestrictedOTPDLP(device=dev, evaluation_frequency=200, summation="tree")
    res = solver.solve_restricted(rows=rows, cols=cols, costs=c.reshape(-1), source_mass=a, target_mass=b,
                                  tolerance=float(tolerance))
    solve_time = time.perf_counter() - t0
    x = res.x if torch.is_tensor(res.x) else torch.as_tensor(res.x, device=dev)
    y = res.y if torch.is_tensor(res.y) else torch.as_tensor(res.y, device=dev)
    keep = x > 1e-12
    r, cc, v = rows[keep], cols[keep], x[keep]
    distance = float((v * c[r, cc]).sum())
    warm = SimpleNamespace(rows=r.to(torch.int32).cpu().numpy(), cols=cc.to(torch.int32).cpu().numpy(),
                           x_prev=v.cpu().numpy(), dual_uv=y.cpu().numpy(), n_source=int(n), n_target=int(m))
    return {
        "distance": distance,
        "time": solve_time,
        "lp_solve_time_total": solve_time,
        "warm_start_state": warm,
        "termination_reason": res.termination_reason,
        "iterations": int(res.iterations),
        "leaf_stage_profile": {"pdhg_solve_time": solve_time, "cost_build_backend": "precomputed"},
        "level_summaries": [{"level": 0, "n_source": int(n), "n_target": int(m), "iters": int(res.iterations),
                             "time": solve_time, "objective": distance, "lp_time": solve_time,
                             "pricing_time": 0.0, "support_final": int(r.numel())}],
    }
