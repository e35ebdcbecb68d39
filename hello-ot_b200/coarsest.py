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

from .pairs import pair_costs
from .pdlp import NativeRestrictedOTPDLP

PLAN_THRESHOLD = 1e-12  # plan entries kept as the warm start (coarsest.py:88, gpu_resident/solver.py:184)
COST_KINDS = {"l1": 0, "linf": 1, "l2": 2, "l2^2": 3}


def leaf_cost_matrix(source, target, kind: str, *, source_offset=None, target_offset=None,
                     perturbation=None) -> torch.Tensor:
    """Dense n x m fp64 cost of a coarsest level, built on the device by the pair-cost
    kernel over every (i, j) (the reference builds it tile by tile on the host for POT:
    gpu_resident/cost.py:73-89 `Cost.tile`, gpu_resident/solver.py:172-180).  l2^2 needs
    the fp64 squared norms as source_offset / target_offset (c = a_i + b_j - 2 <x_i, y_j>)."""
    if kind not in COST_KINDS:
        raise ValueError(f"kind must be one of {sorted(COST_KINDS)}")
    if kind == "l2^2" and (source_offset is None or target_offset is None):
        raise ValueError("l2^2 needs source_offset and target_offset")
    n, m, dev = source.shape[0], target.shape[0], source.device
    rows = torch.arange(n, device=dev, dtype=torch.int64).repeat_interleave(m)
    cols = torch.arange(m, device=dev, dtype=torch.int64).repeat(n)
    return pair_costs(COST_KINDS[kind], source, target, rows, cols, a=source_offset, b=target_offset, dot_scale=2.0,
                      perturbation=perturbation).view(n, m)


def _solve_dense(cost, source_mass, target_mass, tolerance, device):
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("the coarsest solve runs on CUDA devices only")
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
    if res.termination_reason != "OPTIMAL":
        raise RuntimeError(f"coarsest solve did not converge: {res.termination_reason}")
    keep = res.x > PLAN_THRESHOLD
    keys = torch.nonzero(keep).view(-1)  # i * m + j: the complete support is in row-major order
    values = res.x[keep]
    distance = float((values * c.view(-1)[keys]).sum())
    return keys, values, res.y, distance, res, time.perf_counter() - t0, n, m


def solve_leaf_resident(cost, source_mass, target_mass, *, tolerance: float = 1e-9) -> SimpleNamespace:
    """Device-resident leaf (the gpu_resident path's `_leaf`, gpu_resident/solver.py:168-192):
    cost is an n x m CUDA tensor; returns keys (i*m + j, int64, ascending), values and the
    duals (u, v) as CUDA tensors, with the distance, all without a host round trip."""
    if not torch.is_tensor(cost) or not cost.is_cuda:
        raise ValueError("solve_leaf_resident takes a CUDA cost tensor")
    keys, values, dual, distance, res, elapsed, _, _ = _solve_dense(cost, source_mass, target_mass, tolerance,
                                                                    cost.device)
    return SimpleNamespace(keys=keys, values=values, dual=dual, distance=distance, time=elapsed,
                           iterations=int(res.iterations), termination_reason=res.termination_reason)


def solve_leaf_from_cost(*, cost, source_mass, target_mass, tolerance: float = 1e-9, device="cuda",
                         **_unused) -> Dict[str, Any]:
    """Dense OT between source_mass (n) and target_mass (m) with cost (n x m)."""
    keys, values, dual, distance, res, solve_time, n, m = _solve_dense(cost, source_mass, target_mass, tolerance,
                                                                       device)
    r, cc = keys // m, keys % m
    warm = SimpleNamespace(rows=r.to(torch.int32).cpu().numpy(), cols=cc.to(torch.int32).cpu().numpy(),
                           x_prev=values.cpu().numpy(), dual_uv=dual.cpu().numpy(), n_source=int(n), n_target=int(m))
    return {
        "distance": distance,
        "time": solve_time,
        "lp_solve_time_total": solve_time,
        "warm_start_state": warm,
        "termination_reason": res.termination_reason,
        "iterations": int(res.iterations),
        "leaf_stage_profile": {"pdhg_solve_time": solve_time, "cost_build_backend": "precomputed"},
        "level_summaries": [{"level": 0, "n_source": n, "n_target": m, "iters": int(res.iterations),
                             "time": solve_time, "objective": distance, "lp_time": solve_time,
                             "pricing_time": 0.0, "support_final": int(keys.numel())}],
    }
