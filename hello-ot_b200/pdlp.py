"""Restricted-OT PDLP engine with the reference's RestrictedOTPDLP interface.

``NativeRestrictedOTPDLP.solve_restricted`` mirrors
``RestrictedOTPDLP.solve_restricted`` (src/hello_ot/_internal/lp/restricted_ot_pdlp.py:39-100):
same configuration, termination contract, one retry with scalar rescaling on
NUMERICAL_DIVERGENCE, and a ``SolverResult`` with the fields the refinement
loop reads (src/hello_ot/_internal/lp/wrapper.py).  Each solve runs the fused
matrix-free Halpern-PDHG of libhello_b200 (hb_restricted_ot_solve).
"""
from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass, field
from typing import Any, Dict, Optional

import numpy as np
import torch

from ._lib import PdlpControls, PdlpInfo, PdlpTraceRow, Workspace, check, lib, ptr, stream_handle

REASONS = {1: "OPTIMAL", 2: "ITERATION_LIMIT", 3: "NUMERICAL_DIVERGENCE", 4: "TIME_LIMIT"}
SUMMATION = {"ordered": 0, "atomic": 1, "tree": 2}  # hb_pdlp_controls.atomic_sums (HB_PDLP_SUMS_*)
TERMINATION_NORMS = {"l2": 0, "linf": 1}  # hb_pdlp_controls.termination_norm (HB_PDLP_NORM_*)


@dataclass
class SolverResult:
    """Restricted-LP result (fields of hello_ot._internal.lp.wrapper.SolverResult)."""

    success: bool
    x: Any = None
    y: Any = None
    obj_val: float = 0.0
    dual_obj_val: float = None
    duration: float = 0.0
    iterations: int = 0
    peak_mem: float = 0.0
    termination_reason: str = None
    primal_feas: float = None
    dual_feas: float = None
    gap: float = None
    solver_diag: Dict = field(default_factory=dict)


def _vec(v, dtype, device):
    if torch.is_tensor(v):
        return v.detach().to(device=device, dtype=dtype).contiguous().view(-1)
    return torch.as_tensor(np.ascontiguousarray(v), dtype=dtype).to(device).contiguous().view(-1)


class NativeRestrictedOTPDLP:
    """GPU Halpern-PDHG for balanced restricted OT on the active support."""

    def __init__(self, *, device="cuda", evaluation_frequency: int = 200, time_limit_seconds: float = 3600.0,
                 iteration_limit: int = np.iinfo(np.int32).max, record_state_trace: bool = False,
                 initial_primal_weight: float = 0.0, deterministic: bool = True, summation: str = None,
                 termination_norm: str = "l2"):
        """summation (node sums of the primal): "ordered" (the default) adds each node's
        edges in the reference's order, bit-identical to it; "atomic" (also chosen by
        deterministic=False) accumulates with atomics in the edge pass, about 1.2x faster
        per iteration on large random supports, but the order (so the last bits of the
        iterates) varies from run to run; "tree" is "ordered" except on a side whose mean
        degree is >= 64 (a dense support), where a fixed lane tree adds each node's edges:
        reproducible run to run, not the reference's order, several times faster there.
        termination_norm: "l2" (solver.cpp's test) or "linf" (the native engine's
        termination_norm = "linf", cupdlpx/utils.cu:1027-1041: primal and dual residuals in
        the max norm relative to 1 + ||b||_inf and 1 + ||c||_inf; restarts and the primal
        weight stay on the L2 residuals)."""
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("NativeRestrictedOTPDLP runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.evaluation_frequency = int(evaluation_frequency)
        self.time_limit_seconds = float(time_limit_seconds)
        self.iteration_limit = int(iteration_limit)
        self.record_state_trace = bool(record_state_trace)
        self.initial_primal_weight = float(initial_primal_weight)
        if summation is None:
            summation = "ordered" if deterministic else "atomic"
        if summation not in SUMMATION:
            raise ValueError(f"summation must be one of {sorted(SUMMATION)}")
        self.summation = summation
        self.deterministic = summation != "atomic"
        if termination_norm not in TERMINATION_NORMS:
            raise ValueError("termination_norm must be one of: l2, linf")
        self.termination_norm = termination_norm
        if self.evaluation_frequency < 1:
            raise ValueError("evaluation_frequency must be >= 1")
        if self.time_limit_seconds <= 0.0 or self.iteration_limit < 1:
            raise ValueError("time_limit_seconds and iteration_limit must be positive")
        self.last_diagnostics: Dict = {}

    def solve_restricted(self, *, rows, cols, costs, source_mass, target_mass, warm_start_primal=None,
                         warm_start_dual=None, tolerance=1e-6, verbose: bool = False) -> SolverResult:
        if isinstance(tolerance, dict):
            tob = float(tolerance.get("objective", 1e-6))
            tp, td = float(tolerance.get("primal", tob)), float(tolerance.get("dual", tob))
        else:
            tob = tp = td = float(tolerance)
        args = dict(rows=rows, cols=cols, costs=costs, source_mass=source_mass, target_mass=target_mass,
                    warm_start_primal=warm_start_primal, warm_start_dual=warm_start_dual, objective_tolerance=tob,
                    primal_tolerance=tp, dual_tolerance=td, verbose=verbose)
        first = self._solve_once(**args, scalar_rescaling=False)
        if first.termination_reason != "NUMERICAL_DIVERGENCE":
            return first
        retry = self._solve_once(**args, scalar_rescaling=True)
        retry.solver_diag = dict(retry.solver_diag or {})
        retry.solver_diag.update({"numerical_rescaling_retry": True,
                                  "numerical_rescaling_first_termination_reason": first.termination_reason,
                                  "numerical_rescaling_first_iterations": int(first.iterations)})
        return retry

    def _solve_once(self, *, rows, cols, costs, source_mass, target_mass, warm_start_primal, warm_start_dual,
                    objective_tolerance, primal_tolerance, dual_tolerance, scalar_rescaling, verbose):
        started = time.perf_counter()
        dev = self.device
        L = lib()
        rows_t = _vec(rows, torch.int64, dev)
        cols_t = _vec(cols, torch.int64, dev)
        costs_t = _vec(costs, torch.float64, dev)
        a = _vec(source_mass, torch.float64, dev)
        b = _vec(target_mass, torch.float64, dev)
        n, m, e = a.numel(), b.numel(), costs_t.numel()
        if rows_t.numel() != e or cols_t.numel() != e:
            raise ValueError("rows, cols, and costs must have equal lengths")
        if e == 0:
            raise ValueError("restricted OT active support must not be empty")
        if n == 0 or m == 0:
            raise ValueError("both marginals must be nonempty")
        masses = torch.cat((a, b))
        mass_scale = max(1.0, float(masses.abs().max().item()))
        if abs(float(a.sum().item()) - float(b.sum().item())) > 1e-12 * mass_scale:
            raise ValueError("balanced restricted OT requires equal source and target total mass")
        x0 = None if warm_start_primal is None else _vec(warm_start_primal, torch.float64, dev)
        y0 = None if warm_start_dual is None else _vec(warm_start_dual, torch.float64, dev)
        if (x0 is not None and x0.numel() != e) or (y0 is not None and y0.numel() != n + m):
            raise ValueError("warm-start dimensions do not match the restricted OT problem")
        x_out = torch.empty(e, dtype=torch.float64, device=dev)
        y_out = torch.empty(n + m, dtype=torch.float64, device=dev)
        ctl = PdlpControls(self.evaluation_frequency, int(bool(scalar_rescaling)), self.iteration_limit,
                           self.time_limit_seconds, objective_tolerance, primal_tolerance, dual_tolerance,
                           self.initial_primal_weight, SUMMATION[self.summation],
                           TERMINATION_NORMS[self.termination_norm])
        info = PdlpInfo()
        cap = 4096 if self.record_state_trace else 0
        trace = (PdlpTraceRow * max(cap, 1))()
        tlen = ctypes.c_int32(0)
        ws = Workspace.get(dev, L.hb_restricted_ot_workspace(n, m, e))
        with torch.cuda.device(dev):
            rc = L.hb_restricted_ot_solve(ptr(rows_t), ptr(cols_t), ptr(costs_t), e, ptr(masses), n, m, ptr(x0),
                                          ptr(y0), ctypes.byref(ctl), ptr(x_out), ptr(y_out), ctypes.byref(info),
                                          trace if cap else None, cap, ctypes.byref(tlen), ptr(ws), ws.numel(),
                                          stream_handle(dev))
        check(rc)
        reason = REASONS.get(info.termination, "UNSPECIFIED")
        duration = time.perf_counter() - started
        diag = {
            "backend": "hello_b200_pdhg", "device": str(dev), "dtype": "float64",
            "scaling_mode": "degree_sqrt" + ("_with_scalar_retry" if scalar_rescaling else ""),
            "step_size": 0.998, "termination_norm": self.termination_norm,
            "termination_abs_primal_res": info.abs_primal_residual,
            "termination_rel_primal_res": info.rel_primal_residual,
            "termination_abs_dual_res": info.abs_dual_residual,
            "termination_rel_dual_res": info.rel_dual_residual,
            "termination_objective_vector_norm": info.cost_norm,
            "termination_constraint_bound_norm": info.mass_norm,
            "algorithm_abs_primal_res_l2": info.l2_abs_primal_residual,
            "algorithm_rel_primal_res_l2": info.l2_rel_primal_residual,
            "algorithm_abs_dual_res_l2": info.l2_abs_dual_residual,
            "algorithm_rel_dual_res_l2": info.l2_rel_dual_residual,
            "relative_primal_dual_gap": info.rel_gap, "primal_weight": info.primal_weight,
            "restart_count": int(info.restarts), "runtime_sec": duration,
            "setup_time_sec": info.setup_seconds, "iteration_time_sec": info.iteration_seconds,
            "termination_reason": reason, "numerical_rescaling_retry": bool(scalar_rescaling),
        }
        if self.record_state_trace:
            diag["state_trace"] = [dict(iteration=int(r.iteration), primal_objective=r.primal_objective,
                                        dual_objective=r.dual_objective, relative_primal_residual=r.rel_primal,
                                        relative_dual_residual=r.rel_dual, relative_gap=r.rel_gap,
                                        primal_weight=r.primal_weight) for r in trace[:tlen.value]]
        self.last_diagnostics = diag
        if verbose:
            print(f"[NativeRestrictedOTPDLP] termination={reason} iterations={info.iterations} "
                  f"rel_primal={info.rel_primal_residual:.3e} rel_dual={info.rel_dual_residual:.3e} "
                  f"gap={info.rel_gap:.3e}")
        return SolverResult(success=reason == "OPTIMAL", x=x_out, y=y_out, obj_val=info.primal_objective,
                            dual_obj_val=info.dual_objective, duration=duration, iterations=int(info.iterations),
                            termination_reason=reason, primal_feas=info.rel_primal_residual,
                            dual_feas=info.rel_dual_residual, gap=info.rel_gap, solver_diag=diag)
