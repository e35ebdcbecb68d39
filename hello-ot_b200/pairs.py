"""Active-support pair costs (SDDMM) with the reference's interfaces.

``cost_pairs_lowrank`` mirrors ``hello_ot.costs.pairs._cost_pairs_lowrank_batched``
(src/hello_ot/costs/pairs.py:221-440): c_e = a_r + b_c - s<F_r, G_c>.
``pair_costs_metric`` mirrors the fp64 branch of
``hello_ot.costs.metric.pair_costs_metric`` (src/hello_ot/costs/metric.py:85-160),
which calls ``fused_gcost_pairs`` (norm_cost_scan_kernel.cu:249-275).
Both evaluate in fp64 from the fp32 features on the GPU and keep the input
edge order; results come back as numpy unless the indices were torch tensors.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import Workspace, check, lib, ptr, stream_handle

KIND = {"l1": 0, "linf": 1, "l2": 2, "lowrank": 3, "l2^2": 3}


def _dev(a, device, dtype):
    if torch.is_tensor(a):
        return a.detach().to(device=device, dtype=dtype).contiguous()
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype).to(device).contiguous()


def pair_costs(kind: int, x, y, rows, cols, a=None, b=None, dot_scale: float = 1.0, perturbation=None):
    """Device entry: x, y CUDA fp32; rows, cols CUDA int64; returns CUDA fp64.
    perturbation (norm kinds): the (Perturbation, tensors) pair of perturb.make_perturbation."""
    L = lib()
    device = x.device
    x, y = x.contiguous(), y.contiguous()
    rows = rows.to(device=device, dtype=torch.int64).contiguous().view(-1)
    cols = cols.to(device=device, dtype=torch.int64).contiguous().view(-1)
    if rows.numel() != cols.numel():
        raise ValueError("rows and cols must have the same length.")
    out = torch.empty(rows.numel(), dtype=torch.float64, device=device)
    if rows.numel() == 0:
        return out
    if kind == 3:
        a = a.to(device=device, dtype=torch.float64).contiguous()
        b = b.to(device=device, dtype=torch.float64).contiguous()
    ws = Workspace.get(device, L.hb_pair_costs_workspace())
    with torch.cuda.device(device):
        rc = L.hb_pair_costs_ex(int(kind), ptr(x), ptr(y), x.shape[0], y.shape[0], x.shape[1], ptr(a), ptr(b),
                                float(dot_scale), ptr(rows), ptr(cols), rows.numel(), ptr(out), ptr(ws), ws.numel(),
                                stream_handle(device), ctypes.byref(perturbation[0]) if perturbation else None)
    check(rc)
    return out


def cost_pairs_lowrank(level_cache, rows, cols, *, device=None, **_legacy):
    """c_e = a[r] + b[c] - dot_scale <F[r], G[c]> for every edge (fp64)."""
    F, G, a, b = level_cache["F"], level_cache["G"], level_cache["a"], level_cache["b"]
    dot_scale = float(level_cache.get("dot_scale", 1.0))
    if dot_scale not in (1.0, 2.0):
        raise ValueError("dot_scale must be exactly 1 or 2")
    as_torch = torch.is_tensor(rows)
    if device is None:
        device = rows.device if as_torch and rows.is_cuda else torch.device("cuda", torch.cuda.current_device())
    out = pair_costs(3, _dev(F, device, torch.float32), _dev(G, device, torch.float32),
                     _dev(rows, device, torch.int64), _dev(cols, device, torch.int64),
                     _dev(a, device, torch.float64), _dev(b, device, torch.float64), dot_scale)
    return out if as_torch else out.cpu().numpy()


def pair_costs_metric(*, source_points, target_points, rows, cols, cost_type, perturbation=None,
                      compute_precision="fp64", cached_points=None, device=None, **_legacy):
    """fp64 ℓ1/ℓ∞/ℓ2 cost of every edge (h/costs/metric.py:85), with the reference's
    full-cost perturbation dict (mode "full_cost_perturb": sigma, seed, noise "rank2" /
    "index_hash", source_global_index, target_global_index) added in fp64."""
    as_torch = torch.is_tensor(rows)
    if device is None:
        device = rows.device if as_torch and rows.is_cuda else torch.device("cuda", torch.cuda.current_device())
    if cached_points is not None:
        src, tgt = cached_points
    else:
        src, tgt = _dev(source_points, device, torch.float32), _dev(target_points, device, torch.float32)
    pert = None
    if (isinstance(perturbation, dict) and str(perturbation.get("mode", "")).strip().lower() == "full_cost_perturb"
            and float(perturbation.get("sigma", 0.0)) != 0.0):
        from .perturb import make_perturbation
        si, ti = perturbation.get("source_global_index"), perturbation.get("target_global_index")
        if si is None or ti is None:
            raise ValueError("full metric perturbation requires source_global_index and target_global_index.")
        pert = make_perturbation(src, tgt, _dev(si, device, torch.int64), _dev(ti, device, torch.int64),
                                 float(perturbation["sigma"]), int(perturbation.get("seed", 0)),
                                 str(perturbation.get("noise", "rank2")).strip().lower(), True, None)
    out = pair_costs(KIND[str(cost_type)], src, tgt, _dev(rows, device, torch.int64), _dev(cols, device, torch.int64),
                     perturbation=pert)
    return out if as_torch else out.cpu().numpy()
