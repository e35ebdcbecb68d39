"""Active-support maintenance on the GPU.

``filter_new_candidate_pairs`` mirrors ``ActiveSupport.filter_new_candidate_pairs``
(src/hello_ot/restricted_ot/active_support.py:483-506): the candidate pairs of a
scan that are not in the support yet, unique and in ascending key order
(row * n_target + col), as (new_rows int32, new_cols int32, found, new_count).
The work runs in libhello_b200 (radix sorts, a binary-search flag pass and a
compaction); there is no CPU path.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import Workspace, check, lib, ptr, stream_handle


def filter_new_candidate_pairs(active_keys, n_source: int, n_target: int, rows, cols, *, active_sorted: bool = False,
                               device=None):
    """New (row, col) candidate pairs of a support with keys ``active_keys``."""
    dev = torch.device(device) if device is not None else (
        active_keys.device if torch.is_tensor(active_keys) and active_keys.is_cuda else torch.device("cuda"))
    if dev.type != "cuda":
        raise ValueError("filter_new_candidate_pairs runs on CUDA devices only")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    keys = torch.as_tensor(active_keys, dtype=torch.int64, device=dev).contiguous().view(-1)
    r = torch.as_tensor(rows, dtype=torch.int32, device=dev).contiguous().view(-1)
    c = torch.as_tensor(cols, dtype=torch.int32, device=dev).contiguous().view(-1)
    if r.numel() != c.numel():
        raise ValueError("rows and cols must have the same length")
    found = int(r.numel())
    L = lib()
    new_rows = torch.empty(max(found, 1), dtype=torch.int32, device=dev)
    new_cols = torch.empty(max(found, 1), dtype=torch.int32, device=dev)
    count = ctypes.c_int64(0)
    ws = Workspace.get(dev, L.hb_filter_new_pairs_workspace(keys.numel(), found))
    with torch.cuda.device(dev):
        rc = L.hb_filter_new_pairs(ptr(keys) if keys.numel() else None, keys.numel(), int(bool(active_sorted)),
                                   ptr(r), ptr(c), found, int(n_source), int(n_target), ptr(new_rows), ptr(new_cols),
                                   ctypes.byref(count), ptr(ws), ws.numel(), stream_handle(dev))
    check(rc)
    n = int(count.value)
    return new_rows[:n], new_cols[:n], found, n


def support_filter(support, rows, cols):
    """The method form: ``support`` has ``keys``, ``n_source`` and ``n_target`` (an
    ActiveSupport); returns what ActiveSupport.filter_new_candidate_pairs returns."""
    return filter_new_candidate_pairs(support.keys, support.n_source, support.n_target, rows, cols)


POSITIVE_SUPPORT_TOLERANCE = 1e-15  # src/hello_ot/refinement/support_budget.py:7


def select_prune_positions(rows, cols, costs, x_prev, creation_iteration, duals, n_source: int, n_target: int,
                           num_to_remove: int, current_inner_iter: int):
    """Positions DualGapCleaning removes in protect-new mode
    (budgeted_pruning.py:119-175 with _select_zero_flow_removals :27-57): removable =
    old (creation != current_inner_iter, != -1) and zero flow (|x| <= 1e-15); the
    num_to_remove with the largest reduced cost c - u_row - v_col, stable.  Raises
    RuntimeError like the reference when too few edges are removable.  Returns a
    numpy int32 array."""
    import numpy as np
    num = int(num_to_remove)
    if num <= 0:
        return np.empty(0, dtype=np.int32)
    dev = costs.device if torch.is_tensor(costs) and costs.is_cuda else torch.device("cuda", torch.cuda.current_device())
    t = lambda v, dt: torch.as_tensor(v, dtype=dt, device=dev).contiguous().view(-1)  # noqa: E731
    r, c = t(rows, torch.int32), t(cols, torch.int32)
    w, x, cr = t(costs, torch.float64), t(x_prev, torch.float64), t(creation_iteration, torch.int32)
    u = t(duals, torch.float64)
    e = int(r.numel())
    if not (int(c.numel()) == int(w.numel()) == int(x.numel()) == int(cr.numel()) == e):
        raise ValueError("support arrays must have equal lengths")
    if int(u.numel()) < int(n_source) + int(n_target):
        raise ValueError("duals must hold n_source + n_target values")
    L = lib()
    out = torch.empty(max(num, 1), dtype=torch.int32, device=dev)
    count = ctypes.c_int64(0)
    ws = Workspace.get(dev, L.hb_prune_select_workspace(e))
    with torch.cuda.device(dev):
        rc = L.hb_prune_select(ptr(r), ptr(c), ptr(w), ptr(x), ptr(cr), e, ptr(u), int(n_source), int(n_target),
                               int(current_inner_iter), num, ptr(out), ctypes.byref(count), ptr(ws), ws.numel(),
                               stream_handle(dev))
    check(rc)
    if int(count.value) < num:
        raise RuntimeError("HELLO budgeted pruning invariant violated: "
                           f"required_removals={num}, removable_old_zero={int(count.value)}, support_size={e}")
    return out[:num].cpu().numpy()
