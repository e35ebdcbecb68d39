"""Pricing-scan entry points with the reference's interface.

``ScanExtension`` mirrors ``hello_ot.kernels.generic_scan.ScanExtension``
(src/hello_ot/kernels/generic_scan.py:468-597) for the entry points of the
pricing hot path, and ``raw_lowrank_bidir_feasibility_pricing_scan`` mirrors
``hello_ot.kernels.bilinear_topk.raw_lowrank_bidir_feasibility_pricing_scan``
(src/hello_ot/kernels/bilinear_topk.py:207-497).  Both run on the
libhello_b200 CUDA kernels only: tensor-core ℓ2² scan, CUDA-core norm scans.

Differences from the reference, all deliberate:
  * tile arguments (query_tile, db_tile, col_reduce_tile, col_kernel) are
    validated like the reference but the fused kernels plan their own tiles;
  * both clouds stay resident in HBM (a B200 holds a 1.28M x 8192 cloud pair),
    so the scan is one call with no host streaming;
  * the norm scans take the index-hash / rank-2 cost perturbation (sigma > 0) in
    the kernels; the ℓ2² perturbation arrives as two appended feature columns,
    as the reference builds it.
"""
from __future__ import annotations

import ctypes
import math
import time
from collections import Counter
from dataclasses import dataclass
from typing import Any, Dict

import numpy as np
import torch

from ._lib import Workspace, check, lib, ptr, stream_handle
from .perturb import make_perturbation

BUCKETS = (1, 2, 4, 8, 16, 32)
PRECISION = {"fp32": 3, "3xtf32": 3, "f16x3": 3, "tf32": 1}  # "3xtf32": the former name of 3
_ROUTES = Counter()


def scan_routes(*, reset: bool = False) -> dict:
    """Entry-point call counts (generic_scan.py:21-28)."""
    out = dict(_ROUTES)
    if reset:
        _ROUTES.clear()
    return out


def topk_bucket(k: int) -> int:
    """Smallest instantiated bucket >= k (src/hello_ot/kernels/scan_contract.py:80-91)."""
    k = int(k)
    if k < 1:
        raise ValueError("topk must be >= 1")
    for b in BUCKETS:
        if k <= b:
            return b
    raise ValueError(f"custom inner_product scan supports topk <= 32; received topk={k}.")


def _check(x, y, k, *vectors):
    """Same contract as generic_scan._check (generic_scan.py:42-56), fp32 features."""
    if k not in BUCKETS:
        raise ValueError("generic scan requires a power-of-two bucket in [1,32]")
    if (not x.is_cuda or not y.is_cuda or x.device != y.device or x.dtype != torch.float32 or y.dtype != x.dtype
            or x.ndim != 2 or y.ndim != 2 or x.shape[1] != y.shape[1] or min(*x.shape, *y.shape) < 1
            or max(*x.shape, *y.shape) >= 2 ** 31):
        raise ValueError("generic scan requires nonempty matching CUDA FP32 feature matrices with int32 dimensions")
    for v, count in vectors:
        if v.device != x.device or v.dtype != torch.float64 or v.numel() != count:
            raise ValueError("generic scan requires matching CUDA FP64 bias vectors")


def _c(t):
    return t.contiguous()


L2SQ_PASS_FLAGS = {None: 0, 2: 0x10, 1: 0x20}
L2SQ_CTA_FLAGS = {None: 0, 2: 0x100, 1: 0x200}  # HB_L2SQ_CTA_PAIRS, HB_L2SQ_SINGLE_CTA


L2SQ_EXACT = 0x400  # HB_L2SQ_EXACT


def l2sq_scan(x, y, x_cost, y_cost, x_bias, y_bias, k, *, dot_scale=2.0, compute_stats=True, precision="fp32",
              min_groups=0, passes=None, ctas=None, exact=False):
    """Bidirectional ℓ2² scan on the tensor cores.

    passes: 1 (k <= 8 only), 2, or None to let the library choose; both give the
    same lists bit for bit.  ctas (one-pass kernel): 2 runs it as CTA pairs sharing
    each column tile, 1 as single CTAs, None the library's choice.  exact: the fp64
    re-check (HB_L2SQ_EXACT): lists are the exact fp64 top-k, values exact fp64 scores.
    Returns (row_vals q x k fp64, row_idx q x k int32, col_vals n x k, col_idx n x k,
    stats [sum s+^2, sum c^2, max s+, max |c|, count] fp64 on the device)."""
    x, y = _c(x), _c(y)
    x_cost, y_cost, x_bias, y_bias = map(_c, (x_cost, y_cost, x_bias, y_bias))
    q, d = x.shape
    n = y.shape[0]
    prec = PRECISION[precision] if isinstance(precision, str) else int(precision)
    prec |= L2SQ_PASS_FLAGS[passes] | L2SQ_CTA_FLAGS[ctas] | (L2SQ_EXACT if exact and int(k) > 0 else 0)
    L = lib()
    dev = x.device
    kk = int(k)
    rv = torch.empty((q, max(kk, 1)), dtype=torch.float64, device=dev)
    ri = torch.empty((q, max(kk, 1)), dtype=torch.int32, device=dev)
    cv = torch.empty((n, max(kk, 1)), dtype=torch.float64, device=dev)
    ci = torch.empty((n, max(kk, 1)), dtype=torch.int32, device=dev)
    stats = torch.zeros(5, dtype=torch.float64, device=dev)
    nbytes = L.hb_l2sq_scan_workspace(q, n, d, kk, prec, int(min_groups))
    ws = Workspace.get(dev, nbytes)
    with torch.cuda.device(dev):
        rc = L.hb_l2sq_scan(ptr(x), ptr(y), q, n, d, ptr(x_cost), ptr(y_cost), ptr(x_bias), ptr(y_bias), kk,
                            float(dot_scale), int(bool(compute_stats)), prec, int(min_groups), ptr(rv), ptr(ri),
                            ptr(cv), ptr(ci), ptr(stats), ptr(ws), ws.numel(), stream_handle(dev))
    check(rc)
    return rv[:, :kk], ri[:, :kk], cv[:, :kk], ci[:, :kk], stats


def l2sq_last_rescans() -> tuple:
    """(row lists, column lists) the calling thread's last exact l2sq scan recomputed in
    fp64 against every column because a near tie fell within the error bound."""
    out = (ctypes.c_int64 * 2)()
    check(lib().hb_l2sq_last_rescans(out))
    return int(out[0]), int(out[1])


NORM_KIND = {"l1": 0, "linf": 1, "l2": 2, 0: 0, 1: 1, 2: 2}


NORM_TWO_PASS = 0x10


def norm_scan(x, y, f, g, k, cost_type, *, compute_stats=True, passes=None, perturbation=None):
    """Bidirectional ℓ1/ℓ∞/ℓ2 scan on the CUDA cores (outputs as l2sq_scan).
    k <= 8 makes one pass over the pairs unless passes=2 (same lists bit for bit).
    perturbation: the (Perturbation, tensors) pair of perturb.make_perturbation, or None."""
    x, y, f, g = map(_c, (x, y, f, g))
    q, d = x.shape
    n = y.shape[0]
    kind = NORM_KIND[cost_type] | (NORM_TWO_PASS if passes == 2 else 0)
    L = lib()
    dev = x.device
    kk = int(k)
    rv = torch.empty((q, max(kk, 1)), dtype=torch.float64, device=dev)
    ri = torch.empty((q, max(kk, 1)), dtype=torch.int32, device=dev)
    cv = torch.empty((n, max(kk, 1)), dtype=torch.float64, device=dev)
    ci = torch.empty((n, max(kk, 1)), dtype=torch.int32, device=dev)
    stats = torch.zeros(5, dtype=torch.float64, device=dev)
    ws = Workspace.get(dev, L.hb_norm_scan_workspace(q, n, kk))
    with torch.cuda.device(dev):
        rc = L.hb_norm_scan_ex(ptr(x), ptr(y), q, n, d, ptr(f), ptr(g), kind, kk, int(bool(compute_stats)), ptr(rv),
                               ptr(ri), ptr(cv), ptr(ci), ptr(stats), ptr(ws), ws.numel(), stream_handle(dev),
                               ctypes.byref(perturbation[0]) if perturbation else None)
    check(rc)
    return rv[:, :kk], ri[:, :kk], cv[:, :kk], ci[:, :kk], stats


def l2sq_topk(x, y, x_bias, y_bias, k, *, dot_scale=2.0, precision="fp32"):
    """One-sided ℓ2² top-k on the tensor cores (the initial dual-assignment scan):
    for every x row the best k of (fp32(s <x, y_j>) + x_bias) + y_bias_j, descending,
    lower index on ties.  Returns (values q x k fp64, indices q x k int32)."""
    x, y, x_bias, y_bias = map(_c, (x, y, x_bias, y_bias))
    q, d = x.shape
    n = y.shape[0]
    prec = PRECISION[precision] if isinstance(precision, str) else int(precision)
    L = lib()
    dev = x.device
    vals = torch.empty((q, int(k)), dtype=torch.float64, device=dev)
    idx = torch.empty((q, int(k)), dtype=torch.int32, device=dev)
    ws = Workspace.get(dev, L.hb_l2sq_topk_workspace(q, n, d, int(k), prec))
    with torch.cuda.device(dev):
        rc = L.hb_l2sq_topk(ptr(x), ptr(y), q, n, d, ptr(x_bias), ptr(y_bias), int(k), float(dot_scale), prec,
                            ptr(vals), ptr(idx), ptr(ws), ws.numel(), stream_handle(dev))
    check(rc)
    return vals, idx


def norm_topk(x, y, g, k, cost_type, *, compute_stats=False, perturbation=None):
    """One-sided ℓ1/ℓ∞/ℓ2 top-k on the CUDA cores: for every x row the best k of
    g_j - c_ij (fp64 score of the fp32 distance), descending, lower index on ties.
    Returns (scores q x k fp64, indices q x k int32, stats [sum c^2, max |c|] or None)."""
    x, y, g = map(_c, (x, y, g))
    q, d = x.shape
    n = y.shape[0]
    L = lib()
    dev = x.device
    vals = torch.empty((q, int(k)), dtype=torch.float64, device=dev)
    idx = torch.empty((q, int(k)), dtype=torch.int32, device=dev)
    stats = torch.zeros(2, dtype=torch.float64, device=dev) if compute_stats else None
    ws = Workspace.get(dev, L.hb_norm_topk_workspace(q, n, int(k)))
    with torch.cuda.device(dev):
        rc = L.hb_norm_topk_ex(ptr(x), ptr(y), q, n, d, ptr(g), NORM_KIND[cost_type], int(k),
                               int(bool(compute_stats)), ptr(vals), ptr(idx), ptr(stats), ptr(ws), ws.numel(),
                               stream_handle(dev), ctypes.byref(perturbation[0]) if perturbation else None)
    check(rc)
    return vals, idx, stats


class ScanExtension:
    """Scan entry points with the reference ABI (generic_scan.py:468-597)."""

    supports_assignment_statistics = False
    supports_cost_perturbation = True
    supports_fp64_accumulation = True
    index_hash_arithmetic = None

    def __init__(self, *, precision: str = "fp32", exact: bool = True):
        """precision: "fp32" (3-term fp16 split) or "tf32"; exact: the fp64 re-check of
        the ℓ2² lists (HB_L2SQ_EXACT), so the lists are the exact fp64 top-k."""
        self.routes = Counter()
        self.last_backend = "hello_b200"
        self.precision = precision
        self.exact = bool(exact)

    def _record(self, name):
        key = name + ":hello_b200"
        self.routes[key] += 1
        _ROUTES[key] += 1

    def fused_bidir_topk_stats_raw(self, query_feat, db_feat, query_cost, db_cost, query_bias, db_bias, query_tile,
                                   db_tile, col_reduce_tile, k, compute_stats, collect_linf_stats, collect_timing,
                                   col_kernel, dot_scale):
        """[q_vals q x k, q_idx int32, r_vals n x k, r_idx int32, stats(4) = (num, den, count,
        linf), timing(4) cpu zeros] -- generic_scan.py:577-597."""
        x, y, nx, ny, qb, dbb = query_feat, db_feat, query_cost, db_cost, query_bias, db_bias
        if x.dtype != y.dtype:
            raise RuntimeError("query/db feature dtypes must match")
        _check(x, y, k, (nx, len(x)), (ny, len(y)), (qb, len(x)), (dbb, len(y)))
        if (query_tile <= 0 or db_tile <= 0 or not 0 < col_reduce_tile <= 256 or dot_scale not in (1., 2.)
                or col_kernel not in (0, 1, 2) or (col_kernel == 1 and k != 4) or (col_kernel == 2 and k != 2)):
            raise ValueError("invalid raw pricing tile, scale or column mode")
        self._record("raw_pricing")
        rv, ri, cv, ci, s = l2sq_scan(x, y, nx, ny, qb, dbb, k, dot_scale=dot_scale,
                                      compute_stats=bool(compute_stats), precision=self.precision,
                                      exact=self.exact)
        stats = torch.stack((s[0], s[1], s[4], s[3] if collect_linf_stats else s[3].new_zeros(())))
        if not compute_stats:
            stats.zero_()
        return [rv, ri, cv, ci, stats, torch.zeros(4, dtype=torch.float64, device="cpu")]

    def initialization_directional_topk_raw(self, query_feat, db_feat, query_bias, db_bias, query_tile, db_tile, k,
                                            dot_scale):
        """[values q x k fp64 descending, indices q x k int32] of (dot + query_bias) + db_bias
        (generic_scan.py:560-575, cost.cu:248-348)."""
        x, y, qb, dbb = query_feat, db_feat, query_bias, db_bias
        if x.dtype != y.dtype:
            raise RuntimeError("query/db feature dtypes must match")
        _check(x, y, k, (qb, len(x)), (dbb, len(y)))
        if query_tile <= 0 or db_tile <= 0 or dot_scale not in (1., 2.):
            raise ValueError("invalid raw directional tile or scale")
        self._record("raw_initial")
        values, ids = l2sq_topk(x, y, qb, dbb, k, dot_scale=dot_scale, precision=self.precision)
        return [values, ids]

    def fused_directional_topk_raw(self, query_feat, db_feat, query_bias, db_bias, query_tile, db_tile, k, dot_scale):
        """Compatibility name of initialization_directional_topk_raw (generic_scan.py:512-518)."""
        self._record("raw_directional")
        return self.initialization_directional_topk_raw(query_feat, db_feat, query_bias, db_bias, query_tile, db_tile,
                                                        k, dot_scale)

    def fused_gcost_topk(self, query, db, dual_db, k, cost_type, query_global_index=None, database_global_index=None,
                         sigma=0., seed=0, perturb_mode=1, row_is_source=True, index_hash_coeffs=None,
                         compute_precision=0, collect_statistics=False):
        """[values q x k ascending c - g, indices int64 (, stats [sum c^2, max |c|])]
        (generic_scan.py:520-531 -> directional(minimum=True), initial.cu:34-107)."""
        if compute_precision not in (0,):
            raise NotImplementedError("hello_ot_b200 norm scans compute fp32 distances (compute_precision=0)")
        _check(query, db, k, (dual_db, len(db)))
        pert = make_perturbation(query, db, query_global_index, database_global_index, sigma, seed, perturb_mode,
                                 row_is_source, index_hash_coeffs)
        self._record("norm_initial")
        scores, ids, stats = norm_topk(query, db, dual_db, k, cost_type, compute_stats=bool(collect_statistics),
                                       perturbation=pert)
        out = [scores.neg_(), ids.long()]
        if collect_statistics:
            out.append(stats)
        return out

    def raw_lowrank_stats_only(self, x, y, nx, ny, f, g, query_tile, db_tile, dot_scale):
        """Certificate of the bilinear scan without candidates (generic_scan.py:502-510):
        (num, den, max s+, max |c|, count) as 0-d tensors; f, g are the duals."""
        if query_tile <= 0 or db_tile <= 0:
            raise ValueError("tile sizes must be positive")
        _check(x, y, 1, (nx, len(x)), (ny, len(y)), (f, len(x)), (g, len(y)))
        self._record("raw_certificate")
        s = l2sq_scan(x, y, nx, ny, f - nx, g - ny, 0, dot_scale=dot_scale, precision=self.precision)[4]
        return s[0], s[1], s[2], s[3], s[4].long()

    def fused_gcost_bidir_certificate(self, query, db, query_dual, db_dual, k, cost_type, query_global_index=None,
                                      database_global_index=None, sigma=0., seed=0, perturb_mode=1,
                                      row_is_source=True, index_hash_coeffs=None, compute_precision=0,
                                      rows_per_block_hint=8):
        """[rv, ri int64, cv, ci int64, num, den, max s+, max |c|, count int64] (generic_scan.py:533-543)."""
        if compute_precision not in (0,):
            raise NotImplementedError("hello_ot_b200 norm scans compute fp32 distances (compute_precision=0)")
        _check(query, db, k, (query_dual, len(query)), (db_dual, len(db)))
        pert = make_perturbation(query, db, query_global_index, database_global_index, sigma, seed, perturb_mode,
                                 row_is_source, index_hash_coeffs)
        self._record("norm_pricing")
        rv, ri, cv, ci, s = norm_scan(query, db, query_dual, db_dual, k, cost_type, perturbation=pert)
        return [rv, ri.long(), cv, ci.long(), s[0], s[1], s[2], s[3], s[4].long()]

    def fused_gcost_certificate(self, query, db, query_dual, db_dual, cost_type, query_global_index=None,
                                database_global_index=None, sigma=0., seed=0, perturb_mode=1, row_is_source=True,
                                index_hash_coeffs=None, compute_denominator=1, compute_precision=0):
        """[num, den, max s+, max |c|, count int64] (generic_scan.py:545-558)."""
        if isinstance(query_global_index, (int, bool)) and database_global_index is None:
            compute_denominator, query_global_index = query_global_index, None
        _check(query, db, 1, (query_dual, len(query)), (db_dual, len(db)))
        pert = make_perturbation(query, db, query_global_index, database_global_index, sigma, seed, perturb_mode,
                                 row_is_source, index_hash_coeffs)
        self._record("norm_certificate")
        s = norm_scan(query, db, query_dual, db_dual, 0, cost_type, perturbation=pert)[4]
        den = s[1] if compute_denominator else s[1].new_zeros(())
        return [s[0], den, s[2], s[3], s[4].long()]

    def fused_gcost_pairs(self, query, db, rows, cols, cost_type, source_index=None, target_index=None, sigma=0.,
                          seed=0, mode=1, coefficients=None):
        """fp64 cost of each (row, col) edge (norm_cost_scan_kernel.cu:249-275), plus the
        perturbation noise of (source_index[row], target_index[col]) when sigma > 0."""
        from .pairs import pair_costs
        pert = None
        if sigma is not None and float(sigma) != 0.0:
            pert = make_perturbation(query, db, source_index, target_index, sigma, seed, mode, True, coefficients)
        return pair_costs(NORM_KIND[cost_type], query, db, rows, cols, perturbation=pert)


@dataclass
class LowrankBidirScanResult:
    """Result of the bidirectional ℓ2² scan (bilinear_topk.py:26-36)."""

    dual_feasibility: float
    rows: np.ndarray
    cols: np.ndarray
    diagnostics: Dict[str, Any]


def flatten_candidates(rv, ri, cv, ci, theta: float = 0.0, *, query_is_source: bool = True):
    """Candidate pairs with score > theta on the device, in the reference order:
    query rows (row-major, slot order) then database columns
    (bilinear_topk.py:393-448)."""
    rmask = (rv > float(theta)) & (ri >= 0)
    cmask = (cv > float(theta)) & (ci >= 0)
    q_local = torch.nonzero(rmask, as_tuple=False)[:, 0]
    d_local = torch.nonzero(cmask, as_tuple=False)[:, 0]
    q_match = ri[rmask].to(torch.int64)
    d_match = ci[cmask].to(torch.int64)
    if query_is_source:
        rows = torch.cat((q_local, d_match))
        cols = torch.cat((q_match, d_local))
    else:
        rows = torch.cat((q_match, d_local))
        cols = torch.cat((q_local, d_match))
    return rows, cols


def _to_device(a, device, dtype):
    if torch.is_tensor(a):
        return a.detach().to(device=device, dtype=dtype).contiguous()
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype).to(device, non_blocking=True).contiguous()


def _holds_fp32(feat) -> bool:
    """True when every element of feat is an fp32 value (fp32 storage, or fp64 values that
    round-trip through fp32 exactly)."""
    if torch.is_tensor(feat):
        if feat.dtype == torch.float32:
            return True
        v = feat.detach()
        return bool(torch.equal(v.to(torch.float32).to(v.dtype), v))
    arr = np.asarray(feat)
    if arr.dtype == np.float32:
        return True
    return bool(np.array_equal(arr.astype(np.float32).astype(arr.dtype), arr))


def raw_lowrank_bidir_feasibility_pricing_scan(source_feat, target_feat, source_cost, target_cost, source_dual,
                                               target_dual, *, topk, theta=0.0, gpu_id=0, memory_floor_mib=768.0,
                                               resident_multiplier=1.10, col_reduce_tile=256, col_kernel="auto",
                                               collect_timing=False, collect_linf_diagnostics=False, dot_scale=1.0,
                                               compute_precision="fp32", return_device=False, exact=True):
    """Full bidirectional ℓ2² pricing scan + dual-feasibility certificate with the
    signature of bilinear_topk.raw_lowrank_bidir_feasibility_pricing_scan.

    Score of pair (i, j): (s<x_i,y_j> + (f_i - a_i)) + (g_j - b_j); candidates are the
    top-k of every source row and every target column with score > theta.  exact (the
    default): the lists are the exact fp64 top-k (the fp64 re-check, HB_L2SQ_EXACT);
    exact=False keeps the fp32-class ranking of the tensor-core dot.  compute_precision
    "fp64" (the reference's fp64 dots, cost.cu:108-122) gives the exact fp64 lists
    whatever `exact` says, for features holding fp32 values; the certificate terms are
    fp32-class in every mode (diagnostics["certificate_precision"])."""
    k = int(round(float(topk)))
    if abs(float(topk) - k) > 1e-9:
        raise ValueError("fused inner-product scan requires an integer pricing_topk")
    kernel_k = topk_bucket(k)
    if str(compute_precision) not in {"fp32", "fp64", "tf32"}:
        raise ValueError("compute_precision must be one of: fp32, fp64")
    fp64 = str(compute_precision) == "fp64"
    if fp64:
        # fp64 ranking: the exact fp64 top-k lists of the fp64 scores of the fp32 features (the
        # fp64 re-check); features given in fp64 must hold fp32 values (the reference stores
        # points as fp32, types.py:26), and the certificate terms stay fp32-class
        for name, feat in (("source", source_feat), ("target", target_feat)):
            if not _holds_fp32(feat):
                raise NotImplementedError(f"compute_precision='fp64' needs {name} features representable in fp32")
        exact = True
    if col_kernel not in ("auto", "current", "warp2", "warp4"):
        raise ValueError("col_kernel must be one of {auto, current, warp2, warp4}")
    device = torch.device(f"cuda:{int(gpu_id)}")
    lib()
    n_source, n_target = int(source_feat.shape[0]), int(target_feat.shape[0])
    if n_source <= 0 or n_target <= 0:
        raise ValueError("source and target must both be non-empty")
    d = int(source_feat.shape[1])
    if int(target_feat.shape[1]) != d:
        raise ValueError("source and target feature dimensions must match")
    start = time.perf_counter()
    x = _to_device(source_feat, device, torch.float32)
    y = _to_device(target_feat, device, torch.float32)
    a = _to_device(source_cost, device, torch.float64).view(-1)
    b = _to_device(target_cost, device, torch.float64).view(-1)
    f = _to_device(source_dual, device, torch.float64).view(-1)
    g = _to_device(target_dual, device, torch.float64).view(-1)
    rv, ri, cv, ci, stats = l2sq_scan(x, y, a, b, f - a, g - b, k, dot_scale=float(dot_scale),
                                      precision="fp32" if fp64 else str(compute_precision), exact=bool(exact))
    rows_t, cols_t = flatten_candidates(rv, ri, cv, ci, theta)
    s = stats.cpu().tolist()
    num_sq, den_sq, max_pos, cost_linf, count = s[0], s[1], s[2], s[3], int(round(s[4]))
    dual_feas = math.sqrt(max(num_sq, 0.0)) / (1.0 + math.sqrt(max(den_sq, 0.0)))
    if return_device:
        rows, cols = rows_t, cols_t
    else:
        rows = rows_t.cpu().numpy().astype(np.int64, copy=False)
        cols = cols_t.cpu().numpy().astype(np.int64, copy=False)
    max_violation = max(float(rv.max().item()) if rv.numel() else 0.0, 0.0)
    diagnostics: Dict[str, Any] = {
        "dual_feasibility": float(dual_feas),
        "kernel_backend": "hello_b200",
        "dual_feasibility_num_sq": float(num_sq),
        "dual_feasibility_den_sq": float(den_sq),
        "dual_feasibility_positive_count": count,
        "dual_feasibility_max_violation": float(max_violation),
        "dual_feasibility_source": "early_fused_lowrank_bidir_scan",
        "fused_scan_time": time.perf_counter() - start,
        "fused_scan_candidate_count": int(rows.numel() if torch.is_tensor(rows) else rows.size),
        "fused_scan_resident_side": "both",
        "fused_scan_n_source": n_source,
        "fused_scan_n_target": n_target,
        "fused_scan_topk": k,
        "fused_scan_topk_bucket": kernel_k,
        "pairwise_passes": 2,
        "scan_traversal": "fused_tensor_core_bidirectional",
        "cost_compute_precision": str(compute_precision),
        "fp64_recheck": bool(exact),
        "certificate_precision": "fp32-class",  # the certificate terms of the tensor-core scores
    }
    if exact:
        diagnostics["fp64_rescanned_lists"] = sum(l2sq_last_rescans())
    if collect_linf_diagnostics:
        diagnostics.update({"dual_feasibility_cost_linf": float(cost_linf),
                            "relative_linf_dual_feasibility": float(max_violation) / (1.0 + float(cost_linf))})
    return LowrankBidirScanResult(dual_feasibility=float(dual_feas), rows=rows, cols=cols, diagnostics=diagnostics)
