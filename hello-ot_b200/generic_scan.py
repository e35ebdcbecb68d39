"""Module-level scan entry points with the reference's `hello_ot.kernels.generic_scan`
interface (src/hello_ot/kernels/generic_scan.py:219-306 `directional`, :328-404
`bidirectional`, :424-465 `certificate_only`), the calls the gpu_resident solver makes
(src/hello_ot/gpu_resident/cost.py:118-161 `scan`).  Every call runs one library kernel
launch sequence over the whole problem (no host tiling: `workspace_bytes`,
`tile_limits` and `planned_tiles` are accepted and ignored).

raw_extras = (ex, ey, sigma), the l2^2 rank-2 perturbation (generic_scan.py:309-325
`_raw_dots`: dots + 2 <ex, ey> - sigma / 2), is folded into the same product: the extra
columns are appended to the features (scaled by 2 / dot_scale, exact in fp32), sigma / 2
is added to the query cost and subtracted from the query bias, so scores and costs are
those of the perturbed dot product computed at the same fp32-class precision.

compute_precision=1 (fp64 coordinates) is not implemented on this path and raises.
"""
from __future__ import annotations

from collections import Counter

import torch

from .perturb import make_perturbation
from .scan import _check, l2sq_scan, l2sq_topk, norm_scan, norm_topk

_ROUTES = Counter()  # route diagnostics, incremented by callers as in the reference


def _precision(compute_precision, raw, x, fp64_lists=False):
    """compute_precision 1 (fp64) is served only where the lists can be the exact fp64 top-k
    of fp32 coordinates (raw bidirectional scans, fp64_lists=True: the fp64 re-check)."""
    if compute_precision not in (0, 1) or (not raw and x.dtype != torch.float32):
        raise ValueError("norm scans require FP32 coordinate storage and precision 0 or 1")
    if x.dtype != torch.float32 or (compute_precision == 1 and not (raw and fp64_lists)):
        raise NotImplementedError("hello_ot_b200 scans compute from fp32 coordinates (compute_precision=0; "
                                  "compute_precision=1 only for raw bidirectional scans, as exact fp64 lists)")


def _perturbation(x, y, args):
    """The reference's perturbation tuple (qi, di, sigma, seed, mode, direction,
    coefficients) as the library's struct (generic_scan.py:190-205 checks)."""
    if args is None or float(args[2]) == 0:
        return None
    qi, di, sigma, seed, mode, direction, coefficients = args
    if mode == 1 and (coefficients is None or coefficients.dtype != torch.int64 or coefficients.numel() != 6):
        raise ValueError("index_hash requires six int64 coefficients")
    return make_perturbation(x, y, qi, di, sigma, seed, mode, bool(direction), coefficients)


def _fold_extras(x, y, query_cost, query_bias, dot_scale, raw_extras):
    """Append the rank-2 perturbation columns; returns (x', y', query_cost', query_bias')."""
    if raw_extras is None:
        return x, y, query_cost, query_bias
    ex, ey, sigma = raw_extras
    if ex.shape[0] != x.shape[0] or ey.shape[0] != y.shape[0] or ex.ndim != 2 or ey.shape[1] != ex.shape[1]:
        raise ValueError("raw_extras must hold one row per query and per database point")
    scale = 2.0 / float(dot_scale)  # 1 or 2: exact
    x2 = torch.cat((x, ex.to(device=x.device, dtype=x.dtype) * scale), 1).contiguous()
    y2 = torch.cat((y, ey.to(device=y.device, dtype=y.dtype)), 1).contiguous()
    half = 0.5 * float(sigma)
    cost = None if query_cost is None else query_cost + half
    bias = None if query_bias is None else query_bias - half
    return x2, y2, cost, bias


def bidirectional(x, y, f, g, k, kind, *, raw_costs=None, raw_biases=None, dot_scale=2., workspace_bytes=None,
                  perturbation=None, compute_precision=0, raw_extras=None, tile_limits=None, planned_tiles=None,
                  exact=True):
    """(rv q x k, ri int64, cv n x k, ci int64, num, den, max s+, max |c|, count int64):
    row and column top-k of the scores and the full certificate (generic_scan.py:328-404).
    kind 3 (raw l2^2) takes raw_costs = (nx, ny) and raw_biases = (f - nx, g - ny); its lists
    are the exact fp64 top-k (the fp64 re-check, as ScanExtension's default) unless
    exact=False; compute_precision=1 (fp64) asks for them in any case."""
    _check(x, y, k, (f, len(x)), (g, len(y)))
    raw = raw_costs is not None
    _precision(compute_precision, raw, x, fp64_lists=True)
    if compute_precision == 1:
        exact = True
    if raw and perturbation is not None and float(perturbation[2]) != 0:
        raise ValueError("norm perturbation does not apply to raw pricing")
    if kind not in (0, 1, 2, 3) or (kind == 3 and not raw):
        raise ValueError("generic bidirectional cost must be l1, linf, l2 or raw")
    if raw:
        nx, ny = raw_costs
        qb, dbb = raw_biases
        _check(x, y, k, (nx, len(x)), (ny, len(y)), (qb, len(x)), (dbb, len(y)))
        if dot_scale not in (1., 2.):
            raise ValueError("dot_scale must be exactly 1 or 2")
        xx, yy, nxx, qbb = _fold_extras(x, y, nx, qb, dot_scale, raw_extras)
        rv, ri, cv, ci, s = l2sq_scan(xx, yy, nxx, ny, qbb, dbb, k, dot_scale=float(dot_scale), exact=bool(exact))
    else:
        pert = _perturbation(x, y, perturbation)
        rv, ri, cv, ci, s = norm_scan(x, y, f, g, k, kind, perturbation=pert)
    return rv, ri.long(), cv, ci.long(), s[0], s[1], s[2], s[3], s[4].long()


def directional(x, y, db_bias, k, kind, *, query_bias=None, dot_scale=2., workspace_bytes=None, minimum=False,
                perturbation=None, collect_statistics=False, compute_precision=0, raw_extras=None):
    """Best k database points of every query (generic_scan.py:219-306): descending scores
    (raw: (dot + query_bias) + db_bias; norms: db_bias - cost), or with minimum=True the
    negated scores ascending; indices int64 (-1 where fewer than k exist).  Norm calls
    with collect_statistics=True add [sum c^2, max |c|]."""
    raw = query_bias is not None
    vectors = [(db_bias, len(y))]
    if raw:
        vectors.append((query_bias, len(x)))
    _check(x, y, k, *vectors)
    if kind not in (0, 1, 2, 3) or (kind == 3 and not raw):
        raise ValueError("generic directional cost must be l1, linf, l2 or raw")
    _precision(compute_precision, raw, x)
    pert = None if raw else _perturbation(x, y, perturbation)
    if raw and ((perturbation is not None and float(perturbation[2]) != 0) or collect_statistics):
        raise ValueError("norm extensions do not apply to raw initial")
    if raw:
        if dot_scale not in (1., 2.):
            raise ValueError("dot_scale must be exactly 1 or 2")
        xx, yy, _, qbb = _fold_extras(x, y, None, query_bias, dot_scale, raw_extras)
        values, ids = l2sq_topk(xx, yy, qbb, db_bias, k, dot_scale=float(dot_scale))
        stats = None
    else:
        values, ids, stats = norm_topk(x, y, db_bias, k, kind, compute_stats=bool(collect_statistics),
                                       perturbation=pert)
    out = (values.neg_() if minimum else values, ids.long())
    return (*out, stats) if collect_statistics else out


def certificate_only(x, y, f, g, kind, *, perturbation=None, compute_denominator=True, workspace_bytes=None,
                     compute_precision=0, raw_costs=None, dot_scale=2.):
    """(num, den, max s+, max |c|, count int64) of the full scan without candidates
    (generic_scan.py:424-465); den is zero when compute_denominator is false."""
    _check(x, y, 1, (f, len(x)), (g, len(y)))
    raw = raw_costs is not None
    _precision(compute_precision, raw, x)
    if kind not in (0, 1, 2, 3) or (kind == 3 and not raw):
        raise ValueError("certificate-only requires a norm or raw cost")
    if raw:
        nx, ny = raw_costs
        _check(x, y, 1, (nx, len(x)), (ny, len(y)))
        if dot_scale not in (1., 2.) or perturbation is not None:
            raise ValueError("raw certificates require dot_scale 1 or 2 and encoded perturbation")
        s = l2sq_scan(x, y, nx, ny, f - nx, g - ny, 0, dot_scale=float(dot_scale))[4]
    else:
        s = norm_scan(x, y, f, g, 0, kind, perturbation=_perturbation(x, y, perturbation))[4]
    den = s[1] if compute_denominator else s[1].new_zeros(())
    return s[0], den, s[2], s[3], s[4].long()
