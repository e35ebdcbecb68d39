"""CPU oracle for the HELLO hot path (pricing scan, pair costs, restricted-OT PDHG).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` (as the
checker) and ``bench.py`` (its CPU-baseline and reference legs) may import this
package.  The product package ``hello_ot_b200`` never imports it and has no CPU
fallback.

``liboracle.so`` (built from ``oracle.c`` by ``make -C oracle``) restates the
reference algorithms in C; ``_ref/hello_ot_cpp`` holds the reference's own
C++ backend (``src/hello_ot/_native/cpp/{scan,solver}.cpp``) compiled from its
sources by ``make -C oracle ref``.  The restatement is pinned against the
reference by the fixtures in ``tests/golden``.
"""
from __future__ import annotations

import ctypes
import importlib
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
KIND = {"l1": 0, "linf": 1, "l2": 2, "raw": 3, "l2^2": 3, "lowrank": 3}
REASONS = {1: "OPTIMAL", 2: "ITERATION_LIMIT", 3: "NUMERICAL_DIVERGENCE"}

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_LIB = None


class PdlpInfo(ctypes.Structure):
    _fields_ = [("iterations", ctypes.c_int64), ("restarts", ctypes.c_int64),
                ("reason", ctypes.c_int32), ("pad", ctypes.c_int32),
                ("pobj", ctypes.c_double), ("dobj", ctypes.c_double), ("ap", ctypes.c_double),
                ("rp", ctypes.c_double), ("ad", ctypes.c_double), ("rd", ctypes.c_double),
                ("gap", ctypes.c_double), ("weight", ctypes.c_double),
                ("cost_norm", ctypes.c_double), ("mass_norm", ctypes.c_double)]


def build(force: bool = False) -> Path:
    """Compile liboracle.so, and the reference's CPU build when the environment variable
    HELLO_REF names a checkout of the reference project (its sources are not in this
    repository)."""
    lib = HERE / "liboracle.so"
    if force or not lib.exists() or lib.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), f"PYTHON={sys.executable}"], check=True,
                       stdout=subprocess.DEVNULL)
    ref = Path(os.environ["HELLO_REF"]) if os.environ.get("HELLO_REF") else None
    if ref is not None and (ref / "src/hello_ot/_native/cpp/scan.cpp").exists():
        subprocess.run(["make", "-C", str(HERE), "ref", f"REF={ref}", f"PYTHON={sys.executable}"],
                       check=True, stdout=subprocess.DEVNULL)
    return lib


def _lib():
    global _LIB
    if _LIB is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        lib = ctypes.CDLL(str(path))
        lib.orc_scan.argtypes = [ctypes.c_int, ctypes.c_int, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                 ctypes.c_int64, _f64p, _f64p, _f64p, _f64p, ctypes.c_double,
                                 ctypes.c_int, ctypes.c_int, _f64p, _i64p, _f64p, _i64p, _f64p, ctypes.c_int]
        lib.orc_pair_scores.argtypes = [ctypes.c_int, _f32p, _f32p, ctypes.c_int64, _f64p, _f64p, _f64p, _f64p,
                                        ctypes.c_double, _i64p, _i64p, ctypes.c_int64, _f64p,
                                        ctypes.c_void_p, ctypes.c_int]
        lib.orc_pair_costs.argtypes = [ctypes.c_int, _f32p, _f32p, ctypes.c_int64, _f64p, _f64p,
                                       ctypes.c_double, _i64p, _i64p, ctypes.c_int64, _f64p, ctypes.c_int]
        lib.orc_pdlp.argtypes = [_i64p, _i64p, _f64p, ctypes.c_int64, _f64p, ctypes.c_int64, ctypes.c_int64,
                                 _f64p, _f64p, ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_double,
                                 ctypes.c_double, ctypes.c_int, _f64p, _f64p, ctypes.POINTER(PdlpInfo)]
        _LIB = lib
    return _LIB


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _f64(a, n=None):
    if a is None:
        return np.zeros(max(n or 0, 1), dtype=np.float64)
    return np.ascontiguousarray(a, dtype=np.float64).reshape(-1)


def scan(kind, x, y, rowb, colb, nx=None, ny=None, *, dot_scale=1.0, rk=1, ck=1, exact=True, threads=0):
    """Bidirectional pricing scan.  ``rowb``/``colb`` are (f-a, g-b) for the raw
    bilinear kind and (f, g) for the norm kinds.  Returns
    (rv, ri, cv, ci, stats[num, den, max_pos, max_abs_cost, count])."""
    x, y = _f32(x), _f32(y)
    q, d = x.shape
    n = y.shape[0]
    rv = np.empty((q, max(rk, 1))); ri = np.empty((q, max(rk, 1)), np.int64)
    cv = np.empty((n, max(ck, 1))); ci = np.empty((n, max(ck, 1)), np.int64)
    stats = np.zeros(5)
    rc = _lib().orc_scan(KIND[kind], int(exact), x, y, q, n, d, _f64(rowb), _f64(colb), _f64(nx, q),
                         _f64(ny, n), float(dot_scale), int(rk), int(ck), rv, ri, cv, ci, stats, int(threads))
    if rc:
        raise ValueError(f"oracle scan rejected its inputs ({rc})")
    return rv[:, :rk], ri[:, :rk], cv[:, :ck], ci[:, :ck], stats


def pair_scores(kind, x, y, rowb, colb, nx, ny, rows, cols, *, dot_scale=1.0, threads=0):
    """Exact (score, cost) of selected pairs."""
    x, y = _f32(x), _f32(y)
    rows = np.ascontiguousarray(rows, np.int64).reshape(-1)
    cols = np.ascontiguousarray(cols, np.int64).reshape(-1)
    score = np.empty(rows.size)
    cost = np.empty(rows.size)
    _lib().orc_pair_scores(KIND[kind], x, y, x.shape[1], _f64(rowb), _f64(colb), _f64(nx, len(x)),
                           _f64(ny, len(y)), float(dot_scale), rows, cols, rows.size, score,
                           cost.ctypes.data, int(threads))
    return score, cost


def pair_costs(kind, x, y, rows, cols, a=None, b=None, *, dot_scale=1.0, threads=0):
    """Active-support pair costs in fp64 (the SDDMM restatement)."""
    x, y = _f32(x), _f32(y)
    rows = np.ascontiguousarray(rows, np.int64).reshape(-1)
    cols = np.ascontiguousarray(cols, np.int64).reshape(-1)
    out = np.empty(rows.size)
    rc = _lib().orc_pair_costs(KIND[kind], x, y, x.shape[1], _f64(a, len(x)), _f64(b, len(y)),
                               float(dot_scale), rows, cols, rows.size, out, int(threads))
    if rc:
        raise ValueError("oracle pair_costs rejected its inputs")
    return out


def pdlp(rows, cols, costs, source_mass, target_mass, x0=None, y0=None, *, frequency=200,
         iteration_limit=2**31 - 1, tolerance=1e-6, rescale=False):
    """Single-thread restatement of the reference C++ restricted-OT PDHG."""
    rows = np.ascontiguousarray(rows, np.int64).reshape(-1)
    cols = np.ascontiguousarray(cols, np.int64).reshape(-1)
    costs = _f64(costs)
    a, b = _f64(source_mass), _f64(target_mass)
    masses = np.ascontiguousarray(np.concatenate((a, b)))
    x0 = np.zeros(costs.size) if x0 is None else _f64(x0)
    y0 = np.zeros(masses.size) if y0 is None else _f64(y0)
    if isinstance(tolerance, dict):
        tob = float(tolerance.get("objective", 1e-6))
        tp, td = float(tolerance.get("primal", tob)), float(tolerance.get("dual", tob))
    else:
        tob = tp = td = float(tolerance)
    x = np.empty(costs.size)
    y = np.empty(masses.size)
    info = PdlpInfo()
    rc = _lib().orc_pdlp(rows, cols, costs, costs.size, masses, a.size, masses.size, x0, y0, int(frequency),
                         int(iteration_limit), tob, tp, td, int(rescale), x, y, ctypes.byref(info))
    if rc:
        raise ValueError(f"oracle pdlp rejected its inputs ({rc})")
    return dict(x=x, y=y, iterations=info.iterations, restarts=info.restarts,
                termination_reason=REASONS.get(info.reason, "UNSPECIFIED"), obj_val=info.pobj,
                dual_obj_val=info.dobj, primal_feas=info.rp, dual_feas=info.rd, gap=info.gap,
                abs_primal=info.ap, abs_dual=info.ad, primal_weight=info.weight)


def filter_new_pairs(active_keys, rows, cols, n_target):
    """New candidate pairs (ActiveSupport.filter_new_candidate_pairs,
    src/hello_ot/restricted_ot/active_support.py:483-506): the unique candidate
    keys row * n_target + col, ascending, minus the support keys.  Returns
    (new_rows int32, new_cols int32, found, new_count)."""
    rows = np.asarray(rows, np.int64).reshape(-1)
    cols = np.asarray(cols, np.int64).reshape(-1)
    found = int(rows.size)
    keys = np.unique(rows * int(n_target) + cols)
    active = np.asarray(active_keys, np.int64).reshape(-1)
    if active.size:
        keys = keys[~np.isin(keys, active)]
    return (keys // int(n_target)).astype(np.int32), (keys % int(n_target)).astype(np.int32), found, int(keys.size)


def prune_select(rows, cols, costs, x_prev, creation, duals, n_source, num_to_remove, current_iter):
    """Removal positions of DualGapCleaning in protect-new mode
    (src/hello_ot/refinement/budgeted_pruning.py:27-57, 119-175; reduced costs as
    ActiveSupport.pruning_values, src/hello_ot/restricted_ot/active_support.py:401-421).
    Returns (positions int32 or None when too few are removable, removable count)."""
    rows = np.asarray(rows, np.int64)
    cols = np.asarray(cols, np.int64)
    duals = np.asarray(duals, np.float64)
    u, v = duals[:n_source], duals[n_source:]
    rc = np.asarray(costs, np.float64) - (u[rows] + v[cols])
    rc = np.where(np.isfinite(rc), rc, -np.inf)
    creation = np.asarray(creation, np.int64)
    removable = (creation != current_iter) & (creation != -1) & ~(np.abs(np.asarray(x_prev, np.float64)) > 1e-15)
    idx = np.flatnonzero(removable)
    if idx.size < num_to_remove:
        return None, int(idx.size)
    order = np.argsort(-rc[idx], kind="stable")
    return idx[order[:num_to_remove]].astype(np.int32), int(idx.size)


def noise(src, tgt, sigma, seed, mode, coeffs):
    """Norm-cost perturbation noise in fp64 (cost.cu:380-423 sigma_noise; the NumPy form
    of metric_perturbation.py:35-59).  mode 1 (index_hash): every fp32 step rounded
    on its own, bit for bit as the reference.  mode 0 (rank2): np.sin in fp32, an
    approximation of the fused kernels' __sinf."""
    src = np.asarray(src, np.int64)
    tgt = np.asarray(tgt, np.int64)
    f32 = np.float32
    if int(mode) == 0:
        z = (src.astype(f32) * f32(12.9898) + tgt.astype(f32) * f32(78.233)) + f32(int(seed) * 0.001)
        v = np.sin(z).astype(f32) * f32(0.5) + f32(0.5)
        return (f32(sigma) * v).astype(np.float64)
    h = []
    for prime, (a, b, o) in zip((2003, 2011), (coeffs[0:3], coeffs[3:6])):
        s_, t_ = np.remainder(src, prime).astype(f32), np.remainder(tgt, prime).astype(f32)
        x = ((f32(a) * s_ + f32(b) * t_) + s_ * t_) + f32(o)
        h.append(x - f32(prime) * np.floor(x * f32(1.0 / prime)))
    v = ((h[0] + f32(2003) * h[1]) + f32(0.5)) * f32(1.0 / 4028033.0)
    return float(sigma) * v.astype(np.float64)


def load_ref(kind: str):
    """The reference's compiled CPU module ``hello_ot_cpp._scan`` / ``._lp``."""
    if not (REF_DIR / "hello_ot_cpp" / "__init__.py").exists():
        raise RuntimeError("reference CPU backend not built: run `make -C oracle ref`")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    return importlib.import_module(f"hello_ot_cpp._{kind}")
