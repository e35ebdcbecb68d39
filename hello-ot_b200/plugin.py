"""The hello_ot plug-in: routes the reference's native hot path to libhello_b200.

``install()`` binds this package into an imported reference package ``hello_ot``
(WenzhouXia/hello-ot) so that ``hello_ot.solve(..., options=SolverOptions(
backend="native"))`` runs its pricing scans, pair costs, restricted LPs, support
filter, pruning selection and coarsest leaf solves on the B200 kernels, while the
hierarchy driver, active-support storage, result objects and f/g duals stay the
reference's own code.  It replaces, in the reference's modules, exactly the
names the native backend reaches for those operations:

  * ``hello_ot._native_compat.require_native_runtime_compatibility``
    (src/hello_ot/_native_compat.py:36): the prebuilt-wheel ABI check, replaced by
    loading libhello_b200 (which needs CUDA);
  * ``hello_ot._source_build.load_native_module`` (src/hello_ot/_source_build.py:152)
    and ``hello_ot.kernels.generic_scan._module`` (kernels/generic_scan.py:34): any
    request for a reference CUDA module raises, so nothing falls back to it;
  * ``hello_ot.kernels.generic_scan.ScanExtension`` (kernels/generic_scan.py:468)
    and ``bidirectional`` / ``directional`` / ``certificate_only`` (:219-465): norm
    scans, certificates, directional (initial) scans and norm pair costs;
  * ``hello_ot.kernels.bilinear_topk._load_extension`` (kernels/bilinear_topk.py:39)
    and ``raw_lowrank_bidir_feasibility_pricing_scan`` (:207): the ℓ2² pricing scan
    (whole scan, both clouds resident) and the ℓ2² initial scans;
  * ``hello_ot.restricted_ot.runtime.build_lp_backend`` (restricted_ot/runtime.py:75):
    engine "cupdlpx" becomes the library's restricted-OT PDHG, a
    ``RestrictedOTPDLP`` (_internal/lp/restricted_ot_pdlp.py:12) so the LP is
    dispatched through ``solve_restricted`` (restricted_ot/backend.py:866);
  * ``hello_ot.costs.pairs._cost_pairs_{lowrank,l1,linf,euclidean}_batched``
    (costs/pairs.py:88-600): active-support pair costs (SDDMM);
  * ``ActiveSupport.filter_new_candidate_pairs`` (restricted_ot/active_support.py:483)
    and ``DualGapCleaning._select_protect_new_indices`` (refinement/budgeted_pruning.py:119);
  * ``hello_ot.hierarchy.coarsest._build_leaf_costs_pad_batch_gemm`` (:166),
    ``hello_ot.costs.metric._metric_cost_matrix`` and
    ``_solve_lowrank_leaf_with_pot_from_precomputed_cost`` (coarsest.py:50): the
    coarsest leaf (POT's ``ot.emd`` in the reference) on the GPU.

One operation outside the hot path is redirected to the reference's own code:
the support sparsification of an over-dense LP primal
(restricted_ot/sparsification_postprocess.py:84) uses the reference's numba
engine instead of its C++ extension module.

Names are replaced wherever the reference holds them (modules that imported
them by value included), and ``uninstall()`` restores every one.  ``routes()``
counts the calls that reached this package by operation; a reference
implementation of a routed operation that is still called is counted under
``reference:<name>`` (and the reference's CUDA modules raise), so a caller can
check that the whole hot path ran here.
"""
from __future__ import annotations

import importlib
import pkgutil
import sys
import threading
import time
from collections import Counter
from typing import Any, Dict, List, Tuple

import numpy as np
import torch

from ._lib import lib, load_library
from .coarsest import solve_leaf_from_cost
from .pairs import KIND, pair_costs
from .pdlp import NativeRestrictedOTPDLP
from .scan import ScanExtension, raw_lowrank_bidir_feasibility_pricing_scan
from .support import filter_new_candidate_pairs, select_prune_positions
from . import generic_scan as _generic

_ROUTES: Counter = Counter()
_LOCK = threading.Lock()
_STATE: Dict[str, Any] = {"installed": False, "undo": []}


def routes(*, reset: bool = False) -> Dict[str, int]:
    """Calls per routed operation since the last reset."""
    with _LOCK:
        out = dict(_ROUTES)
        if reset:
            _ROUTES.clear()
    return out


def _count(key: str) -> None:
    with _LOCK:
        _ROUTES[key] += 1


class BoundScanExtension(ScanExtension):
    """The reference's ScanExtension interface on libhello_b200, with route counts."""

    def _record(self, name):
        super()._record(name)
        _count("scan:" + name)

    def fused_gcost_pairs(self, *args, **kwargs):
        _count("pair_costs:norm_fused")
        return super().fused_gcost_pairs(*args, **kwargs)


def _dev(v, device, dtype):
    if torch.is_tensor(v):
        return v.detach().to(device=device, dtype=dtype).contiguous()
    return torch.as_tensor(np.ascontiguousarray(v), dtype=dtype).to(device).contiguous()


def _device_of(*values):
    for v in values:
        if torch.is_tensor(v) and v.is_cuda:
            return v.device
    return torch.device("cuda", torch.cuda.current_device())


def _pair_cost_function(name: str, kind: int):
    """A replacement of costs/pairs.py ``_cost_pairs_<name>_batched``: same arguments,
    fp64 costs in the input order, torch on the indices' device when the indices are
    tensors, else numpy (the reference returns fp32 for the norms; fp64 is kept)."""

    def cost_pairs(level_cache, rows, cols, *args, **kwargs):
        _count(f"pair_costs:{name}")
        as_torch = torch.is_tensor(rows)
        dev = _device_of(rows, cols)
        r = _dev(rows, dev, torch.int64).view(-1)
        c = _dev(cols, dev, torch.int64).view(-1)
        if kind == 3:
            x, y = level_cache["F"], level_cache["G"]
            a = _dev(level_cache["a"], dev, torch.float64).view(-1)
            b = _dev(level_cache["b"], dev, torch.float64).view(-1)
            scale = float(level_cache.get("dot_scale", 1.0))
            if str(level_cache.get("compute_precision", "fp32")) == "fp64":
                raise NotImplementedError("hello_ot_b200 pair costs read fp32 features (cost_precision='fp32')")
        else:
            x, y, a, b, scale = level_cache["S"], level_cache["T"], None, None, 1.0
        out = pair_costs(kind, _dev(x, dev, torch.float32), _dev(y, dev, torch.float32), r, c, a, b, scale)
        return out if as_torch else out.cpu().numpy()

    cost_pairs.__name__ = f"_cost_pairs_{name}_batched"
    cost_pairs.__qualname__ = cost_pairs.__name__
    return cost_pairs


def _refuse_native_module(module_name, *args, **kwargs):
    _count(f"reference:native_module:{module_name}")
    raise RuntimeError(f"hello_ot_b200 plug-in: the reference's CUDA module {module_name!r} was requested; "
                       "the native hot path is bound to libhello_b200 and has no fallback")


def _tripwire(name: str, original):
    """Count a call into a reference implementation of a routed operation, then run it."""

    def wrapper(*args, **kwargs):
        _count(f"reference:{name}")
        return original(*args, **kwargs)

    wrapper.__name__ = getattr(original, "__name__", name)
    wrapper.__wrapped__ = original
    return wrapper


def _import_all(root):
    """Import every submodule of the reference package so that names imported by
    value are visible for rebinding (subpackages that need absent optional
    dependencies are skipped)."""
    for info in pkgutil.walk_packages(root.__path__, root.__name__ + "."):
        if ".variants" in info.name or info.name.endswith("__main__"):
            continue
        try:
            importlib.import_module(info.name)
        except Exception:  # noqa: BLE001  (an optional dependency of an unrelated module)
            continue


def _rebind(root_name: str, original, replacement, undo: List[Tuple[Any, str, Any]]):
    """Replace ``original`` by ``replacement`` in every loaded module of the package."""
    hits = 0
    for name, module in list(sys.modules.items()):
        if module is None or not (name == root_name or name.startswith(root_name + ".")):
            continue
        for attr, value in list(vars(module).items()):
            if value is original:
                undo.append((module, attr, value))
                setattr(module, attr, replacement)
                hits += 1
    return hits


def _set(obj, attr, value, undo):
    undo.append((obj, attr, getattr(obj, attr)))
    setattr(obj, attr, value)


def install(hello_ot=None, *, device=None):
    """Bind libhello_b200 into the reference package (imports ``hello_ot`` when not
    given).  Idempotent; returns the reference package."""
    if hello_ot is None:
        hello_ot = importlib.import_module("hello_ot")
    if _STATE["installed"]:
        return hello_ot
    load_library()  # loads without a GPU; a solve checks for CUDA when it starts
    root = hello_ot.__name__
    _import_all(hello_ot)
    m = lambda name: importlib.import_module(f"{root}.{name}")  # noqa: E731
    undo: List[Tuple[Any, str, Any]] = []

    compat = m("_native_compat")

    def require_native_runtime_compatibility():
        lib()
        if not torch.cuda.is_available():
            raise RuntimeError("hello_ot_b200 plug-in: the native backend needs a CUDA device (no CPU fallback)")

    _rebind(root, compat.require_native_runtime_compatibility, require_native_runtime_compatibility, undo)
    _rebind(root, m("_source_build").load_native_module, _refuse_native_module, undo)
    gs = m("kernels.generic_scan")
    _rebind(root, gs._module, _refuse_native_module, undo)

    # scans
    _rebind(root, gs.ScanExtension, BoundScanExtension, undo)
    for name in ("bidirectional", "directional", "certificate_only"):
        ours = getattr(_generic, name)

        def counted(*args, _f=ours, _n=name, **kwargs):
            _count(f"scan:module_{_n}")
            return _f(*args, **kwargs)

        _rebind(root, getattr(gs, name), counted, undo)
    shared_ext = BoundScanExtension()
    bt = m("kernels.bilinear_topk")

    def _load_extension():
        return shared_ext

    _rebind(root, bt._load_extension, _load_extension, undo)
    _set(bt, "_EXT_MODULE", shared_ext, undo)
    init_state = m("initialization.state")
    _set(init_state, "_fused_mips_ext", None, undo)
    stopping = m("refinement.stopping")
    if hasattr(stopping, "_CUDA_CPP_DUAL_FEASIBILITY_EXT"):
        _set(stopping, "_CUDA_CPP_DUAL_FEASIBILITY_EXT", None, undo)

    def pricing_scan(*args, **kwargs):
        _count("scan:l2sq_pricing")
        return raw_lowrank_bidir_feasibility_pricing_scan(*args, **kwargs)

    _rebind(root, bt.raw_lowrank_bidir_feasibility_pricing_scan, pricing_scan, undo)
    for mod_name, fn in (("kernels.torch_scan", "bidirectional_violation_scan"),
                         ("kernels.torch_scan", "directional_assignment"),
                         ("kernels.cpp_scan", "cpp_violation_scan")):
        orig = getattr(m(mod_name), fn)
        _rebind(root, orig, _tripwire(fn, orig), undo)

    # restricted LP
    rt = m("restricted_ot.runtime")
    base = m("_internal.lp.restricted_ot_pdlp").RestrictedOTPDLP
    lp_device = device

    class B200RestrictedOTPDLP(NativeRestrictedOTPDLP, base):
        """The library's restricted-OT PDHG as a reference RestrictedOTPDLP engine."""

        def __init__(self, **kwargs):
            NativeRestrictedOTPDLP.__init__(self, **kwargs)

        def solve_restricted(self, **kwargs):
            _count("lp:restricted_ot_pdhg")
            return NativeRestrictedOTPDLP.solve_restricted(self, **kwargs)

    original_build = rt.build_lp_backend

    def build_lp_backend(config):
        if config.solver_engine == "cupdlpx":
            _count("lp:engine")
            dev = lp_device if lp_device is not None else torch.device("cuda", torch.cuda.current_device())
            return B200RestrictedOTPDLP(device=dev,
                                        termination_norm=str(getattr(config, "lp_termination_norm", "l2")))
        return original_build(config)

    _rebind(root, original_build, build_lp_backend, undo)

    # pair costs (SDDMM)
    pairs_mod = m("costs.pairs")
    for name, kind in (("lowrank", KIND["lowrank"]), ("l1", KIND["l1"]), ("linf", KIND["linf"]),
                       ("euclidean", KIND["l2"])):
        _rebind(root, getattr(pairs_mod, f"_cost_pairs_{name}_batched"), _pair_cost_function(name, kind), undo)
    sq = pairs_mod._cost_pairs_sqeuclidean_batched
    _rebind(root, sq, _tripwire("_cost_pairs_sqeuclidean_batched", sq), undo)

    # active support: candidate filter and pruning selection
    active = m("restricted_ot.active_support").ActiveSupport

    def filter_new(self, rows, cols):
        _count("support:filter")
        return filter_new_candidate_pairs(self.keys, self.n_source, self.n_target, rows, cols)

    _set(active, "filter_new_candidate_pairs", filter_new, undo)
    cleaning = m("refinement.budgeted_pruning").DualGapCleaning

    def select_protect_new(self, current_active_support, num_to_remove, duals, n_source, current_inner_iter, *,
                           log_prefix="DualGapCleaning"):
        _count("support:prune")
        if current_inner_iter is None:
            return np.empty(0, dtype=np.int32)
        s = current_active_support
        n_source = int(n_source)
        n_total = int(duals.numel() if torch.is_tensor(duals) else np.asarray(duals).size)
        n_target = n_total - n_source
        rows, cols = s.rows, s.cols
        if s.size and (int(rows.max()) >= n_source or int(cols.max()) >= n_target):
            return np.empty(0, dtype=np.int32)  # pruning_values() -> None (active_support.py:415-416)
        return select_prune_positions(rows, cols, s.c_vec, s.x_prev, s.creation_iteration, duals, n_source,
                                      n_target, int(num_to_remove), int(current_inner_iter))

    _set(cleaning, "_select_protect_new_indices", select_protect_new, undo)

    # coarsest leaf
    coarsest = m("hierarchy.coarsest")
    warm_state_cls = m("state").WarmStartState

    def build_leaf_costs(*, leaf_inputs, tracer=None, depth_level=None, dot_scale=1.0, compute_precision="fp32"):
        _count("coarsest:cost")
        if str(compute_precision) == "fp64":
            raise NotImplementedError("hello_ot_b200 leaf costs read fp32 features (cost_precision='fp32')")
        out = {}
        dev = torch.device("cuda", torch.cuda.current_device())
        for item in leaf_inputs:
            t0 = time.perf_counter()
            ns, nt = int(item["n_source"]), int(item["n_target"])
            x, y = _dev(item["source_f"], dev, torch.float32), _dev(item["target_g"], dev, torch.float32)
            rows = torch.arange(ns, device=dev, dtype=torch.int64).repeat_interleave(nt)
            cols = torch.arange(nt, device=dev, dtype=torch.int64).repeat(ns)
            cost = pair_costs(3, x, y, rows, cols, _dev(item["source_cost"], dev, torch.float64).view(-1),
                              _dev(item["target_cost"], dev, torch.float64).view(-1), float(dot_scale)).view(ns, nt)
            out[int(item["leaf_id"])] = {"cost": cost, "cost_build_time": time.perf_counter() - t0,
                                         "batch_size": len(leaf_inputs), "device": str(dev),
                                         "backend": "hello_b200_pair_costs"}
        return out

    _rebind(root, coarsest._build_leaf_costs_pad_batch_gemm, build_leaf_costs, undo)
    metric = m("costs.metric")

    def metric_cost_matrix(source, target, cost_type, compute_precision="fp32"):
        _count("coarsest:cost")
        dev = torch.device("cuda", torch.cuda.current_device())
        x, y = _dev(source, dev, torch.float32), _dev(target, dev, torch.float32)
        ns, nt = int(x.shape[0]), int(y.shape[0])
        rows = torch.arange(ns, device=dev, dtype=torch.int64).repeat_interleave(nt)
        cols = torch.arange(nt, device=dev, dtype=torch.int64).repeat(ns)
        return pair_costs(KIND[str(cost_type)], x, y, rows, cols).view(ns, nt).cpu().numpy()

    _rebind(root, metric._metric_cost_matrix, metric_cost_matrix, undo)

    def leaf_solve(*, cost, source_f, target_g, source_mass, target_mass, tracer=None, trace_args=None,
                   precomputed_cost_build_time=0.0, cost_build_backend="precomputed", cost_build_batch_size=1,
                   cost_build_device="cpu"):
        _count("coarsest:solve")
        out = solve_leaf_from_cost(cost=cost, source_mass=np.asarray(source_mass, dtype=np.float64),
                                   target_mass=np.asarray(target_mass, dtype=np.float64))
        w = out["warm_start_state"]
        out["warm_start_state"] = warm_state_cls(rows=np.asarray(w.rows, dtype=np.int32),
                                                 cols=np.asarray(w.cols, dtype=np.int32),
                                                 x_prev=np.asarray(w.x_prev, dtype=np.float64),
                                                 dual_uv=np.asarray(w.dual_uv, dtype=np.float64),
                                                 n_source=int(np.shape(source_f)[0]),
                                                 n_target=int(np.shape(target_g)[0]))
        profile = dict(out.get("leaf_stage_profile") or {})
        profile.update({"pot_cost_build_time": float(precomputed_cost_build_time),
                        "pot_solve_time": float(out["time"]), "cost_build_backend": str(cost_build_backend),
                        "cost_build_batch_size": int(cost_build_batch_size),
                        "cost_build_device": str(cost_build_device), "leaf_solver": "hello_b200_pdhg"})
        out["leaf_stage_profile"] = profile
        return out

    _rebind(root, coarsest._solve_lowrank_leaf_with_pot_from_precomputed_cost, leaf_solve, undo)

    # support sparsification (outside the hot path): the reference's numba engine
    post = m("restricted_ot.sparsification_postprocess")
    sparsify = post.sparsify_transport_support

    def sparsify_numba(*args, **kwargs):
        if kwargs.get("engine") == "cpp_lct":
            kwargs["engine"] = "numba_lct"
        return sparsify(*args, **kwargs)

    _set(post, "sparsify_transport_support", sparsify_numba, undo)

    _STATE.update(installed=True, undo=undo, module=hello_ot)
    return hello_ot


def uninstall() -> None:
    """Restore every name install() replaced."""
    if not _STATE["installed"]:
        return
    for obj, attr, value in reversed(_STATE["undo"]):
        setattr(obj, attr, value)
    _STATE.update(installed=False, undo=[])


def installed() -> bool:
    return bool(_STATE["installed"])
