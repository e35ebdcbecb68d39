"""CPU checks of the hello_ot plug-in (no kernel runs): which reference names it
binds, that it restores them, and that the bound native backend refuses to run
without CUDA instead of falling back.  The reference package is the unmodified
pip install in baseline/_ref."""
from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

import refpkg

pytestmark = pytest.mark.skipif(not refpkg.available(), reason="reference package not installed in baseline/_ref")


@pytest.fixture()
def bound(hb):
    hello_ot = refpkg.import_reference()
    from hello_ot_b200 import plugin
    plugin.install(hello_ot)
    yield hello_ot, plugin
    plugin.uninstall()


def _m(name):
    return importlib.import_module(f"hello_ot.{name}")


def test_install_binds_the_native_hot_path(bound):
    hello_ot, plugin = bound
    gs = _m("kernels.generic_scan")
    assert gs.ScanExtension is plugin.BoundScanExtension
    assert _m("kernels.norm_cost_scan")._require_norm_cost_scan_ext().__class__ is plugin.BoundScanExtension
    bt = _m("kernels.bilinear_topk")
    assert isinstance(bt._load_extension(), plugin.BoundScanExtension)
    assert _m("refinement.dual_feasibility").raw_lowrank_bidir_feasibility_pricing_scan.__module__ == plugin.__name__
    solver_mod = _m("_internal.core.solver")
    for name in ("lowrank", "l1", "linf", "euclidean"):
        fn = getattr(solver_mod, f"_cost_pairs_{name}_batched")
        assert fn.__module__ == plugin.__name__, name
        assert getattr(_m("costs.pairs"), f"_cost_pairs_{name}_batched") is fn
    assert _m("restricted_ot.active_support").ActiveSupport.filter_new_candidate_pairs.__module__ == plugin.__name__
    assert _m("refinement.budgeted_pruning").DualGapCleaning._select_protect_new_indices.__module__ == plugin.__name__
    assert _m("hierarchy.coarsest")._solve_lowrank_leaf_with_pot_from_precomputed_cost.__module__ == plugin.__name__
    assert _m("costs.metric")._solve_lowrank_leaf_with_pot_from_precomputed_cost.__module__ == plugin.__name__
    with pytest.raises(RuntimeError, match="was requested"):
        _m("_source_build").load_native_module("hello_ot_native.hierot_generic_cost_ext")
    assert plugin.routes(reset=True).get("reference:native_module:hello_ot_native.hierot_generic_cost_ext") == 1


def test_lp_engine_is_a_restricted_ot_pdlp(bound):
    hello_ot, plugin = bound
    rt = _m("restricted_ot.runtime")
    base = _m("_internal.lp.restricted_ot_pdlp").RestrictedOTPDLP

    class Config:
        solver_engine = "cupdlpx"

    plugin.uninstall()
    plugin.install(hello_ot, device=torch.device("cuda", 0))  # an explicit device: no CUDA call here
    engine = rt.build_lp_backend(Config())
    assert isinstance(engine, base)
    from hello_ot_b200 import NativeRestrictedOTPDLP
    assert isinstance(engine, NativeRestrictedOTPDLP)


def test_uninstall_restores_every_name(hb):
    hello_ot = refpkg.import_reference()
    from hello_ot_b200 import plugin
    gs = _m("kernels.generic_scan")
    before = (gs.ScanExtension, _m("_internal.core.solver")._cost_pairs_lowrank_batched,
              _m("restricted_ot.active_support").ActiveSupport.filter_new_candidate_pairs,
              _m("restricted_ot.runtime").build_lp_backend, _m("_source_build").load_native_module)
    plugin.install(hello_ot)
    plugin.uninstall()
    after = (gs.ScanExtension, _m("_internal.core.solver")._cost_pairs_lowrank_batched,
             _m("restricted_ot.active_support").ActiveSupport.filter_new_candidate_pairs,
             _m("restricted_ot.runtime").build_lp_backend, _m("_source_build").load_native_module)
    assert before == after
    assert not plugin.installed()


def test_bound_native_solve_needs_cuda(bound, monkeypatch):
    hello_ot, plugin = bound
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    x = np.random.default_rng(0).normal(size=(16, 3)).astype(np.float32)
    with pytest.raises(RuntimeError, match="CUDA"):
        hello_ot.solve(x, x + 1, options=hello_ot.SolverOptions(backend="native", verbose="off"))


def test_pot_standin_matches_exact_small_lp():
    """The ot.emd stand-in used by the reference's CPU runs: a 3 x 3 assignment with a
    known optimum, and duals that certify it (c_ij - u_i - v_j >= 0, equality on the plan)."""
    from oracle import pot_emd
    M = np.array([[4.0, 1.0, 3.0], [2.0, 0.0, 5.0], [3.0, 2.0, 2.0]])
    a = b = np.full(3, 1 / 3)
    plan, log = pot_emd.emd(a, b, M, log=True)
    assert abs(log["cost"] - 5.0 / 3.0) < 1e-12
    red = M - log["u"][:, None] - log["v"][None, :]
    assert red.min() > -1e-9
    assert np.all(np.abs(red[plan > 1e-12]) < 1e-9)
    assert abs(a @ log["u"] + b @ log["v"] - log["cost"]) < 1e-9
