"""Pair-cost (SDDMM) and restricted-OT PDHG parity on the GPU through the C ABI."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("d", [1, 3, 4, 16, 70, 128, 256, 257, 512, 1024])
@pytest.mark.parametrize("kind", ["l1", "linf", "l2", "lowrank"])
def test_pair_costs_match_oracle(hb, cuda, oracle, d, kind):
    rng = np.random.default_rng(d)
    x = rng.normal(size=(300, d)).astype(np.float32)
    y = rng.normal(size=(200, d)).astype(np.float32)
    e = 5000
    rows, cols = rng.integers(0, 300, e), rng.integers(0, 200, e)
    a = (x.astype(np.float64) ** 2).sum(1)
    b = (y.astype(np.float64) ** 2).sum(1)
    if kind == "lowrank":
        got = hb.cost_pairs_lowrank(dict(F=x, G=y, a=a, b=b, dot_scale=2.0), rows, cols)
        exp = oracle.pair_costs("raw", x, y, rows, cols, a, b, dot_scale=2.0)
        np.testing.assert_allclose(got, exp, rtol=0, atol=1e-12 * (np.abs(a[rows]) + np.abs(b[cols]) + 1).max())
    else:
        got = hb.pair_costs_metric(source_points=x, target_points=y, rows=rows, cols=cols, cost_type=kind)
        exp = oracle.pair_costs(kind, x, y, rows, cols)
        if kind == "linf":
            assert np.array_equal(got, exp)
        else:
            np.testing.assert_allclose(got, exp, rtol=1e-13, atol=0)


@pytest.mark.parametrize("d", [128, 256, 512])
@pytest.mark.parametrize("kind", ["l1", "linf", "l2", "lowrank"])
def test_pair_costs_source_grouped(hb, cuda, oracle, d, kind):
    """Edges grouped by source row: runs of equal rows, which the kernel for d = 128, 256,
    512 serves from the source row it holds in registers."""
    rng = np.random.default_rng(d + 7)
    x = rng.normal(size=(90, d)).astype(np.float32)
    y = rng.normal(size=(300, d)).astype(np.float32)
    rows = np.sort(rng.integers(0, 90, 4000))
    cols = rng.integers(0, 300, 4000)
    a = (x.astype(np.float64) ** 2).sum(1)
    b = (y.astype(np.float64) ** 2).sum(1)
    if kind == "lowrank":
        got = hb.cost_pairs_lowrank(dict(F=x, G=y, a=a, b=b, dot_scale=2.0), rows, cols)
        exp = oracle.pair_costs("raw", x, y, rows, cols, a, b, dot_scale=2.0)
        np.testing.assert_allclose(got, exp, rtol=0, atol=1e-12 * (np.abs(a[rows]) + np.abs(b[cols]) + 1).max())
    else:
        got = hb.pair_costs_metric(source_points=x, target_points=y, rows=rows, cols=cols, cost_type=kind)
        exp = oracle.pair_costs(kind, x, y, rows, cols)
        if kind == "linf":
            assert np.array_equal(got, exp)
        else:
            np.testing.assert_allclose(got, exp, rtol=1e-13, atol=0)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("pairs_*.npz")))
def test_pair_costs_golden(hb, cuda, path):
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    for kind in ("l1", "l2", "linf"):
        got = hb.pair_costs_metric(source_points=z["x"], target_points=z["y"], rows=z["rows"], cols=z["cols"],
                                   cost_type=kind)
        np.testing.assert_allclose(got, z[kind], rtol=1e-13, atol=0)
    got = hb.cost_pairs_lowrank(dict(F=z["x"], G=z["y"], a=z["a"], b=z["b"], dot_scale=2.0), z["rows"], z["cols"])
    # the reference evaluates this in fp32
    np.testing.assert_allclose(got, z["lowrank"], rtol=1e-5, atol=1e-4)


def test_pair_costs_edges_and_errors(hb, cuda):
    x = torch.randn(10, 8, device=cuda)
    y = torch.randn(12, 8, device=cuda)
    empty = torch.empty(0, dtype=torch.int64, device=cuda)
    assert hb.pair_costs(0, x, y, empty, empty).numel() == 0
    with pytest.raises(ValueError, match="index out of range"):
        hb.pair_costs(0, x, y, torch.tensor([0, 10], device=cuda), torch.tensor([1, 2], device=cuda))
    with pytest.raises(ValueError):
        hb.pair_costs(0, x, y, torch.tensor([0, 1], device=cuda), torch.tensor([1, 12], device=cuda))


@pytest.mark.parametrize("d", [128, 256, 512])
def test_pair_costs_ring_bad_indices(hb, cuda, d):
    """The ring kernel (d = 128, 256, 512) reports an out-of-range index inside a run of one
    source row (no copy is issued for it, its slot still completes) and stays usable."""
    x = torch.randn(40, d, device=cuda)
    y = torch.randn(70, d, device=cuda)
    rows = torch.arange(40, device=cuda).repeat_interleave(5)
    cols = torch.randint(0, 70, (200,), device=cuda)
    for bad_rows, bad_cols in ((None, 70), (-1, None)):
        r, c = rows.clone(), cols.clone()
        if bad_cols is not None:
            c[37] = bad_cols
        if bad_rows is not None:
            r[101] = bad_rows
        with pytest.raises(ValueError):
            hb.pair_costs(0, x, y, r, c)
    got = hb.pair_costs(0, x, y, rows, cols).cpu().numpy()
    want = (x[rows].double() - y[cols].double()).abs().sum(1).cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-13, atol=0)


def _random_support(ns, nt, extra, seed):
    rng = np.random.default_rng(seed)
    rows = np.concatenate([np.arange(ns), rng.integers(0, ns, extra), rng.integers(0, ns, nt)])
    cols = np.concatenate([rng.integers(0, nt, ns), rng.integers(0, nt, extra), np.arange(nt)])
    key = np.unique(rows * nt + cols)
    rows, cols = key // nt, key % nt
    perm = rng.permutation(rows.size)
    wa, wb = rng.uniform(0.5, 1.5, ns), rng.uniform(0.5, 1.5, nt)
    return rows[perm], cols[perm], rng.random(rows.size) * 3, wa / wa.sum(), wb / wb.sum()


def _complete_support(ns, nt, seed):
    rng = np.random.default_rng(seed)
    rows, cols = np.repeat(np.arange(ns), nt), np.tile(np.arange(nt), ns)
    perm = rng.permutation(rows.size)
    wa, wb = rng.uniform(0.5, 1.5, ns), rng.uniform(0.5, 1.5, nt)
    return rows[perm], cols[perm], rng.random(rows.size) * 3, wa / wa.sum(), wb / wb.sum()


# (sources, targets, extra edges) of a random support; extra == -1: the complete support
# (mean degree >= 64 on both sides, or on the source side only: the warp-per-node passes)
@pytest.mark.parametrize("shape", [(30, 40, 180), (300, 400, 4000), (1000, 700, 20000), (96, 130, -1),
                                   (40, 700, -1)])
def test_pdlp_block_is_bit_exact(hb, cuda, oracle, shape):
    """One block of iterations with the same step sizes reproduces the reference
    arithmetic exactly (no restart inside the block)."""
    rows, cols, c, a, b = (_complete_support(shape[0], shape[1], 3) if shape[2] < 0
                           else _random_support(*shape, seed=shape[0]))
    F = 60
    ref = oracle.pdlp(rows, cols, c, a, b, frequency=F, iteration_limit=F, tolerance=0.0)
    solver = hb.NativeRestrictedOTPDLP(device=cuda, evaluation_frequency=F, iteration_limit=F,
                                       initial_primal_weight=ref["primal_weight"])
    got = solver.solve_restricted(rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b, tolerance=0.0)
    assert got.iterations == ref["iterations"] == F
    assert np.array_equal(got.x.cpu().numpy(), ref["x"])
    assert np.array_equal(got.y.cpu().numpy(), ref["y"])


@pytest.mark.parametrize("shape", [(30, 40, 180), (300, 400, 4000), (1000, 700, 20000)])
def test_pdlp_converges_like_oracle(hb, cuda, oracle, shape):
    rows, cols, c, a, b = _random_support(*shape, seed=shape[1])
    ref = oracle.pdlp(rows, cols, c, a, b, frequency=200, tolerance=1e-7)
    got = hb.NativeRestrictedOTPDLP(device=cuda).solve_restricted(rows=rows, cols=cols, costs=c, source_mass=a,
                                                                   target_mass=b, tolerance=1e-7)
    assert ref["termination_reason"] == got.termination_reason == "OPTIMAL"
    assert got.obj_val == pytest.approx(ref["obj_val"], rel=1e-6)
    assert got.primal_feas < 1e-7 and got.dual_feas < 1e-7 and got.gap < 1e-7
    assert abs(got.iterations - ref["iterations"]) <= 2 * 200


@pytest.mark.parametrize("shape", [(300, 400, 4000), (1000, 700, 20000)])
def test_pdlp_linf_termination(hb, cuda, shape):
    """termination_norm="linf" (the native engine's cuPDLPx rule): at termination the
    reported residuals are the max-norm residuals of the returned iterate relative to
    1 + ||b||_inf and 1 + ||c||_inf, below the tolerance; the L2 ones are reported beside."""
    rows, cols, c, a, b = _random_support(*shape, seed=shape[0] + 1)
    n, m = len(a), len(b)
    tol = 1e-7
    res = {}
    for norm in ("l2", "linf"):
        solver = hb.NativeRestrictedOTPDLP(device=cuda, termination_norm=norm)
        res[norm] = solver.solve_restricted(rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b,
                                            tolerance=tol)
        assert res[norm].termination_reason == "OPTIMAL"
        assert res[norm].solver_diag["termination_norm"] == norm
    r = res["linf"]
    x, y = r.x.cpu().numpy(), r.y.cpu().numpy()
    masses = np.concatenate((a, b))
    sums = np.concatenate((np.bincount(rows, x, minlength=n), np.bincount(cols, x, minlength=m)))
    primal = np.abs(sums - masses).max() / (1.0 + np.abs(masses).max())
    dual = np.maximum(y[rows] + y[n + cols] - c, 0.0).max() / (1.0 + np.abs(c).max())
    assert r.primal_feas == pytest.approx(primal, rel=1e-9, abs=1e-16) and r.primal_feas < tol
    assert r.dual_feas == pytest.approx(dual, rel=1e-9, abs=1e-16) and r.dual_feas < tol
    d = r.solver_diag
    assert d["termination_rel_primal_res"] == r.primal_feas
    l2p = np.sqrt(((sums - masses) ** 2).sum()) / (1.0 + np.sqrt((masses ** 2).sum()))
    assert d["algorithm_rel_primal_res_l2"] == pytest.approx(l2p, rel=1e-9, abs=1e-16)
    assert r.obj_val == pytest.approx(res["l2"].obj_val, rel=1e-6)
    with pytest.raises(ValueError):
        hb.NativeRestrictedOTPDLP(device=cuda, termination_norm="l1")


def _hub_support(ns, nt, seed):
    """A transport-feasible support with one source joined to every target (a node whose
    edges span many stages of the fused pass) and degree-1 or 2 elsewhere."""
    rng = np.random.default_rng(seed)
    rows = np.concatenate([np.zeros(nt, dtype=np.int64), np.arange(ns), rng.integers(0, ns, ns // 2)])
    cols = np.concatenate([np.arange(nt), rng.integers(0, nt, ns), rng.integers(0, nt, ns // 2)])
    key = np.unique(rows * nt + cols)
    rows, cols = key // nt, key % nt
    perm = rng.permutation(rows.size)
    wa, wb = rng.uniform(0.5, 1.5, ns), rng.uniform(0.5, 1.5, nt)
    return rows[perm], cols[perm], rng.random(rows.size) * 3, wa / wa.sum(), wb / wb.sum()


def _sparse_support(ns, nt, seed):
    """Degree 1-2 on both sides (a ring plus a few chords): tiles of few edges, so one stage of
    the fused pass spans many tiles."""
    rng = np.random.default_rng(seed)
    k = max(ns, nt)
    rows = np.concatenate([np.arange(k) % ns, (np.arange(k) + 1) % ns, rng.integers(0, ns, k // 8)])
    cols = np.concatenate([np.arange(k) % nt, np.arange(k) % nt, rng.integers(0, nt, k // 8)])
    key = np.unique(rows * nt + cols)
    rows, cols = key // nt, key % nt
    perm = rng.permutation(rows.size)
    wa, wb = rng.uniform(0.5, 1.5, ns), rng.uniform(0.5, 1.5, nt)
    return rows[perm], cols[perm], rng.random(rows.size) * 3, wa / wa.sum(), wb / wb.sum()


@pytest.mark.parametrize("kind", ["hub", "sparse"])
def test_pdlp_block_is_bit_exact_irregular(hb, cuda, oracle, kind):
    """One block of iterations bit-exact on irregular supports: a node with thousands of edges
    among degree-1/2 nodes, and degree 1-2 everywhere (stages spanning many tiles)."""
    rows, cols, c, a, b = _hub_support(6000, 5000, 3) if kind == "hub" else _sparse_support(20000, 17000, 4)
    assert rows.size < 64 * min(len(a), len(b))  # both sides sparse: the fused pass
    F = 40
    ref = oracle.pdlp(rows, cols, c, a, b, frequency=F, iteration_limit=F, tolerance=0.0)
    solver = hb.NativeRestrictedOTPDLP(device=cuda, evaluation_frequency=F, iteration_limit=F,
                                       initial_primal_weight=ref["primal_weight"])
    got = solver.solve_restricted(rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b, tolerance=0.0)
    assert got.iterations == ref["iterations"] == F
    assert np.array_equal(got.x.cpu().numpy(), ref["x"])
    assert np.array_equal(got.y.cpu().numpy(), ref["y"])


def test_pdlp_block_is_bit_exact_large_tiles(hb, cuda, oracle):
    """Above about 300k nodes per side the fused pass takes 256-node tiles (64 below, which
    the smaller cases cover): one block of iterations is bit-exact there as well."""
    rows, cols, c, a, b = _random_support(320000, 310000, 1_200_000, seed=9)
    F = 20
    ref = oracle.pdlp(rows, cols, c, a, b, frequency=F, iteration_limit=F, tolerance=0.0)
    solver = hb.NativeRestrictedOTPDLP(device=cuda, evaluation_frequency=F, iteration_limit=F,
                                       initial_primal_weight=ref["primal_weight"])
    got = solver.solve_restricted(rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b, tolerance=0.0)
    assert got.iterations == ref["iterations"] == F
    assert np.array_equal(got.x.cpu().numpy(), ref["x"])
    assert np.array_equal(got.y.cpu().numpy(), ref["y"])


@pytest.mark.parametrize("shape", [(30, 40, 180), (1000, 700, 20000), (3000, 2500, 60000)])
def test_pdlp_atomic_sums_converge_like_oracle(hb, cuda, oracle, shape):
    """Atomic node sums change the summation order (so the last bits) but not the solve:
    same termination, objective within the tolerance, and one block of iterations
    within round-off of the ordered sums."""
    rows, cols, c, a, b = _random_support(*shape, seed=shape[0] + 7)
    ref = oracle.pdlp(rows, cols, c, a, b, frequency=200, tolerance=1e-7)
    got = hb.NativeRestrictedOTPDLP(device=cuda, deterministic=False).solve_restricted(
        rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b, tolerance=1e-7)
    assert ref["termination_reason"] == got.termination_reason == "OPTIMAL"
    assert got.obj_val == pytest.approx(ref["obj_val"], rel=1e-6)
    assert got.primal_feas < 1e-7 and got.dual_feas < 1e-7 and got.gap < 1e-7
    F = 60
    blk = oracle.pdlp(rows, cols, c, a, b, frequency=F, iteration_limit=F, tolerance=0.0)
    fast = hb.NativeRestrictedOTPDLP(device=cuda, evaluation_frequency=F, iteration_limit=F, deterministic=False,
                                     initial_primal_weight=blk["primal_weight"])
    out = fast.solve_restricted(rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b, tolerance=0.0)
    np.testing.assert_allclose(out.x.cpu().numpy(), blk["x"], rtol=1e-9, atol=1e-12 * np.abs(blk["x"]).max())
    np.testing.assert_allclose(out.y.cpu().numpy(), blk["y"], rtol=1e-9, atol=1e-12 * np.abs(blk["y"]).max())


@pytest.mark.parametrize("shape", [(96, 130), (40, 700), (300, 20)])
def test_pdlp_tree_sums(hb, cuda, oracle, shape):
    """summation="tree" on complete supports: one block within round-off of the
    reference's ordered sums, bit-reproducible from run to run, and the same solve."""
    rows, cols, c, a, b = _complete_support(*shape, seed=11)
    F = 60
    blk = oracle.pdlp(rows, cols, c, a, b, frequency=F, iteration_limit=F, tolerance=0.0)
    outs = []
    for _ in range(2):
        s = hb.NativeRestrictedOTPDLP(device=cuda, evaluation_frequency=F, iteration_limit=F, summation="tree",
                                      initial_primal_weight=blk["primal_weight"])
        outs.append(s.solve_restricted(rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b, tolerance=0.0))
    assert torch.equal(outs[0].x, outs[1].x) and torch.equal(outs[0].y, outs[1].y)
    np.testing.assert_allclose(outs[0].x.cpu().numpy(), blk["x"], rtol=1e-9, atol=1e-12 * np.abs(blk["x"]).max())
    np.testing.assert_allclose(outs[0].y.cpu().numpy(), blk["y"], rtol=1e-9, atol=1e-12 * np.abs(blk["y"]).max())
    ref = oracle.pdlp(rows, cols, c, a, b, frequency=200, tolerance=1e-8)
    got = hb.NativeRestrictedOTPDLP(device=cuda, summation="tree").solve_restricted(
        rows=rows, cols=cols, costs=c, source_mass=a, target_mass=b, tolerance=1e-8)
    assert ref["termination_reason"] == got.termination_reason == "OPTIMAL"
    assert got.obj_val == pytest.approx(ref["obj_val"], rel=1e-7)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("pdlp_*.npz")))
def test_pdlp_golden(hb, cuda, path):
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    x0 = z["x0"] if z["x0"].size else None
    y0 = z["y0"] if z["y0"].size else None
    got = hb.NativeRestrictedOTPDLP(device=cuda, evaluation_frequency=20, iteration_limit=200000).solve_restricted(
        rows=z["rows"], cols=z["cols"], costs=z["costs"], source_mass=z["source_mass"], target_mass=z["target_mass"],
        warm_start_primal=x0, warm_start_dual=y0, tolerance=1e-7)
    meta = z["cpp_meta"]
    assert got.termination_reason == "OPTIMAL"
    assert got.obj_val == pytest.approx(meta[2], rel=1e-6, abs=1e-9)
    np.testing.assert_allclose(got.x.cpu().numpy(), z["cpp_x"], atol=1e-5)


def test_pdlp_input_errors(hb, cuda):
    rows, cols = np.array([0, 0, 1, 1]), np.array([0, 1, 0, 1])
    costs = np.array([0.0, 2.0, 1.0, 0.0])
    s = hb.NativeRestrictedOTPDLP(device=cuda)
    with pytest.raises(ValueError, match="equal source and target total mass"):
        s.solve_restricted(rows=rows, cols=cols, costs=costs, source_mass=[0.4, 0.6], target_mass=[0.4, 0.5])
    with pytest.raises(ValueError, match="out of bounds"):
        s.solve_restricted(rows=[0, 0, 1, 2], cols=cols, costs=costs, source_mass=[0.4, 0.6], target_mass=[0.5, 0.5])
    with pytest.raises(ValueError, match="must not be empty"):
        s.solve_restricted(rows=[], cols=[], costs=[], source_mass=[0.4, 0.6], target_mass=[0.5, 0.5])
    r = s.solve_restricted(rows=rows, cols=cols, costs=costs, source_mass=[0.4, 0.6], target_mass=[0.5, 0.5],
                           tolerance=1e-7)
    assert r.success and r.obj_val == pytest.approx(0.1, abs=2e-6)
    with pytest.raises(ValueError, match="summation"):
        hb.NativeRestrictedOTPDLP(device=cuda, summation="pairwise")
    bad = hb.NativeRestrictedOTPDLP(device=cuda)
    bad.summation = "invalid"
    hb.pdlp.SUMMATION["invalid"] = 3  # an out-of-range order reaches the C ABI check
    try:
        with pytest.raises(ValueError, match="HB_PDLP_SUMS"):
            bad.solve_restricted(rows=rows, cols=cols, costs=costs, source_mass=[0.4, 0.6], target_mass=[0.5, 0.5])
    finally:
        del hb.pdlp.SUMMATION["invalid"]


def test_sharded_pair_costs_single_rank(hb, cuda):
    """World size 1 (no process group): the sharded pair costs are the kernel's."""
    from hello_ot_b200.sharded import ShardedPairCosts
    rng = np.random.default_rng(2)
    x = torch.as_tensor(rng.normal(size=(300, 40)).astype(np.float32), device=cuda)
    y = torch.as_tensor(rng.normal(size=(500, 40)).astype(np.float32), device=cuda)
    a, b = (x.double() ** 2).sum(1), (y.double() ** 2).sum(1)
    rows = torch.as_tensor(rng.integers(0, 300, 4000), device=cuda)
    cols = torch.as_tensor(rng.integers(0, 500, 4000), device=cuda)
    got = ShardedPairCosts().costs(rows, cols, x, y, row_offset=0, a_block=a, b=b)
    assert torch.equal(got, hb.pair_costs(3, x, y, rows, cols, a=a, b=b, dot_scale=2.0))
