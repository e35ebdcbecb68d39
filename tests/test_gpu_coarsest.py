"""Coarsest-level dense transport (the stand-in for the reference's POT leaf solve)
against SciPy's HiGHS on the same LP: objective to the tolerance, feasible plan,
dual feasibility and complementary slackness to the tolerance."""
import numpy as np
import pytest
import scipy.sparse as sp
import torch
from scipy.optimize import linprog

pytestmark = pytest.mark.gpu


def _highs(C, a, b):
    n, m = C.shape
    rows = np.repeat(np.arange(n), m)
    cols = np.tile(np.arange(m), n)
    A = sp.vstack([sp.csr_matrix((np.ones(n * m), (rows, np.arange(n * m))), shape=(n, n * m)),
                   sp.csr_matrix((np.ones(n * m), (cols, np.arange(n * m))), shape=(m, n * m))])
    res = linprog(C.ravel(), A_eq=A, b_eq=np.concatenate([a, b]), bounds=(0, None), method="highs")
    assert res.status == 0
    return res.fun


@pytest.mark.parametrize("n,m,d,seed", [(40, 60, 2, 0), (200, 150, 3, 1), (512, 512, 8, 2)])
def test_coarsest_matches_highs(hb, cuda, n, m, d, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(n, d))
    y = rng.normal(size=(m, d)) + 0.3
    C = ((x[:, None, :] - y[None, :, :]) ** 2).sum(-1)
    a = rng.uniform(0.5, 1.5, n); a /= a.sum()
    b = rng.uniform(0.5, 1.5, m); b /= b.sum()
    out = hb.solve_leaf_from_cost(cost=C, source_mass=a, target_mass=b, tolerance=1e-9)
    assert out["termination_reason"] == "OPTIMAL"
    ref = _highs(C, a, b)
    assert out["distance"] == pytest.approx(ref, rel=2e-8)
    w = out["warm_start_state"]
    plan = np.zeros((n, m)); plan[w.rows, w.cols] = w.x_prev
    np.testing.assert_allclose(plan.sum(1), a, atol=1e-8)
    np.testing.assert_allclose(plan.sum(0), b, atol=1e-8)
    # duals: c_ij - u_i - v_j >= 0 and complementary slackness, both to the tolerance
    u, v = w.dual_uv[:n], w.dual_uv[n:]
    reduced = C - u[:, None] - v[None, :]
    assert reduced.min() >= -1e-6 * np.abs(C).max()
    assert float((w.x_prev * np.abs(reduced[w.rows, w.cols])).sum()) <= 1e-7 * abs(ref)
    assert len(out["level_summaries"]) == 1 and out["warm_start_state"].rows.dtype == np.int32


def test_coarsest_permutation_case(hb, cuda):
    """Uniform masses, n = m: the optimum is a permutation (one entry per row)."""
    rng = np.random.default_rng(7)
    n = 128
    x, y = rng.normal(size=(n, 4)), rng.normal(size=(n, 4))
    C = ((x[:, None, :] - y[None, :, :]) ** 2).sum(-1)
    a = np.full(n, 1.0 / n)
    out = hb.solve_leaf_from_cost(cost=C, source_mass=a, target_mass=a, tolerance=1e-9)
    assert out["distance"] == pytest.approx(_highs(C, a, a), rel=2e-8)
    w = out["warm_start_state"]
    big = w.x_prev > 1e-6
    assert big.sum() == n and len(set(w.rows[big])) == n and len(set(w.cols[big])) == n


@pytest.mark.parametrize("kind", ["l2^2", "l1", "linf", "l2"])
def test_leaf_cost_matrix(hb, cuda, kind):
    rng = np.random.default_rng(3)
    x = rng.normal(size=(70, 5)).astype(np.float32)
    y = rng.normal(size=(90, 5)).astype(np.float32)
    X, Y = torch.as_tensor(x, device=cuda), torch.as_tensor(y, device=cuda)
    xd, yd = x.astype(np.float64), y.astype(np.float64)
    diff = np.abs(xd[:, None, :] - yd[None, :, :])
    if kind == "l2^2":
        a, b = (xd * xd).sum(1), (yd * yd).sum(1)
        got = hb.leaf_cost_matrix(X, Y, kind, source_offset=torch.as_tensor(a, device=cuda),
                                  target_offset=torch.as_tensor(b, device=cuda))
        want = a[:, None] + b[None, :] - 2.0 * xd @ yd.T
    else:
        got = hb.leaf_cost_matrix(X, Y, kind)
        want = {"l1": diff.sum(-1), "linf": diff.max(-1), "l2": np.sqrt((diff ** 2).sum(-1))}[kind]
    assert got.shape == (70, 90) and got.dtype == torch.float64
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-5)


def test_leaf_resident_matches_host_form(hb, cuda):
    """The device-resident leaf (gpu_resident path) returns the same plan, duals and
    distance as the host-facing form, as device tensors with ascending keys i*m + j."""
    rng = np.random.default_rng(5)
    n, m = 150, 110
    x = torch.as_tensor(rng.normal(size=(n, 3)).astype(np.float32), device=cuda)
    y = torch.as_tensor(rng.normal(size=(m, 3)).astype(np.float32), device=cuda)
    C = hb.leaf_cost_matrix(x, y, "l1")
    a = torch.as_tensor(rng.uniform(0.5, 1.5, n), device=cuda)
    b = torch.as_tensor(rng.uniform(0.5, 1.5, m), device=cuda)
    a, b = a / a.sum(), b / b.sum()
    leaf = hb.solve_leaf_resident(C, a, b)
    assert leaf.keys.is_cuda and leaf.values.is_cuda and leaf.dual.is_cuda
    assert bool((leaf.keys[1:] > leaf.keys[:-1]).all())
    host = hb.solve_leaf_from_cost(cost=C.cpu().numpy(), source_mass=a.cpu().numpy(), target_mass=b.cpu().numpy())
    w = host["warm_start_state"]
    np.testing.assert_array_equal(leaf.keys.cpu().numpy(), w.rows.astype(np.int64) * m + w.cols)
    np.testing.assert_array_equal(leaf.values.cpu().numpy(), w.x_prev)
    np.testing.assert_array_equal(leaf.dual.cpu().numpy(), w.dual_uv)
    assert leaf.distance == host["distance"]
    assert leaf.distance == pytest.approx(_highs(C.cpu().numpy(), a.cpu().numpy(), b.cpu().numpy()), rel=2e-8)
