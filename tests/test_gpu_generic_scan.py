"""Module-level scan entry points (the reference's generic_scan.bidirectional /
directional / certificate_only, as the gpu_resident solver calls them) against the
ScanExtension methods they route to and against fp64 brute force, including the l2^2
rank-2 perturbation passed as raw_extras."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(v, dev, dt=torch.float64):
    return torch.as_tensor(v, dtype=dt, device=dev)


def _problem(q, n, d, seed, dev):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (rng.normal(size=(n, d)) + 0.2).astype(np.float32)
    nx, ny = (x.astype(np.float64) ** 2).sum(1), (y.astype(np.float64) ** 2).sum(1)
    f = 0.5 * nx + rng.normal(size=q) * 2
    g = 0.5 * ny + rng.normal(size=n) * 2
    return x, y, nx, ny, f, g


def _same_certificate(a, b):
    """The certificate-only scan (k = 0) and the pricing scan agree up to the order of the
    fp32 products behind the cost terms (their roles are exchanged in the k = 0 schedule):
    sums and maxima to 1e-7 relative, counts to the pairs at zero."""
    for j in range(4):
        assert float(a[j]) == pytest.approx(float(b[j]), rel=1e-7)
    assert abs(int(a[4]) - int(b[4])) <= 2


def _extras(q, n, sigma, seed):
    """The gpu_resident l2^2 perturbation columns (gpu_resident/solver.py:205-210 form)."""
    s = np.sqrt(0.25 * sigma)
    sa = np.arange(q) * 12.9898 + seed * 0.001
    ta = np.arange(n) * 78.233
    ex = (s * np.stack((np.sin(sa), np.cos(sa)), 1)).astype(np.float32)
    ey = (-s * np.stack((np.cos(ta), np.sin(ta)), 1)).astype(np.float32)
    return ex, ey


def test_bidirectional_raw_matches_scan_extension(hb, cuda):
    gs = hb.generic_scan
    x, y, nx, ny, f, g = _problem(300, 500, 24, 1, cuda)
    X, Y = _t(x, cuda, torch.float32), _t(y, cuda, torch.float32)
    NX, NY, F, G = (_t(v, cuda) for v in (nx, ny, f, g))
    out = gs.bidirectional(X, Y, F, G, 8, 3, raw_costs=(NX, NY), raw_biases=(F - NX, G - NY))
    ref = hb.ScanExtension().fused_bidir_topk_stats_raw(X, Y, NX, NY, F - NX, G - NY, 8192, 65536, 256, 8, True,
                                                        True, False, 0, 2.0)
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1].long())
    assert torch.equal(out[2], ref[2]) and torch.equal(out[3], ref[3].long())
    assert out[1].dtype == torch.int64 and out[8].dtype == torch.int64
    # compute_precision=1 (fp64): the exact fp64 lists whatever exact says
    out64 = gs.bidirectional(X, Y, F, G, 8, 3, raw_costs=(NX, NY), raw_biases=(F - NX, G - NY), compute_precision=1,
                             exact=False)
    assert all(torch.equal(u, v) for u, v in zip(out64[:4], out[:4]))
    _same_certificate(gs.certificate_only(X, Y, F, G, 3, raw_costs=(NX, NY)), out[4:])
    assert float(gs.certificate_only(X, Y, F, G, 3, raw_costs=(NX, NY), compute_denominator=False)[1]) == 0.0


@pytest.mark.parametrize("dot_scale", [2.0, 1.0])
def test_bidirectional_raw_extras_brute_force(hb, cuda, dot_scale):
    gs = hb.generic_scan
    q, n, sigma = 257, 333, 3.0
    x, y, nx, ny, f, g = _problem(q, n, 16, 2, cuda)
    ex, ey = _extras(q, n, sigma, 7)
    X, Y, EX, EY = (_t(v, cuda, torch.float32) for v in (x, y, ex, ey))
    NX, NY, F, G = (_t(v, cuda) for v in (nx, ny, f, g))
    if dot_scale == 1.0:  # the cost then carries 1 <x, y>: shift the norms accordingly
        nx, ny = 0.5 * nx, 0.5 * ny
        NX, NY = _t(nx, cuda), _t(ny, cuda)
    rv, ri, cv, ci, num, den, mx, cmax, cnt = gs.bidirectional(
        X, Y, F, G, 4, 3, raw_costs=(NX, NY), raw_biases=(F - NX, G - NY), dot_scale=dot_scale,
        raw_extras=(EX, EY, sigma))
    xd, yd, exd, eyd = (v.astype(np.float64) for v in (x, y, ex, ey))
    cost = nx[:, None] + ny[None, :] - dot_scale * xd @ yd.T - 2.0 * exd @ eyd.T + 0.5 * sigma
    score = f[:, None] + g[None, :] - cost
    tol = 1e-5 * (np.abs(cost).max() + np.abs(score).max())
    ri_, ci_ = ri.cpu().numpy(), ci.cpu().numpy()
    np.testing.assert_allclose(rv.cpu().numpy(), score[np.arange(q)[:, None], ri_], atol=tol)
    np.testing.assert_allclose(cv.cpu().numpy(), score[ci_, np.arange(n)[:, None]], atol=tol)
    # the reported top-1 is the true best up to the fp32 product error
    assert np.all(rv.cpu().numpy()[:, 0] >= score.max(1) - 2 * tol)
    pos = np.maximum(score, 0.0)
    assert float(num) == pytest.approx((pos ** 2).sum(), rel=1e-4)
    assert float(den) == pytest.approx((cost ** 2).sum(), rel=1e-6)
    assert float(mx) == pytest.approx(pos.max(), abs=tol)
    assert float(cmax) == pytest.approx(np.abs(cost).max(), rel=1e-6)
    assert abs(int(cnt) - int((score > 0).sum())) <= max(2, int(0.001 * score.size))


def test_directional_raw_and_norm(hb, cuda):
    gs = hb.generic_scan
    x, y, nx, ny, f, g = _problem(200, 300, 12, 3, cuda)
    X, Y = _t(x, cuda, torch.float32), _t(y, cuda, torch.float32)
    NX, G = _t(nx, cuda), _t(g - ny, cuda)
    v, i = gs.directional(X, Y, G, 8, 3, query_bias=-NX)
    rv, ri = hb.ScanExtension().initialization_directional_topk_raw(X, Y, -NX, G, 2048, 8192, 8, 2.0)
    assert torch.equal(v, rv) and torch.equal(i, ri.long())
    vm, im = gs.directional(X, Y, G, 8, 3, query_bias=-NX, minimum=True)
    assert torch.equal(vm, -rv) and torch.equal(im, i)
    Gn = _t(np.random.default_rng(4).normal(size=300) * 5, cuda)
    s, si, st = gs.directional(X, Y, Gn, 4, 0, collect_statistics=True)
    c, ci, cst = hb.ScanExtension().fused_gcost_topk(X, Y, Gn, 4, "l1", collect_statistics=True)
    assert torch.equal(-s, c) and torch.equal(si, ci) and torch.equal(st, cst)
    sm, _ = gs.directional(X, Y, Gn, 4, 0, minimum=True)
    assert torch.equal(sm, c)


def test_bidirectional_norm_with_perturbation(hb, cuda):
    gs = hb.generic_scan
    rng = np.random.default_rng(9)
    q, n = 150, 170
    X = _t(rng.normal(size=(q, 5)), cuda, torch.float32)
    Y = _t(rng.normal(size=(n, 5)), cuda, torch.float32)
    F, G = _t(rng.normal(size=q), cuda), _t(rng.normal(size=n), cuda)
    qi = torch.arange(q, device=cuda, dtype=torch.int64) * 3
    di = torch.arange(n, device=cuda, dtype=torch.int64) * 5 + 1
    coeffs = torch.tensor(hb.perturb.index_hash_coefficients(11), dtype=torch.int64)
    pert = (qi, di, 0.25, 11, 1, True, coeffs)
    out = gs.bidirectional(X, Y, F, G, 8, 0, perturbation=pert)
    ref = hb.ScanExtension().fused_gcost_bidir_certificate(X, Y, F, G, 8, "l1", qi, di, 0.25, 11, 1, True, coeffs)
    for a, b in zip(out, ref):
        assert torch.equal(a, b)
    _same_certificate(gs.certificate_only(X, Y, F, G, 0, perturbation=pert), out[4:])
    with pytest.raises(ValueError, match="raw pricing"):
        gs.bidirectional(X, Y, F, G, 8, 3, raw_costs=(F, G), raw_biases=(F, G), perturbation=pert)
    with pytest.raises(NotImplementedError):
        gs.bidirectional(X, Y, F, G, 8, 0, compute_precision=1)
