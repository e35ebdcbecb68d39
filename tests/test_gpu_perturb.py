"""Perturbed norm costs on the GPU (the reference's sigma > 0 path of its fused
norm kernels).  Index-hash noise is fp32 arithmetic with every step rounded, so
perturbed pair costs match the reference's fixture to fp64 rounding of the
distance, and perturbed scans match a brute force over the oracle's fp32
distances plus the oracle's noise bit for bit."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _t(v, dt, dev):
    return torch.as_tensor(v, dtype=dt, device=dev)


def _load():
    with np.load(GOLDEN / "perturb.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("kind", ["l1", "l2", "linf"])
def test_perturbed_pair_costs_golden(hb, cuda, kind):
    z = _load()
    ext = hb.ScanExtension()
    got = ext.fused_gcost_pairs(_t(z["x"], torch.float32, cuda), _t(z["y"], torch.float32, cuda),
                                _t(z["rows"], torch.int64, cuda), _t(z["cols"], torch.int64, cuda), kind,
                                _t(z["si"], torch.int64, cuda), _t(z["ti"], torch.int64, cuda), 0.05, int(z["seed"]),
                                1, _t(z["coeffs"], torch.int64, cuda))
    np.testing.assert_allclose(got.cpu().numpy(), z[f"pairs_{kind}"], rtol=1e-13, atol=0)
    # the dict form of h/costs/metric.py:85
    got2 = hb.pair_costs_metric(source_points=z["x"], target_points=z["y"], rows=z["rows"], cols=z["cols"],
                                cost_type=kind, perturbation={"mode": "full_cost_perturb", "sigma": 0.05,
                                                              "seed": int(z["seed"]), "noise": "index_hash",
                                                              "source_global_index": z["si"],
                                                              "target_global_index": z["ti"]})
    assert np.array_equal(got2, got.cpu().numpy())


def _brute(oracle, kind, x, y, f, g, si, ti, sigma, seed, mode, coeffs, k, row_is_source=True):
    """Perturbed fp32-model costs of all pairs, scores (g - c') + f, exact top-k lists and stats."""
    q, n = len(x), len(y)
    v, i, _, _, _ = oracle.scan(kind, x, y, np.full(q, -0.0), np.zeros(n), rk=n, ck=0, exact=False)
    cost = np.empty((q, n))
    np.put_along_axis(cost, i, -v, axis=1)  # score (0 - c) + (-0) = -c
    rr, cc = np.meshgrid(np.arange(q), np.arange(n), indexing="ij")
    src, tgt = (si[rr], ti[cc]) if row_is_source else (ti[cc], si[rr])
    cp = cost + oracle.noise(src.ravel(), tgt.ravel(), sigma, seed, mode, coeffs).reshape(q, n)
    s = (g[None, :] - cp) + f[:, None]
    order_r = np.lexsort((np.broadcast_to(np.arange(n), (q, n)), -s), axis=1)[:, :k]
    order_c = np.lexsort((np.broadcast_to(np.arange(q)[:, None], (q, n)), -s), axis=0)[:k, :].T
    rv, cv = np.take_along_axis(s, order_r, 1), np.take_along_axis(s.T, order_c, 1)
    pos = s > 0
    stats = np.array([np.sum(np.where(pos, s * s, 0)), np.sum(cp * cp), np.max(np.where(pos, s, 0)),
                      np.max(np.abs(cp)), np.sum(pos)])
    return rv, order_r, cv, order_c, stats


@pytest.mark.parametrize("kind", ["l1", "l2", "linf"])
@pytest.mark.parametrize("q,n,d,k,passes", [(90, 70, 5, 4, None), (130, 150, 3, 8, 2), (40, 33, 12, 16, None)])
def test_perturbed_norm_scan_bit_exact(hb, cuda, oracle, kind, q, n, d, k, passes):
    rng = np.random.default_rng(q + n + d)
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (x[rng.integers(0, q, n)] + 0.4 * rng.normal(size=(n, d))).astype(np.float32)
    f = rng.normal(size=q) * d * 0.3
    g = rng.normal(size=n) * d * 0.3 + d
    si, ti = rng.permutation(10 ** 6)[:q], rng.permutation(10 ** 6)[:n]
    seed, sigma = 77, 0.25 * d
    from hello_ot_b200.perturb import index_hash_coefficients, make_perturbation
    coeffs = np.array(index_hash_coefficients(seed))
    X, Y = _t(x, torch.float32, cuda), _t(y, torch.float32, cuda)
    pert = make_perturbation(X, Y, _t(si, torch.int64, cuda), _t(ti, torch.int64, cuda), sigma, seed, 1, True, None)
    rv, ri, cv, ci, st = (t.cpu().numpy() for t in hb.norm_scan(X, Y, _t(f, torch.float64, cuda),
                                                                _t(g, torch.float64, cuda), k, kind, passes=passes,
                                                                perturbation=pert))
    ev, ei, fv, fi, es = _brute(oracle, kind, x, y, f, g, si, ti, sigma, seed, 1, coeffs, k)
    kr, kc = min(k, n), min(k, q)
    assert np.array_equal(ri[:, :kr], ei[:, :kr]) and np.array_equal(rv[:, :kr], ev[:, :kr])
    assert np.array_equal(ci[:, :kc], fi[:, :kc]) and np.array_equal(cv[:, :kc], fv[:, :kc])
    assert st[2] == es[2] and st[3] == es[3] and st[4] == es[4]
    np.testing.assert_allclose(st[:2], es[:2], rtol=1e-12)


def test_perturbed_topk_and_certificate(hb, cuda, oracle):
    """fused_gcost_topk (c' - g ascending) and fused_gcost_certificate with the noise."""
    rng = np.random.default_rng(5)
    q, n, d, k = 60, 80, 4, 8
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = rng.normal(size=(n, d)).astype(np.float32)
    f, g = rng.normal(size=q), rng.normal(size=n) * 3
    si, ti = rng.permutation(50000)[:q], rng.permutation(50000)[:n]
    from hello_ot_b200.perturb import index_hash_coefficients
    coeffs = np.array(index_hash_coefficients(9))
    args = dict(query_global_index=_t(si, torch.int64, cuda), database_global_index=_t(ti, torch.int64, cuda),
                sigma=0.5, seed=9, perturb_mode=1, index_hash_coeffs=_t(coeffs, torch.int64, cuda))
    ext = hb.ScanExtension()
    X, Y = _t(x, torch.float32, cuda), _t(y, torch.float32, cuda)
    vals, idx = ext.fused_gcost_topk(X, Y, _t(g, torch.float64, cuda), k, "l1", **args)
    ev, ei, _, _, _ = _brute(oracle, "l1", x, y, np.full(q, -0.0), g, si, ti, 0.5, 9, 1, coeffs, k)
    assert np.array_equal(idx.cpu().numpy(), ei) and np.array_equal(vals.cpu().numpy(), -ev)
    cert = ext.fused_gcost_certificate(X, Y, _t(f, torch.float64, cuda), _t(g, torch.float64, cuda), "l1", **args)
    es = _brute(oracle, "l1", x, y, f, g, si, ti, 0.5, 9, 1, coeffs, 1)[4]
    assert float(cert[2]) == es[2] and float(cert[3]) == es[3] and int(cert[4]) == es[4]
    np.testing.assert_allclose([float(cert[0]), float(cert[1])], es[:2], rtol=1e-12)


def test_perturbed_scan_golden(hb, cuda):
    """The reference's torch scan adds the noise in fp32 tiles: candidate pairs agree
    except within that rounding, the certificate within it."""
    z = _load()
    ext = hb.ScanExtension()
    out = ext.fused_gcost_bidir_certificate(_t(z["x"], torch.float32, cuda), _t(z["y"], torch.float32, cuda),
                                            _t(z["f"], torch.float64, cuda), _t(z["g"], torch.float64, cuda), 4, "l1",
                                            _t(z["si"], torch.int64, cuda), _t(z["ti"], torch.int64, cuda), 0.3,
                                            int(z["seed"]), 1, True, _t(z["coeffs"], torch.int64, cuda))
    rv, ri, cv, ci = (t.cpu().numpy() for t in out[:4])
    rows = np.concatenate([np.repeat(np.arange(len(rv)), 4)[(rv > 0).ravel()], ci[cv > 0]])
    cols = np.concatenate([ri[rv > 0], np.repeat(np.arange(len(cv)), 4)[(cv > 0).ravel()]])
    ours = set(zip(rows.tolist(), cols.tolist()))
    ref = set(zip(z["scan_rows"].tolist(), z["scan_cols"].tolist()))
    assert len(ours ^ ref) <= max(2, len(ref) // 50)
    feas = np.sqrt(float(out[4])) / (1 + np.sqrt(float(out[5])))
    assert feas == pytest.approx(float(z["dual_feasibility"]), rel=1e-5)


def test_rank2_noise_in_range_and_consistent(hb, cuda):
    """rank2 (the reference's fused kernels use __sinf): scan and pair costs add the
    same noise, within [0, sigma]."""
    rng = np.random.default_rng(8)
    x = rng.normal(size=(20, 3)).astype(np.float32)
    y = rng.normal(size=(30, 3)).astype(np.float32)
    si, ti = np.arange(20) * 7, np.arange(30) * 11
    X, Y = _t(x, torch.float32, cuda), _t(y, torch.float32, cuda)
    ext = hb.ScanExtension()
    rows = np.repeat(np.arange(20), 30)
    cols = np.tile(np.arange(30), 20)
    base = ext.fused_gcost_pairs(X, Y, _t(rows, torch.int64, cuda), _t(cols, torch.int64, cuda), "linf")
    pert = ext.fused_gcost_pairs(X, Y, _t(rows, torch.int64, cuda), _t(cols, torch.int64, cuda), "linf",
                                 _t(si, torch.int64, cuda), _t(ti, torch.int64, cuda), 0.5, 3, 0)
    noise = (pert - base).cpu().numpy()
    assert np.all(noise >= 0) and np.all(noise <= 0.5 + 1e-7) and noise.std() > 0.05
