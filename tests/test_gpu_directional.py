"""Directional (initial) scans on the GPU through the C ABI vs the oracle.

ℓ2² (`hb_l2sq_topk`, the reference's initialization_directional_topk_raw): every
reported score within the stated bound of its exact fp64 score, index sets equal
the exact top-k wherever the boundary gap exceeds twice the bound; the lists are
bit-identical to the row side of the bidirectional scan (same kernel).
Norms (`hb_norm_topk`, the reference's fused_gcost_topk): distances in the
oracle's fp32 order, so scores, indices and the (c - g) values the reference
reports are identical bit for bit; the cost statistics agree to summation order.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from parity import check_topk
from test_gpu_scan import _bound, _cloud, _pad

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"

# (q, n, d, k): k = 16 (the initial scan's kappa), k > n, ragged tiles, wide features, k = 32
L2SQ_CASES = [(300, 520, 64, 16), (129, 20, 33, 32), (1000, 700, 130, 8), (64, 2100, 256, 1), (513, 300, 2048, 4)]
NORM_CASES = [(41, 29, 3, 2), (300, 200, 128, 16), (129, 257, 1, 1), (1000, 1200, 3, 32), (5, 3, 2, 8)]


def _t(v, dt, dev):
    return torch.as_tensor(v, dtype=dt, device=dev)


@pytest.mark.parametrize("q,n,d,k", L2SQ_CASES)
@pytest.mark.parametrize("precision", ["fp32", "tf32"])
def test_l2sq_topk_matches_oracle(hb, cuda, oracle, q, n, d, k, precision):
    x, y, a, b, f, g = _cloud(q, n, d, seed=q + n + 5 * d)
    qb, dbb = f - a, g - b
    vals, idx = hb.l2sq_topk(_t(x, torch.float32, cuda), _t(y, torch.float32, cuda), _t(qb, torch.float64, cuda),
                             _t(dbb, torch.float64, cuda), k, dot_scale=2.0, precision=precision)
    vals, idx = vals.cpu().numpy(), idx.cpu().numpy()
    ev, ei, _, _, _ = oracle.scan("raw", x, y, qb, dbb, a, b, dot_scale=2.0, rk=min(k + 1, n), ck=0)
    ev, ei = _pad(ev, ei, k + 1)

    def score(r, c):
        return oracle.pair_scores("raw", x, y, qb, dbb, a, b, r, c, dot_scale=2.0)[0]

    def eps(r, c):
        return _bound(x, y, r, c, 2.0, (a[r], b[c], qb[r], dbb[c]), precision)

    check_topk(vals, idx, ev, ei, score, eps, min_clear=0.5 if precision == "fp32" else 0.05, label="directional")


@pytest.mark.parametrize("passes", [1, 2])
def test_l2sq_topk_equals_scan_rows(hb, cuda, passes):
    """Same kernel, same arithmetic: the directional lists are the scan's row lists."""
    x, y, a, b, f, g = _cloud(700, 900, 96, seed=21)
    args = [_t(v, torch.float32, cuda) for v in (x, y)] + [_t(v, torch.float64, cuda) for v in (a, b, f - a, g - b)]
    rv, ri, _, _, _ = hb.l2sq_scan(*args, 8, dot_scale=2.0, passes=passes)
    vals, idx = hb.l2sq_topk(args[0], args[1], args[4], args[5], 8, dot_scale=2.0)
    assert torch.equal(vals, rv) and torch.equal(idx, ri)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("directional_l2sq_*.npz")))
def test_l2sq_topk_golden(hb, cuda, oracle, path):
    """The reference's directional assignment (inner-product family, known side target)."""
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    x, y, a, b, g, k = z["x"], z["y"], z["a"], z["b"], z["g"], int(z["k"])
    q, n = len(x), len(y)
    ext = hb.ScanExtension()
    vals, idx = ext.initialization_directional_topk_raw(_t(x, torch.float32, cuda), _t(y, torch.float32, cuda),
                                                        _t(-a, torch.float64, cuda), _t(g - b, torch.float64, cuda),
                                                        2048, 8192, hb.topk_bucket(k), 2.0)
    assert idx.dtype == torch.int32
    vals, idx = vals.cpu().numpy(), idx.cpu().numpy().astype(np.int64)
    rk = min(k, n)
    e1 = _bound(x, y, np.arange(q), z["top1_indices"], 2.0, (a, b[z["top1_indices"]], g[z["top1_indices"]]), "fp32")
    assert np.all(np.abs(vals[:, 0] - z["top1_values"]) <= 2 * e1 + 1e-9 * np.abs(z["top1_values"]))
    ours = {(r, int(c)) for r in range(q) for c in idx[r, :rk] if c >= 0}
    ref = set(zip(z["rows"].tolist(), z["cols"].tolist()))
    assert len(ours ^ ref) <= max(2, len(ref) // 100)
    if k > n:  # missing slots: (-inf, -1)
        assert np.all(idx[:, n:] == -1) and np.all(np.isneginf(vals[:, n:]))


@pytest.mark.parametrize("kind", ["l1", "linf", "l2"])
@pytest.mark.parametrize("q,n,d,k", NORM_CASES)
def test_norm_topk_bit_exact(hb, cuda, oracle, kind, q, n, d, k):
    rng = np.random.default_rng(q * 3 + n + d)
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (x[rng.integers(0, q, n)] + 0.4 * rng.normal(size=(n, d))).astype(np.float32)
    g = rng.normal(size=n) * d * 0.5
    ext = hb.ScanExtension()
    out = ext.fused_gcost_topk(_t(x, torch.float32, cuda), _t(y, torch.float32, cuda), _t(g, torch.float64, cuda), k,
                               kind, collect_statistics=True)
    vals, idx, stats = (t.cpu().numpy() for t in out)
    assert out[1].dtype == torch.int64
    ev, ei, _, _, es = oracle.scan(kind, x, y, np.full(q, -0.0), g, rk=min(k, n), ck=0, exact=False)
    ev, ei = _pad(ev, ei, k)
    # the reference reports c - g ascending: the negated scores, missing slots (+inf, -1)
    assert np.array_equal(idx, ei)
    assert np.array_equal(vals, -ev)
    assert stats[1] == es[3]
    np.testing.assert_allclose(stats[0], es[1], rtol=1e-12)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("directional_l*.npz")
                                        if "l2sq" not in p.name))
def test_norm_topk_golden(hb, cuda, oracle, path):
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    x, y, g, k, kind = z["x"], z["y"], z["g"], int(z["k"]), str(z["cost"])
    q, n = len(x), len(y)
    ext = hb.ScanExtension()
    vals, idx = ext.fused_gcost_topk(_t(x, torch.float32, cuda), _t(y, torch.float32, cuda), _t(g, torch.float64, cuda),
                                     hb.topk_bucket(k), kind)
    vals, idx = vals.cpu().numpy(), idx.cpu().numpy()
    # top-1: the reference's score g - c within the fp32 distance error
    e1 = np.abs(z["top1_values"]) * 1e-6 + 1e-6
    assert np.all(np.abs(-vals[:, 0] - z["top1_values"]) <= e1)
    ours = {(r, int(c)) for r in range(q) for c in idx[r, :min(k, n)] if c >= 0}
    ref = set(zip(z["rows"].tolist(), z["cols"].tolist()))
    assert len(ours ^ ref) <= max(2, len(ref) // 100)


def test_directional_input_errors(hb, cuda):
    x = torch.zeros((8, 4), device=cuda)
    v = torch.zeros(8, dtype=torch.float64, device=cuda)
    ext = hb.ScanExtension()
    with pytest.raises(ValueError, match="power-of-two bucket"):
        ext.initialization_directional_topk_raw(x, x, v, v, 64, 64, 3, 2.0)
    with pytest.raises(ValueError, match="tile or scale"):
        ext.initialization_directional_topk_raw(x, x, v, v, 64, 64, 4, 3.0)
    with pytest.raises(ValueError, match="global indices"):  # sigma > 0 needs the global indices
        ext.fused_gcost_topk(x, x, v, 4, "l1", sigma=0.5)
    L = hb.lib()
    assert L.hb_l2sq_topk(x.data_ptr(), x.data_ptr(), 8, 8, 4, v.data_ptr(), v.data_ptr(), 64, 2.0, 3,
                          v.data_ptr(), v.data_ptr(), v.data_ptr(), 1 << 20, None) == hb._lib.HB_BAD_ARGUMENT
    assert L.hb_norm_topk(x.data_ptr(), x.data_ptr(), 8, 8, 4, v.data_ptr(), 3, 4, 0, v.data_ptr(), v.data_ptr(),
                          None, v.data_ptr(), 1 << 20, None) == hb._lib.HB_BAD_ARGUMENT
