"""fp64 re-check of the ℓ2² scan (HB_L2SQ_EXACT) against the oracle's exact fp64 scan.

With the re-check every list must be the exact top-k of the fp64 score
(s <x_i, y_j> + qb_i) + dbb_j: reported values within the fp64 rounding of
the exact scores, index sets equal wherever the k-th/(k+1)-th exact gap exceeds
that rounding, on clouds where the fp32-class dot is far from exact:
Gaussian, heavy-tailed (Cauchy), one outlier row 2^16 or 2^24 times the rest, a
block of rows 2^-24 times the rest (fp16-subnormal range of the split),
duplicated points and groups of eight identical points (exact ties, broken by
the lower index; the eight-way ties force every row list through the fp64
rescan).  The same wide-range clouds also run without the re-check against the
approximate bound, which carries the fp16-subnormal floor.
"""
import numpy as np
import pytest
import torch

from parity import check_topk

pytestmark = pytest.mark.gpu
U64 = 2.0 ** -53


def _cloud(kind, q, n, d, seed):
    rng = np.random.default_rng(seed)
    if kind == "cauchy":
        x = rng.standard_cauchy(size=(q, d))
        y = x[rng.integers(0, q, n)] + rng.standard_cauchy(size=(n, d))
        x, y = np.clip(x, -1e6, 1e6), np.clip(y, -1e6, 1e6)
    else:
        x = rng.normal(size=(q, d))
        y = x[rng.integers(0, q, n)] + 0.5 * rng.normal(size=(n, d))
    if kind == "outlier16":
        x[3] *= 2.0 ** 16
    elif kind == "outlier24":
        y[5] *= 2.0 ** 24
    elif kind == "tiny_block":
        x[: q // 3] *= 2.0 ** -24
    elif kind == "duplicates":
        y[1::2] = y[0::2][: n // 2]
    elif kind == "ties8":  # groups of eight identical targets: ties wider than any list
        y = y[np.arange(n) // 8 * 8]
    x, y = x.astype(np.float32), y.astype(np.float32)
    a = (x.astype(np.float64) ** 2).sum(1)
    b = (y.astype(np.float64) ** 2).sum(1)
    scale = float(np.median(a)) + 1.0
    f = 0.5 * a + rng.normal(size=q) * 0.3 * scale
    g = 0.5 * b + rng.normal(size=n) * 0.3 * scale
    if kind == "duplicates":  # duplicated targets with equal duals: exact ties in every list
        g[1::2] = g[0::2][: n // 2]
    elif kind == "ties8":
        g = g[np.arange(n) // 8 * 8]
    return x, y, a, b, f, g


def _pad(v, i, width):
    if v.shape[1] < width:
        v = np.pad(v, ((0, 0), (0, width - v.shape[1])), constant_values=-np.inf)
        i = np.pad(i, ((0, 0), (0, width - i.shape[1])), constant_values=-1)
    return v, i


def _eps64(x, y, r, c, scale, biases):
    """fp64 rounding of an exactly computed score: the dot summed in any order
    (d + 2) 2^-53 sum |x y|, the two additions a few ulps of the magnitudes."""
    x64, y64 = np.asarray(x, np.float64), np.asarray(y, np.float64)
    absdot = np.einsum("ij,ij->i", np.abs(x64[r]), np.abs(y64[c]))
    d = x64.shape[1]
    return scale * 2 * (d + 2) * U64 * absdot + 16 * U64 * (sum(np.abs(v) for v in biases) + scale * absdot) + 1e-300


def _run(hb, oracle, cuda, kind, q, n, d, k, passes, exact, precision="fp32", ctas=None):
    x, y, a, b, f, g = _cloud(kind, q, n, d, seed=q + 3 * n + d + k)
    qb, dbb = f - a, g - b
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    rv, ri, cv, ci, _ = hb.l2sq_scan(T(x, torch.float32), T(y, torch.float32), T(a, torch.float64),
                                     T(b, torch.float64), T(qb, torch.float64), T(dbb, torch.float64), k,
                                     dot_scale=2.0, precision=precision, passes=passes, exact=exact, ctas=ctas)
    rescans = hb.l2sq_last_rescans()
    rv, ri, cv, ci = (t.cpu().numpy() for t in (rv, ri, cv, ci))
    ev, ei, fv, fi, _ = oracle.scan("raw", x, y, qb, dbb, a, b, dot_scale=2.0, rk=min(k + 1, n), ck=min(k + 1, q))
    ev, ei = _pad(ev, ei, k + 1)
    fv, fi = _pad(fv, fi, k + 1)

    def score(r, c):
        return oracle.pair_scores("raw", x, y, qb, dbb, a, b, r, c, dot_scale=2.0)[0]

    return (x, y, a, b, qb, dbb), (rv, ri, cv, ci), (ev, ei, fv, fi), score, rescans


EXACT_CASES = [  # (cloud, q, n, d, k)
    ("gauss", 700, 900, 64, 8), ("gauss", 333, 1200, 16, 2), ("gauss", 300, 500, 130, 16),
    ("cauchy", 600, 800, 32, 8), ("cauchy", 500, 400, 64, 1),
    ("outlier16", 500, 700, 64, 4), ("outlier24", 400, 900, 48, 8),
    ("tiny_block", 600, 500, 40, 8), ("duplicates", 400, 800, 24, 8), ("duplicates", 256, 300, 16, 32),
    ("ties8", 200, 400, 24, 2), ("ties8", 150, 320, 96, 4),
]


@pytest.mark.parametrize("cloud,q,n,d,k", EXACT_CASES)
@pytest.mark.parametrize("passes", [1, 2])
def test_exact_lists_equal_fp64_topk(hb, cuda, oracle, cloud, q, n, d, k, passes):
    if passes == 1 and k > 8:
        pytest.skip("the one-pass scan keeps k <= 8 column lists")
    (x, y, a, b, qb, dbb), (rv, ri, cv, ci), (ev, ei, fv, fi), score, rescans = _run(hb, oracle, cuda, cloud, q, n,
                                                                                     d, k, passes, True)

    def eps(r, c):
        return _eps64(x, y, r, c, 2.0, (a[r], b[c], qb[r], dbb[c]))

    min_clear = 0.0 if cloud in ("duplicates", "ties8") else 0.95
    check_topk(rv, ri, ev, ei, score, eps, min_clear=min_clear, label="rows")
    check_topk(cv, ci, fv, fi, lambda r, c: score(c, r), lambda r, c: eps(c, r), min_clear=min_clear, label="cols")
    if cloud in ("duplicates", "ties8"):  # exact ties: the lower index wins, as in the oracle
        assert np.array_equal(ri, ei[:, :k]) and np.array_equal(ci, fi[:, :k])
    if cloud == "ties8":  # every row list ends inside a tie wider than the list: all rescanned
        assert rescans[0] == q, rescans


def test_exact_tf32_and_cta_pairs(hb, cuda, oracle):
    """The re-check also makes the TF32 mode and the CTA-pair kernel exact."""
    for precision, d, ctas in (("tf32", 96, None), ("fp32", 1100, 2)):
        (x, y, a, b, qb, dbb), (rv, ri, cv, ci), (ev, ei, fv, fi), score, _ = _run(
            hb, oracle, cuda, "gauss", 400, 600, d, 8, 1, True, precision=precision, ctas=ctas)

        def eps(r, c):
            return _eps64(x, y, r, c, 2.0, (a[r], b[c], qb[r], dbb[c]))

        check_topk(rv, ri, ev, ei, score, eps, min_clear=0.95, label=f"rows {precision}")
        check_topk(cv, ci, fv, fi, lambda r, c: score(c, r), lambda r, c: eps(c, r), min_clear=0.95,
                   label=f"cols {precision}")


@pytest.mark.parametrize("cloud", ["cauchy", "outlier16", "outlier24", "tiny_block"])
def test_approximate_lists_within_floor_bound(hb, cuda, oracle, cloud):
    """Without the re-check, wide-range clouds stay within the split's bound including the
    fp16-subnormal floor s 2^-38 (max|x| sum|y_k| + max|y| sum|x_k|)."""
    from test_gpu_scan import _bound
    (x, y, a, b, qb, dbb), (rv, ri, cv, ci), (ev, ei, fv, fi), score, _ = _run(hb, oracle, cuda, cloud, 500, 700, 48,
                                                                               8, None, False)

    def eps(r, c):
        return _bound(x, y, r, c, 2.0, (a[r], b[c], qb[r], dbb[c]), "fp32")

    check_topk(rv, ri, ev, ei, score, eps, min_clear=0.0, label="rows")
    check_topk(cv, ci, fv, fi, lambda r, c: score(c, r), lambda r, c: eps(c, r), min_clear=0.0, label="cols")
