"""Pricing-scan parity on the GPU: libhello_b200 (through the C ABI) vs the oracle.

ℓ2² (tensor cores): every reported value lies within the stated error bound of
its exact fp64 score, index sets equal the exact top-k wherever the boundary
gap exceeds twice the bound, and the certificate agrees within the bound.
ℓ1/ℓ∞/ℓ2 (CUDA cores): distances are accumulated in the oracle's fp32 order,
so top-k values and indices must be identical bit for bit.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from parity import check_stats, check_topk, flatten

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
U32 = 2.0 ** -24

# (q, n, d, k): tiny, ragged tiles, d % 4 != 0, k > n, wide features, big k
L2SQ_CASES = [(37, 53, 8, 3), (200, 150, 16, 2), (129, 257, 5, 1), (5, 3, 4, 8), (300, 520, 64, 8),
              (1000, 700, 130, 32), (2048, 1500, 256, 4), (4100, 300, 33, 16), (640, 900, 2048, 8)]


def _cloud(q, n, d, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (x[rng.integers(0, q, n)] + 0.5 * rng.normal(size=(n, d))).astype(np.float32)
    a = (x.astype(np.float64) ** 2).sum(1)
    b = (y.astype(np.float64) ** 2).sum(1)
    scale = float(np.median(a)) + 1.0
    f = 0.5 * a + rng.normal(size=q) * 0.3 * scale
    g = 0.5 * b + rng.normal(size=n) * 0.3 * scale
    return x, y, a, b, f, g


def _bound(x, y, r, c, scale, biases, precision):
    """Per-pair error bound of the tensor-core score.
    fp32 mode (3-term split on fp16 halves of the power-of-two scaled clouds): the
    dropped lo*lo term and the rounding of lo, within 3 2^-22 |x||y| per product,
    plus fp32 accumulation (d+2)u (any order), plus the fp16-subnormal floor of
    elements far below their cloud's largest: lo keeps an absolute 2^-25 of the
    scaled value, 2^-39 max|x| per element of x in real units, doubled
    (tests/test_split_model.py restates the split).  TF32: 2^-9 per product."""
    x64, y64 = np.asarray(x, np.float64), np.asarray(y, np.float64)
    d = x64.shape[1]
    absdot = np.einsum("ij,ij->i", np.abs(x64[r]), np.abs(y64[c]))
    prod = 2.0 ** -9 if precision == "tf32" else 2.0 ** -19
    mag = sum(np.abs(v) for v in biases) + scale * absdot
    floor = 0.0
    if precision != "tf32":
        floor = 2.0 ** -38 * (np.abs(x64).max() * np.abs(y64[c]).sum(1) + np.abs(y64).max() * np.abs(x64[r]).sum(1))
    return scale * ((prod + 2 * (d + 2) * U32) * absdot + floor) + 16 * 2.0 ** -53 * mag


def _cert_bounds(x, y, r, c, scale, a, b, qb, dbb, precision):
    """Error bounds of the certificate terms: the kernel evaluates scores and
    costs in fp32 from the tensor-core dot (2^-22 of the magnitudes it adds)."""
    x64, y64 = np.asarray(x, np.float64), np.asarray(y, np.float64)
    e = _bound(x, y, r, c, scale, (a[r], b[c], qb[r], dbb[c]), precision)
    dot = scale * np.abs(np.einsum("ij,ij->i", x64[r], y64[c]))
    return e + 2.0 ** -22 * (dot + np.abs(qb[r]) + np.abs(dbb[c])), e + 2.0 ** -22 * (dot + np.abs(a[r]) + np.abs(b[c]))


CERT_REL = 2.0 ** -20  # fp32 partial sums over 8 terms


def _pad(v, i, width):
    if v.shape[1] < width:
        v = np.pad(v, ((0, 0), (0, width - v.shape[1])), constant_values=-np.inf)
        i = np.pad(i, ((0, 0), (0, width - i.shape[1])), constant_values=-1)
    return v, i


def _check_l2sq(hb, oracle, cuda, x, y, a, b, f, g, k, precision, dot_scale=2.0, min_clear=0.5, passes=None):
    q, n = len(x), len(y)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    qb, dbb = f - a, g - b
    rv, ri, cv, ci, stats = hb.l2sq_scan(T(x, torch.float32), T(y, torch.float32), T(a, torch.float64),
                                         T(b, torch.float64), T(qb, torch.float64), T(dbb, torch.float64), k,
                                         dot_scale=dot_scale, precision=precision, passes=passes)
    rv, ri, cv, ci, stats = (t.cpu().numpy() for t in (rv, ri, cv, ci, stats))
    ev, ei, fv, fi, es = oracle.scan("raw", x, y, qb, dbb, a, b, dot_scale=dot_scale, rk=min(k + 1, n),
                                     ck=min(k + 1, q))
    ev, ei = _pad(ev, ei, k + 1)
    fv, fi = _pad(fv, fi, k + 1)

    def score(r, c, with_cost=False):
        out = oracle.pair_scores("raw", x, y, qb, dbb, a, b, r, c, dot_scale=dot_scale)
        return out if with_cost else out[0]

    def eps(r, c):
        return _bound(x, y, r, c, dot_scale, (a[r], b[c], qb[r], dbb[c]), precision)

    check_topk(rv, ri, ev, ei, score, eps, min_clear=min_clear, label="rows")
    check_topk(cv, ci, fv, fi, lambda r, c: score(c, r), lambda r, c: eps(c, r), min_clear=min_clear, label="cols")
    if q * n <= 4_000_000:
        rr, cc = np.divmod(np.arange(q * n), n)
        s, c = score(rr, cc, with_cost=True)
        es_, ec_ = _cert_bounds(x, y, rr, cc, dot_scale, a, b, qb, dbb, precision)
        check_stats(stats, es, s, c, es_, ec_, rel=CERT_REL, label="stats")
    return rv, ri, cv, ci, stats


@pytest.mark.parametrize("q,n,d,k", L2SQ_CASES)
@pytest.mark.parametrize("precision", ["fp32", "tf32"])
@pytest.mark.parametrize("passes", [1, 2])
def test_l2sq_scan_matches_oracle(hb, cuda, oracle, q, n, d, k, precision, passes):
    if passes == 1 and k > 8:
        pytest.skip("the one-pass scan keeps k <= 8 column lists")
    x, y, a, b, f, g = _cloud(q, n, d, seed=q * 7 + n + d)
    _check_l2sq(hb, oracle, cuda, x, y, a, b, f, g, k, precision,
                min_clear=0.5 if precision == "fp32" else 0.05, passes=passes)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("scan_l2sq_*.npz")))
def test_l2sq_scan_golden(hb, cuda, oracle, path):
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    k = int(z["k"])
    rv, ri, cv, ci, _ = _check_l2sq(hb, oracle, cuda, z["x"], z["y"], z["a"], z["b"], z["f"], z["g"], k, "fp32")
    # candidate pairs: equal to the reference's except pairs inside the error band
    rows, cols = flatten(rv, ri, cv, ci)
    ours = set(zip(rows.tolist(), cols.tolist()))
    ref = set(zip(z["rows"].tolist(), z["cols"].tolist()))
    assert len(ours ^ ref) <= max(2, len(ref) // 100), f"{len(ours ^ ref)} candidate differences"


def test_l2sq_certificate_only_and_scale1(hb, cuda, oracle):
    x, y, a, b, f, g = _cloud(500, 333, 40, seed=3)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    out = hb.l2sq_scan(T(x, torch.float32), T(y, torch.float32), T(a, torch.float64), T(b, torch.float64),
                       T(f - a, torch.float64), T(g - b, torch.float64), 0, dot_scale=1.0)
    es = oracle.scan("raw", x, y, f - a, g - b, a, b, dot_scale=1.0, rk=0, ck=0)[4]
    rr, cc = np.divmod(np.arange(500 * 333), 333)
    s, c = oracle.pair_scores("raw", x, y, f - a, g - b, a, b, rr, cc, dot_scale=1.0)
    es_, ec_ = _cert_bounds(x, y, rr, cc, 1.0, a, b, f - a, g - b, "fp32")
    check_stats(out[4].cpu().numpy(), es, s, c, es_, ec_, rel=CERT_REL, label="certificate")


def test_l2sq_pass_symmetry(hb, cuda):
    """Row and column passes see bit-identical scores for the same pair."""
    x, y, a, b, f, g = _cloud(256, 512, 96, seed=11)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    rv, ri, cv, ci, _ = hb.l2sq_scan(T(x, torch.float32), T(y, torch.float32), T(a, torch.float64),
                                     T(b, torch.float64), T(f - a, torch.float64), T(g - b, torch.float64), 1,
                                     dot_scale=2.0)
    rv, ri, cv, ci = (t.cpu().numpy() for t in (rv, ri, cv, ci))
    # the best pair overall is the top of its row and of its column
    i = int(np.argmax(rv[:, 0]))
    j = int(ri[i, 0])
    assert ci[j, 0] == i and cv[j, 0] == rv[i, 0]


# (q, n, d, k, min_groups): one row group, several row blocks per row group (q > 8 * 128),
# ragged last blocks, k > rows, forced column groups, tf32
ONE_PASS_CASES = [(37, 53, 8, 3, 0, "fp32"), (2048, 1500, 64, 4, 0, "fp32"), (3001, 777, 20, 8, 0, "fp32"),
                  (5, 3, 4, 8, 0, "fp32"), (1300, 2600, 33, 1, 7, "fp32"), (2500, 900, 48, 2, 3, "tf32"),
                  (4096, 4096, 256, 8, 0, "fp32")]


@pytest.mark.parametrize("q,n,d,k,groups,precision", ONE_PASS_CASES)
def test_l2sq_one_pass_equals_two_pass(hb, cuda, q, n, d, k, groups, precision):
    """The one-pass scan (column lists kept per row group in the workspace) and the
    two-pass scan (roles exchanged) report the same lists bit for bit: both insert
    the same fp32 tensor-core dots with the same fp64 score arithmetic and tie rule.
    The certificate differs only in the order of its fp32 partial sums."""
    x, y, a, b, f, g = _cloud(q, n, d, seed=q + 3 * n + d)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    args = (T(x, torch.float32), T(y, torch.float32), T(a, torch.float64), T(b, torch.float64),
            T(f - a, torch.float64), T(g - b, torch.float64), k)
    hb.set_kernel_timing(True)
    try:
        one = [t.clone() for t in hb.l2sq_scan(*args, precision=precision, min_groups=groups, passes=1)]
        assert len(hb.last_kernel_times()) == 1  # one scan kernel launch
        two = [t.clone() for t in hb.l2sq_scan(*args, precision=precision, min_groups=groups, passes=2)]
        assert len(hb.last_kernel_times()) == 2
    finally:
        hb.set_kernel_timing(False)
    for u, v in zip(one[:4], two[:4]):
        assert torch.equal(u, v)
    s1, s2 = one[4].cpu().numpy(), two[4].cpu().numpy()
    # maxima and the count are order-free; (a + b) - dot and (b + a) - dot agree in fp32
    assert s1[2] == s2[2] and s1[3] == s2[3] and s1[4] == s2[4]
    assert s1[0] == pytest.approx(s2[0], rel=4 * CERT_REL) and s1[1] == pytest.approx(s2[1], rel=4 * CERT_REL)


NORM_CASES = [(41, 29, 3, 2), (64, 80, 20, 8), (129, 257, 1, 1), (300, 200, 128, 4), (1000, 1200, 3, 16),
              (5, 3, 2, 8), (513, 260, 9, 32)]


@pytest.mark.parametrize("kind", ["l1", "linf", "l2"])
@pytest.mark.parametrize("q,n,d,k", NORM_CASES)
def test_norm_scan_bit_exact(hb, cuda, oracle, kind, q, n, d, k):
    rng = np.random.default_rng(q + n * 3 + d)
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (x[rng.integers(0, q, n)] + 0.4 * rng.normal(size=(n, d))).astype(np.float32)
    f = rng.normal(size=q) * d * 0.5
    g = rng.normal(size=n) * d * 0.5 + d
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    rv, ri, cv, ci, stats = hb.norm_scan(T(x, torch.float32), T(y, torch.float32), T(f, torch.float64),
                                         T(g, torch.float64), k, kind)
    rv, ri, cv, ci, stats = (t.cpu().numpy() for t in (rv, ri, cv, ci, stats))
    ev, ei, fv, fi, es = oracle.scan(kind, x, y, f, g, rk=min(k, n), ck=min(k, q), exact=False)
    ev, ei = _pad(ev, ei, k)
    fv, fi = _pad(fv, fi, k)
    assert np.array_equal(ri, ei) and np.array_equal(ci, fi)
    assert np.array_equal(rv, ev) and np.array_equal(cv, fv)
    assert stats[2] == es[2] and stats[3] == es[3] and stats[4] == es[4]
    np.testing.assert_allclose(stats[:2], es[:2], rtol=1e-12)


@pytest.mark.parametrize("kind", ["l1", "l2"])
def test_norm_scan_unaligned_features(hb, cuda, kind):
    """d % 4 == 0 but feature bases 4 bytes past a 16-byte boundary: the kernel reads the rows
    with scalar loads instead of 16-byte ones and returns the same lists and certificate."""
    rng = np.random.default_rng(17)
    q, n, d, k = 300, 260, 12, 8
    x = torch.as_tensor(rng.normal(size=(q, d)), dtype=torch.float32, device=cuda)
    y = torch.as_tensor(rng.normal(size=(n, d)), dtype=torch.float32, device=cuda)
    f = torch.as_tensor(rng.normal(size=q) * 3, dtype=torch.float64, device=cuda)
    g = torch.as_tensor(rng.normal(size=n) * 3 + 5, dtype=torch.float64, device=cuda)
    xb = torch.empty(q * d + 1, dtype=torch.float32, device=cuda)
    yb = torch.empty(n * d + 1, dtype=torch.float32, device=cuda)
    xu, yu = xb[1:].view(q, d), yb[1:].view(n, d)
    xu.copy_(x)
    yu.copy_(y)
    assert xu.data_ptr() % 16 != 0 and yu.data_ptr() % 16 != 0
    ref = hb.norm_scan(x, y, f, g, k, kind)
    out = hb.norm_scan(xu, yu, f, g, k, kind)
    for a, b in zip(out, ref):
        assert torch.equal(a, b)


# (q, n, d, k): several row blocks per row group, ragged tiles, k > n, one feature
@pytest.mark.parametrize("shift", [-20, 20])
@pytest.mark.parametrize("passes", [1, 2])
def test_l2sq_power_of_two_scaling(hb, cuda, shift, passes):
    """Each cloud's fp16 halves are taken after scaling it by a power of two, so a
    cloud scaled by 2^s gives the same halves: the lists of the clouds scaled by 2^s
    (costs and biases by 2^2s) are the unscaled lists, with every score times 2^2s
    exactly."""
    x, y, a, b, f, g = _cloud(700, 900, 40, seed=31)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    c = 2.0 ** shift

    def run(sx, sc):
        return [t.clone() for t in hb.l2sq_scan(T(x * sx, torch.float32), T(y * sx, torch.float32), T(a * sc, torch.float64),
                                               T(b * sc, torch.float64), T((f - a) * sc, torch.float64),
                                               T((g - b) * sc, torch.float64), 8, passes=passes)]
    base, scaled = run(1.0, 1.0), run(c, c * c)
    assert torch.equal(base[1], scaled[1]) and torch.equal(base[3], scaled[3])
    assert torch.equal(base[0] * (c * c), scaled[0]) and torch.equal(base[2] * (c * c), scaled[2])


def test_l2sq_rejects_non_finite_features(hb, cuda):
    x, y, a, b, f, g = _cloud(64, 80, 8, seed=2)
    x[3, 2] = np.inf
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    with pytest.raises(ValueError, match="magnitude"):
        hb.l2sq_scan(T(x, torch.float32), T(y, torch.float32), T(a, torch.float64), T(b, torch.float64),
                     T(f - a, torch.float64), T(g - b, torch.float64), 4)


@pytest.mark.parametrize("q,n,d,k,groups,precision", ONE_PASS_CASES)
def test_l2sq_cta_pairs_equal_single_ctas(hb, cuda, q, n, d, k, groups, precision):
    """The one-pass kernel run as CTA pairs (one M = 256 cta_group::2 MMA over both
    CTAs' rows, each CTA staging half of the column tile) reports the same lists as
    the single-CTA kernel: the same dots in the same fp32 order feed the same
    epilogue.  The certificate differs only in the order of its partial sums."""
    x, y, a, b, f, g = _cloud(q, n, d, seed=q + 5 * n + d)
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    args = (T(x, torch.float32), T(y, torch.float32), T(a, torch.float64), T(b, torch.float64),
            T(f - a, torch.float64), T(g - b, torch.float64), k)
    pair = [t.clone() for t in hb.l2sq_scan(*args, precision=precision, min_groups=groups, passes=1, ctas=2)]
    single = [t.clone() for t in hb.l2sq_scan(*args, precision=precision, min_groups=groups, passes=1, ctas=1)]
    for u, v in zip(pair[:4], single[:4]):
        assert torch.equal(u, v)
    s1, s2 = pair[4].cpu().numpy(), single[4].cpu().numpy()
    assert s1[2] == s2[2] and s1[3] == s2[3] and s1[4] == s2[4]
    assert s1[0] == pytest.approx(s2[0], rel=4 * CERT_REL) and s1[1] == pytest.approx(s2[1], rel=4 * CERT_REL)


NORM_ONE_PASS_CASES = [(3000, 777, 20, 8), (130, 2600, 3, 4), (5, 3, 2, 8), (1100, 900, 1, 1), (2049, 2050, 64, 2)]


@pytest.mark.parametrize("kind", ["l1", "linf", "l2"])
@pytest.mark.parametrize("q,n,d,k", NORM_ONE_PASS_CASES)
def test_norm_one_pass_equals_two_pass(hb, cuda, kind, q, n, d, k):
    """One pass (column lists per row group) and two passes (roles exchanged) see the same
    fp32 distances and fp64 scores: identical lists; certificate sums to summation order."""
    rng = np.random.default_rng(q + 2 * n + d)
    x = rng.normal(size=(q, d)).astype(np.float32)
    y = (x[rng.integers(0, q, n)] + 0.4 * rng.normal(size=(n, d))).astype(np.float32)
    f = rng.normal(size=q) * d * 0.5
    g = rng.normal(size=n) * d * 0.5 + d
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    args = (T(x, torch.float32), T(y, torch.float32), T(f, torch.float64), T(g, torch.float64), k, kind)
    hb.set_kernel_timing(True)
    try:
        one = [t.clone() for t in hb.norm_scan(*args)]
        assert len(hb.last_kernel_times()) == 1  # one scan kernel launch
        two = [t.clone() for t in hb.norm_scan(*args, passes=2)]
        assert len(hb.last_kernel_times()) == 2
    finally:
        hb.set_kernel_timing(False)
    for u, v in zip(one[:4], two[:4]):
        assert torch.equal(u, v)
    s1, s2 = one[4].cpu().numpy(), two[4].cpu().numpy()
    assert s1[2] == s2[2] and s1[3] == s2[3] and s1[4] == s2[4]
    np.testing.assert_allclose(s1[:2], s2[:2], rtol=1e-12)


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("scan_l*.npz") if "l2sq" not in p.name))
def test_norm_scan_golden_certificate(hb, cuda, oracle, path):
    with np.load(GOLDEN / path) as z:
        z = {k: z[k] for k in z.files}
    kind, k = str(z["kind"]), int(z["k"])
    T = lambda v, dt: torch.as_tensor(v, dtype=dt, device=cuda)  # noqa: E731
    ext = hb.ScanExtension()
    out = ext.fused_gcost_bidir_certificate(T(z["x"], torch.float32), T(z["y"], torch.float32),
                                            T(z["f"], torch.float64), T(z["g"], torch.float64), hb.topk_bucket(k),
                                            kind)
    num, den = float(out[4]), float(out[5])
    feas = np.sqrt(num) / (1 + np.sqrt(den))
    assert feas == pytest.approx(float(z["dual_feasibility"]), rel=1e-5, abs=1e-9)
    assert abs(int(out[8]) - int(z["stats"][4])) <= 2
