"""CPU-only checks: the C ABI's export table, host-side logic and error paths.

No kernel runs here (no GPU in this container); entry points that need CUDA
must raise instead of falling back to a CPU path.
"""
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from parity import flatten

REPO = Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol(hb):
    header = (REPO / "include" / "hello_b200.h").read_text()
    declared = set(re.findall(r"^\s*(?:size_t|int|void|unsigned long long|const char\*)\s+(hb_\w+)\s*\(",
                              header, flags=re.M))
    assert declared, "no declarations parsed"
    lib = hb.load_library()
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in hello_b200.h but not exported"
    assert declared == set(hb._lib.EXPORTS)
    assert lib.hb_abi_version() == hb._lib.ABI_VERSION == 2


def test_header_cites_reference_interfaces():
    header = (REPO / "include" / "hello_b200.h").read_text()
    for cite in ("generic_scan.py:577-597", "generic_scan.py:533-558", "pairs.py:221-440",
                 "norm_cost_scan_kernel.cu:249-275", "restricted_ot_pdlp.py:39-100", "solver.cpp:39-381",
                 "generic_scan.py:520-531", "initial.cu:34-107", "cost.cu:248-348"):
        assert cite in header


def test_no_cpu_fallback(hb, monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(hb.HBError, match="requires a CUDA device"):
        hb.lib()
    x = torch.zeros(4, 3)
    with pytest.raises(hb.HBError):
        hb.l2sq_scan(x, x, torch.zeros(4, dtype=torch.float64), torch.zeros(4, dtype=torch.float64),
                     torch.zeros(4, dtype=torch.float64), torch.zeros(4, dtype=torch.float64), 2)
    with pytest.raises(hb.HBError):
        hb.raw_lowrank_bidir_feasibility_pricing_scan(x.numpy(), x.numpy(), np.zeros(4), np.zeros(4), np.zeros(4),
                                                      np.zeros(4), topk=2)


def test_topk_buckets(hb):
    assert [hb.topk_bucket(k) for k in (1, 2, 3, 4, 5, 8, 9, 17, 32)] == [1, 2, 4, 4, 8, 8, 16, 32, 32]
    with pytest.raises(ValueError):
        hb.topk_bucket(0)
    with pytest.raises(ValueError, match="topk <= 32"):
        hb.topk_bucket(33)


def test_flatten_candidates_matches_reference_order(hb):
    rng = np.random.default_rng(0)
    rv = rng.normal(size=(50, 4))
    ri = rng.integers(-1, 70, size=(50, 4)).astype(np.int32)
    cv = rng.normal(size=(70, 4))
    ci = rng.integers(-1, 50, size=(70, 4)).astype(np.int32)
    rows, cols = hb.flatten_candidates(*(torch.as_tensor(v) for v in (rv, ri, cv, ci)), theta=0.1)
    er, ec = flatten(rv, ri, cv, ci, theta=0.1)
    assert np.array_equal(rows.numpy(), er) and np.array_equal(cols.numpy(), ec)
    # target-side queries swap the roles
    rows2, cols2 = hb.flatten_candidates(*(torch.as_tensor(v) for v in (rv, ri, cv, ci)), theta=0.1,
                                         query_is_source=False)
    assert np.array_equal(rows2.numpy(), ec) and np.array_equal(cols2.numpy(), er)


def test_scan_extension_validates_before_launch(hb):
    ext = hb.ScanExtension()
    x = torch.zeros(4, 3)
    v = torch.zeros(4, dtype=torch.float64)
    with pytest.raises(ValueError, match="CUDA FP32 feature"):
        ext.fused_bidir_topk_stats_raw(x, x, v, v, v, v, 8, 8, 64, 2, True, True, False, 2, 2.0)
    with pytest.raises(ValueError, match="power-of-two bucket"):
        ext.fused_bidir_topk_stats_raw(x, x, v, v, v, v, 8, 8, 64, 3, True, True, False, 0, 2.0)
    with pytest.raises(ValueError):  # CPU tensors (and, with sigma > 0, no global indices)
        ext.fused_gcost_bidir_certificate(x, x, v, v, 2, 0, sigma=0.1)


def test_pdlp_validates_controls(hb):
    with pytest.raises(ValueError):
        hb.NativeRestrictedOTPDLP(device="cpu")
    with pytest.raises(ValueError):
        hb.NativeRestrictedOTPDLP(device="cuda:0", evaluation_frequency=0)


def test_l2sq_pass_flags_are_validated_before_launch(hb):
    """Bad precision / pass-flag combinations are refused before any device work."""
    lib = hb.load_library()
    fake = 256  # never dereferenced: the argument checks come first
    base = [fake, fake, 100, 100, 8, fake, fake, fake, fake]

    def call(k, precision):
        return lib.hb_l2sq_scan(*base, k, 2.0, 1, precision, 0, fake, fake, fake, fake, fake, fake, 1 << 20, None)

    one, two = 0x20, 0x10
    assert call(8, 2) == hb._lib.HB_BAD_ARGUMENT
    assert "precision must be 1" in lib.hb_last_error().decode()
    assert call(8, 3 | one | two) == hb._lib.HB_BAD_ARGUMENT
    assert "exclusive" in lib.hb_last_error().decode()
    assert call(16, 3 | one) == hb._lib.HB_BAD_ARGUMENT
    assert "one-pass scan needs" in lib.hb_last_error().decode()
    assert call(0, 1 | one) == hb._lib.HB_BAD_ARGUMENT


def test_coarsest_rejects_cpu_device(hb):
    with pytest.raises(ValueError, match="CUDA"):
        hb.solve_leaf_from_cost(cost=np.ones((2, 2)), source_mass=[0.5, 0.5], target_mass=[0.5, 0.5], device="cpu")


def test_python_flags_match_the_header(hb):
    """The binding's flag values are the header's (a mismatch would silently select
    another pass mode, CTA layout or node-sum order)."""
    header = (REPO / "include" / "hello_b200.h").read_text()
    defs = {m.group(1): int(m.group(2), 0) for m in re.finditer(r"#define (HB_\w+) (0x[0-9a-fA-F]+|\d+)\b", header)}
    enums = {m.group(1): int(m.group(2)) for m in re.finditer(r"(HB_PDLP_(?:SUMS|NORM)_\w+) = (\d+)", header)}
    scan = hb.scan
    assert scan.L2SQ_PASS_FLAGS[2] == defs["HB_L2SQ_TWO_PASS"] and scan.L2SQ_PASS_FLAGS[1] == defs["HB_L2SQ_ONE_PASS"]
    assert scan.L2SQ_CTA_FLAGS[2] == defs["HB_L2SQ_CTA_PAIRS"] and scan.L2SQ_CTA_FLAGS[1] == defs["HB_L2SQ_SINGLE_CTA"]
    assert scan.NORM_TWO_PASS == defs["HB_NORM_TWO_PASS"]
    assert hb.pdlp.SUMMATION == {"ordered": enums["HB_PDLP_SUMS_ORDERED"], "atomic": enums["HB_PDLP_SUMS_ATOMIC"],
                                 "tree": enums["HB_PDLP_SUMS_TREE"]}
    assert hb.pdlp.TERMINATION_NORMS == {"l2": enums["HB_PDLP_NORM_L2"], "linf": enums["HB_PDLP_NORM_LINF"]}
    # the ctypes structures carry the header's fields in its order
    from hello_ot_b200._lib import PdlpControls, PdlpInfo
    assert [f[0] for f in PdlpControls._fields_][-2:] == ["atomic_sums", "termination_norm"]
    assert [f[0] for f in PdlpInfo._fields_][-4:] == ["l2_abs_primal_residual", "l2_rel_primal_residual",
                                                       "l2_abs_dual_residual", "l2_rel_dual_residual"]


def test_generic_scan_validates_before_launch(hb):
    """The module-level scan entry points reject bad buckets, kinds and non-CUDA inputs
    with the reference's ValueError before anything reaches the library."""
    gs = hb.generic_scan
    x = torch.zeros((4, 3))
    v = torch.zeros(4, dtype=torch.float64)
    with pytest.raises(ValueError, match="power-of-two bucket"):
        gs.bidirectional(x, x, v, v, 3, 0)
    with pytest.raises(ValueError, match="CUDA"):
        gs.bidirectional(x, x, v, v, 4, 0)
    with pytest.raises(ValueError, match="CUDA"):
        gs.directional(x, x, v, 4, 0)
    with pytest.raises(ValueError, match="CUDA"):
        gs.certificate_only(x, x, v, v, 3, raw_costs=(v, v))


def test_leaf_cost_matrix_validates_kind(hb):
    x = torch.zeros((4, 3))
    with pytest.raises(ValueError, match="kind"):
        hb.leaf_cost_matrix(x, x, "cosine")
    with pytest.raises(ValueError, match="offset"):
        hb.leaf_cost_matrix(x, x, "l2^2")


def test_fp64_pricing_needs_fp32_representable_features(hb):
    """compute_precision="fp64" is served as exact fp64 lists over fp32 features; features that
    are not fp32 values are refused before anything reaches the library."""
    from hello_ot_b200.scan import _holds_fp32
    x = np.random.default_rng(0).normal(size=(5, 3))
    assert not _holds_fp32(x) and _holds_fp32(x.astype(np.float32)) and _holds_fp32(x.astype(np.float32).astype(float))
    v = np.zeros(5)
    with pytest.raises(NotImplementedError, match="representable in fp32"):
        hb.raw_lowrank_bidir_feasibility_pricing_scan(x, x, v, v, v, v, topk=2, compute_precision="fp64")

