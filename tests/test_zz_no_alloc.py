"""hb_norm_scan_noalloc: the scan for callers that cannot allocate device memory.

Some hosts reach this library through an FFI without a CUDA allocator, or run
under a device-memory budget that forbids new allocations mid-solve; they
cannot provide the workspace hb_norm_scan asks for.  The allocation-free entry
point keeps its scratch in a static device array of the library (a fixed
16 MiB, held for the life of the process).  This test calls it through the C
ABI and checks it against the workspace entry point on two calls in a row
(the array keeps the previous call's contents), and that a problem whose
scratch exceeds the array is refused with a clear error.

The file name sorts last so a run that stops at the first failure has already
run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
NOALLOC_BYTES = 16 << 20


def _outputs(dev, q, n, k):
    return (torch.empty((q, k), dtype=torch.float64, device=dev), torch.empty((q, k), dtype=torch.int32, device=dev),
            torch.empty((n, k), dtype=torch.float64, device=dev), torch.empty((n, k), dtype=torch.int32, device=dev),
            torch.zeros(5, dtype=torch.float64, device=dev))


def _call_noalloc(hb, x, y, f, g, kind, k):
    L = hb.lib()
    dev = x.device
    q, d = x.shape
    n = y.shape[0]
    out = _outputs(dev, q, n, k)
    rc = L.hb_norm_scan_noalloc(x.data_ptr(), y.data_ptr(), q, n, d, f.data_ptr(), g.data_ptr(), kind, k, 1,
                                *(t.data_ptr() for t in out), torch.cuda.current_stream(dev).cuda_stream)
    hb._lib.check(rc)
    return out


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_noalloc_matches_workspace_entry_twice(hb, cuda, kind):
    L = hb.lib()
    rng = np.random.default_rng(100 + kind)
    # two different problems in a row: the second call must not see the first one's scratch
    for q, n, d, k in ((700, 900, 24, 8), (333, 150, 5, 4)):
        assert L.hb_norm_scan_workspace(q, n, k) <= NOALLOC_BYTES
        x = torch.as_tensor(rng.normal(size=(q, d)), dtype=torch.float32, device=cuda)
        y = torch.as_tensor(rng.normal(size=(n, d)), dtype=torch.float32, device=cuda)
        f = torch.as_tensor(rng.normal(size=q) * d, dtype=torch.float64, device=cuda)
        g = torch.as_tensor(rng.normal(size=n) * d + d, dtype=torch.float64, device=cuda)
        got = _call_noalloc(hb, x, y, f, g, kind, k)
        ref = hb.norm_scan(x, y, f, g, k, kind)
        # the same kernels on the same grid: identical results
        for a, b in zip(got[:4], ref[:4]):
            assert torch.equal(a, b)
        assert torch.equal(got[4], ref[4])


def test_noalloc_rejects_problems_beyond_its_buffer(hb, cuda):
    L = hb.lib()
    q = n = 400_000
    assert L.hb_norm_scan_workspace(q, n, 8) > NOALLOC_BYTES
    x = torch.zeros((8, 2), dtype=torch.float32, device=cuda)  # never read: the size check comes first
    f = torch.zeros(8, dtype=torch.float64, device=cuda)
    out = _outputs(cuda, 1, 1, 8)
    rc = L.hb_norm_scan_noalloc(x.data_ptr(), x.data_ptr(), q, n, 2, f.data_ptr(), f.data_ptr(), 0, 8, 1,
                                *(t.data_ptr() for t in out), None)
    assert rc == hb._lib.HB_WORKSPACE
    msg = L.hb_last_error().decode()
    assert "static buffer holds" in msg and str(NOALLOC_BYTES) in msg
