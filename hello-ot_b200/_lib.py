"""ctypes binding of libhello_b200.so (the C ABI in include/hello_b200.h).

The library is loaded from this package's folder; there is no fallback: if it
is missing or CUDA is unavailable every entry point raises.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libhello_b200.so"
ABI_VERSION = 2

HB_OK, HB_BAD_ARGUMENT, HB_BAD_INPUT, HB_WORKSPACE = 0, 1, 2, 3
HB_CUDA, HB_TENSOR_MAP, HB_LAUNCH, HB_DEVICE_TIMEOUT = 4, 5, 6, 7

EXPORTS = ("hb_abi_version", "hb_last_error", "hb_kernel_launch_count", "hb_set_kernel_timing",
           "hb_last_kernel_times", "hb_l2sq_scan_workspace", "hb_l2sq_scan", "hb_l2sq_topk_workspace",
           "hb_l2sq_topk", "hb_norm_topk_workspace", "hb_norm_topk", "hb_norm_scan_workspace",
           "hb_norm_scan", "hb_norm_scan_noalloc", "hb_merge_topk", "hb_pair_costs_workspace", "hb_pair_costs", "hb_restricted_ot_workspace",
           "hb_restricted_ot_solve", "hb_filter_new_pairs_workspace", "hb_filter_new_pairs",
           "hb_prune_select_workspace", "hb_prune_select", "hb_norm_scan_ex", "hb_norm_topk_ex",
           "hb_pair_costs_ex", "hb_l2sq_last_rescans")


class HBError(RuntimeError):
    """A libhello_b200 entry point returned a nonzero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[hello_b200 error {code}] {message}")
        self.code = code


class PdlpControls(ctypes.Structure):
    _fields_ = [("evaluation_frequency", c_int32), ("scalar_rescaling", c_int32), ("iteration_limit", c_int64),
                ("time_limit_seconds", c_double), ("tol_objective", c_double), ("tol_primal", c_double),
                ("tol_dual", c_double), ("initial_primal_weight", c_double), ("atomic_sums", c_int32),
                ("termination_norm", c_int32)]


class Perturbation(ctypes.Structure):
    """hb_perturbation: norm-cost noise (sigma == 0: none)."""
    _fields_ = [("sigma", c_double), ("seed", c_int64), ("mode", c_int32), ("row_is_source", c_int32),
                ("query_index", c_void_p), ("database_index", c_void_p), ("coefficients", c_int64 * 6)]


class PdlpInfo(ctypes.Structure):
    _fields_ = [("iterations", c_int64), ("restarts", c_int64), ("termination", c_int32), ("pad", c_int32),
                ("primal_objective", c_double), ("dual_objective", c_double), ("abs_primal_residual", c_double),
                ("rel_primal_residual", c_double), ("abs_dual_residual", c_double), ("rel_dual_residual", c_double),
                ("rel_gap", c_double), ("primal_weight", c_double), ("cost_norm", c_double),
                ("mass_norm", c_double), ("setup_seconds", c_double), ("iteration_seconds", c_double),
                ("l2_abs_primal_residual", c_double), ("l2_rel_primal_residual", c_double),
                ("l2_abs_dual_residual", c_double), ("l2_rel_dual_residual", c_double)]


class PdlpTraceRow(ctypes.Structure):
    _fields_ = [("iteration", c_double), ("primal_objective", c_double), ("dual_objective", c_double),
                ("rel_primal", c_double), ("rel_dual", c_double), ("rel_gap", c_double),
                ("primal_weight", c_double)]


_LIB = None


def load_library(path: Path | str = LIB_PATH):
    """Load the shared library and declare its signatures (no GPU needed)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(path)
    if not path.exists():
        raise HBError(HB_CUDA, f"{path.name} is not built; run __graft_entry__.build() "
                               "(python hello-ot_b200/build.py)")
    lib = ctypes.CDLL(str(path))
    P = c_void_p
    lib.hb_abi_version.restype = c_int
    lib.hb_last_error.restype = ctypes.c_char_p
    lib.hb_kernel_launch_count.restype = ctypes.c_ulonglong
    lib.hb_set_kernel_timing.argtypes = [c_int]
    lib.hb_set_kernel_timing.restype = None
    lib.hb_last_kernel_times.argtypes = [POINTER(c_double), c_int]
    lib.hb_last_kernel_times.restype = c_int
    lib.hb_l2sq_scan_workspace.restype = c_size_t
    lib.hb_l2sq_scan_workspace.argtypes = [c_int64, c_int64, c_int64, c_int, c_int, c_int]
    lib.hb_l2sq_scan.restype = c_int
    lib.hb_l2sq_scan.argtypes = [P, P, c_int64, c_int64, c_int64, P, P, P, P, c_int, c_double, c_int, c_int, c_int,
                                 P, P, P, P, P, P, c_size_t, P]
    lib.hb_l2sq_last_rescans.restype = c_int
    lib.hb_l2sq_last_rescans.argtypes = [POINTER(c_int64)]
    lib.hb_l2sq_topk_workspace.restype = c_size_t
    lib.hb_l2sq_topk_workspace.argtypes = [c_int64, c_int64, c_int64, c_int, c_int]
    lib.hb_l2sq_topk.restype = c_int
    lib.hb_l2sq_topk.argtypes = [P, P, c_int64, c_int64, c_int64, P, P, c_int, c_double, c_int, P, P, P, c_size_t, P]
    lib.hb_norm_topk_workspace.restype = c_size_t
    lib.hb_norm_topk_workspace.argtypes = [c_int64, c_int64, c_int]
    lib.hb_norm_topk.restype = c_int
    lib.hb_norm_topk.argtypes = [P, P, c_int64, c_int64, c_int64, P, c_int, c_int, c_int, P, P, P, P, c_size_t, P]
    lib.hb_filter_new_pairs_workspace.restype = c_size_t
    lib.hb_filter_new_pairs_workspace.argtypes = [c_int64, c_int64]
    lib.hb_filter_new_pairs.restype = c_int
    lib.hb_filter_new_pairs.argtypes = [P, c_int64, c_int32, P, P, c_int64, c_int64, c_int64, P, P,
                                        ctypes.POINTER(c_int64), P, c_size_t, P]
    lib.hb_prune_select_workspace.restype = c_size_t
    lib.hb_prune_select_workspace.argtypes = [c_int64]
    lib.hb_prune_select.restype = c_int
    lib.hb_prune_select.argtypes = [P, P, P, P, P, c_int64, P, c_int64, c_int64, c_int32, c_int64, P,
                                    ctypes.POINTER(c_int64), P, c_size_t, P]
    lib.hb_norm_scan_workspace.restype = c_size_t
    lib.hb_norm_scan_workspace.argtypes = [c_int64, c_int64, c_int]
    lib.hb_norm_scan.restype = c_int
    lib.hb_norm_scan.argtypes = [P, P, c_int64, c_int64, c_int64, P, P, c_int, c_int, c_int, P, P, P, P, P, P,
                                 c_size_t, P]
    lib.hb_norm_scan_ex.restype = c_int
    lib.hb_norm_scan_ex.argtypes = lib.hb_norm_scan.argtypes + [POINTER(Perturbation)]
    lib.hb_norm_topk_ex.restype = c_int
    lib.hb_norm_topk_ex.argtypes = lib.hb_norm_topk.argtypes + [POINTER(Perturbation)]
    lib.hb_norm_scan_noalloc.restype = c_int
    lib.hb_norm_scan_noalloc.argtypes = [P, P, c_int64, c_int64, c_int64, P, P, c_int, c_int, c_int, P, P, P, P, P, P]
    lib.hb_merge_topk.restype = c_int
    lib.hb_merge_topk.argtypes = [P, P, c_int, c_int64, c_int, c_int, P, P, P]
    lib.hb_pair_costs_workspace.restype = c_size_t
    lib.hb_pair_costs.restype = c_int
    lib.hb_pair_costs.argtypes = [c_int, P, P, c_int64, c_int64, c_int64, P, P, c_double, P, P, c_int64, P, P,
                                  c_size_t, P]
    lib.hb_pair_costs_ex.restype = c_int
    lib.hb_pair_costs_ex.argtypes = lib.hb_pair_costs.argtypes + [POINTER(Perturbation)]
    lib.hb_restricted_ot_workspace.restype = c_size_t
    lib.hb_restricted_ot_workspace.argtypes = [c_int64, c_int64, c_int64]
    lib.hb_restricted_ot_solve.restype = c_int
    lib.hb_restricted_ot_solve.argtypes = [P, P, P, c_int64, P, c_int64, c_int64, P, P, POINTER(PdlpControls), P, P,
                                           POINTER(PdlpInfo), POINTER(PdlpTraceRow), c_int32, POINTER(c_int32), P,
                                           c_size_t, P]
    if lib.hb_abi_version() != ABI_VERSION:
        raise HBError(HB_BAD_ARGUMENT, f"libhello_b200 ABI {lib.hb_abi_version()} != {ABI_VERSION}; rebuild")
    _LIB = lib
    return lib


def lib():
    """The loaded library, after checking that a CUDA device is present."""
    if not torch.cuda.is_available():
        raise HBError(HB_CUDA, "hello_ot_b200 requires a CUDA device (B200, sm_100a); there is no CPU path")
    return load_library()


def check(rc: int) -> None:
    if rc != HB_OK:
        msg = (_LIB.hb_last_error() or b"").decode(errors="replace") if _LIB is not None else ""
        if rc in (HB_BAD_ARGUMENT, HB_BAD_INPUT):
            raise ValueError(f"[hello_b200 error {rc}] {msg}")
        raise HBError(rc, msg)


def kernel_launch_count() -> int:
    """Kernels launched by libhello_b200 in this process so far."""
    return int(load_library().hb_kernel_launch_count())


def set_kernel_timing(enable: bool) -> None:
    load_library().hb_set_kernel_timing(int(bool(enable)))


def last_kernel_times() -> list:
    """Device times (ms) of the main kernels of this thread's last call."""
    buf = (c_double * 16)()
    n = load_library().hb_last_kernel_times(buf, 16)
    return [buf[i] for i in range(min(n, 16))]


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_handle(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class Workspace:
    """Grow-only scratch buffer per device, handed to the C ABI as workspace."""

    _buffers: dict = {}

    @classmethod
    def get(cls, device, nbytes: int) -> torch.Tensor:
        key = torch.device(device).index or 0
        buf = cls._buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            cls._buffers[key] = None
            buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            cls._buffers[key] = buf
        return buf

    @classmethod
    def release(cls) -> None:
        cls._buffers.clear()
