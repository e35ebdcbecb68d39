"""hello_ot_b200: B200-native hot path of HELLO (WenzhouXia/hello-ot).

Pricing scan (tensor-core ℓ2², CUDA-core ℓ1/ℓ∞/ℓ2), active-support pair costs
and the restricted-OT Halpern-PDHG, as hand-written sm_100a CUDA kernels
behind the C ABI of libhello_b200.so (include/hello_b200.h), with host code
that mirrors the reference's scan / pair-cost / PDLP interfaces.

Import name: ``hello_ot_b200`` (the folder is ``hello-ot_b200``; see
``__graft_entry__.load_package``).
"""
from ._lib import (HBError, Workspace, kernel_launch_count, last_kernel_times, lib, load_library,  # noqa: F401
                   set_kernel_timing)
from .scan import (ScanExtension, LowrankBidirScanResult, flatten_candidates, l2sq_last_rescans, l2sq_scan,  # noqa: F401
                   l2sq_topk, norm_scan, norm_topk, raw_lowrank_bidir_feasibility_pricing_scan, scan_routes,
                   topk_bucket)
from .pairs import cost_pairs_lowrank, pair_costs, pair_costs_metric  # noqa: F401
from .pdlp import NativeRestrictedOTPDLP, SolverResult  # noqa: F401
from .support import filter_new_candidate_pairs, select_prune_positions, support_filter  # noqa: F401
from .coarsest import leaf_cost_matrix, solve_leaf_from_cost, solve_leaf_resident  # noqa: F401
from . import generic_scan, perturb  # noqa: F401

__version__ = "0.1.0"
