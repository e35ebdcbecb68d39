"""Cost perturbation arguments of the fused norm kernels.

``make_perturbation`` validates the reference's perturbation tuple the way
``generic_scan._norm_perturbation`` does (src/hello_ot/kernels/generic_scan.py:190-205)
and packs it into ``hb_perturbation``.  ``index_hash_coefficients`` restates
``_index_hash_parameters`` (src/hello_ot/costs/metric_perturbation.py:19-33):
per prime (2003, 2011) a source coefficient in [1, p), a target coefficient in
[1, p) and an offset in [0, p) drawn from numpy's default_rng(seed).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from ._lib import Perturbation

INDEX_HASH_PRIMES = (2003, 2011)
MODE_IDS = {"rank2": 0, "index_hash": 1, 0: 0, 1: 1}


def index_hash_coefficients(seed: int) -> tuple:
    rng = np.random.default_rng(int(seed) & ((1 << 63) - 1))
    out = []
    for prime in INDEX_HASH_PRIMES:
        out += [int(rng.integers(1, prime)), int(rng.integers(1, prime)), int(rng.integers(0, prime))]
    return tuple(out)


def make_perturbation(x, y, query_global_index, database_global_index, sigma, seed, mode, row_is_source,
                      coefficients):
    """None when sigma == 0, else (Perturbation struct, the index tensors it points to)."""
    if sigma is None or float(sigma) == 0.0:
        return None
    sigma = float(sigma)
    mode = MODE_IDS.get(mode, mode)
    if not math.isfinite(sigma) or sigma < 0 or mode not in (0, 1):
        raise ValueError("invalid norm perturbation configuration")
    idx = []
    for index, count in ((query_global_index, len(x)), (database_global_index, len(y))):
        if index is None:
            raise ValueError("norm perturbation requires matching CUDA int64 global indices")
        t = torch.as_tensor(index, device=x.device) if not torch.is_tensor(index) else index
        if t.device != x.device or t.dtype != torch.int64 or t.numel() != count:
            raise ValueError("norm perturbation requires matching CUDA int64 global indices")
        idx.append(t.contiguous().view(-1))
    coeffs = [0] * 6
    if mode == 1:
        c = coefficients if coefficients is not None else index_hash_coefficients(seed)
        c = c.detach().cpu().tolist() if torch.is_tensor(c) else list(c)
        if len(c) != 6:
            raise ValueError("index_hash requires six int64 coefficients")
        coeffs = [int(v) for v in c]
    p = Perturbation()
    p.sigma, p.seed, p.mode, p.row_is_source = sigma, int(seed), int(mode), int(bool(row_is_source))
    p.query_index, p.database_index = idx[0].data_ptr(), idx[1].data_ptr()
    for i, v in enumerate(coeffs):
        p.coefficients[i] = v
    return p, idx
