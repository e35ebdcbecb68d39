"""Access to the reference package ``hello_ot`` for the end-to-end tests.

The reference (WenzhouXia/hello-ot) is pip-installed, unmodified, into
``baseline/_ref`` (``python -m pip install --no-index --no-build-isolation
--no-deps --target baseline/_ref <copy of the reference>``); that folder travels
with the repository to the GPU box.  Its C++ CPU backend, compiled from the
reference's sources, is ``oracle/_ref/hello_ot_cpp``.  POT, which the reference
uses for its coarsest level, is absent: CPU (``backend="cpp"``) runs use the
HiGHS stand-in of ``oracle/pot_emd.py``; native runs use the plug-in's GPU
leaf solve.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]
REF_SITE = REPO / "baseline" / "_ref"
CPP_SITE = REPO / "oracle" / "_ref"


def available() -> bool:
    return (REF_SITE / "hello_ot" / "__init__.py").exists()


def import_reference(*, cpp: bool = False):
    """Import the installed reference package; with cpp=True also make its C++
    backend and the ot.emd stand-in importable."""
    for p in (str(REF_SITE), str(CPP_SITE)):
        if p not in sys.path:
            sys.path.insert(0, p)
    if cpp:
        from oracle import pot_emd
        pot_emd.install()
    import hello_ot
    return hello_ot


def solve_config(name: str, seed: int = 42):
    """Inputs of the baseline's end-to-end configurations (numpy, fp32 points):
    C1 Brenier ℓ2² 2048 x 32 (examples/quickstart.py), C2 ℓ2 32768 x 3 with
    non-uniform masses, C3 ℓ1 Gaussian mixtures 262144 x 128; ``n=`` overrides
    the size for smaller cases of the same distribution."""
    import bench
    return bench.solve_config(name, seed=seed)
