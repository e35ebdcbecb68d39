"""Record the reference's own end-to-end solve results on the baseline configs.

    python tests/golden/make_solve_golden.py [C1 C2 ...]

Runs the unmodified reference package (``baseline/_ref``) with its C++ CPU
backend (``SolverOptions(backend="cpp")``, built from the reference's sources
into ``oracle/_ref``) on the inputs of ``bench.solve_config`` and writes the
final objective, the relative KKT terms (``hello_ot.progress.final_metrics``),
the refinement iteration count and the wall time to ``solve_reference.json``
beside this script.  POT, the reference's coarsest-level solver, is absent; the
HiGHS stand-in of ``oracle/pot_emd.py`` takes its place (the optimal objective
does not depend on which optimal vertex a leaf returns).  Config 3 (262144²,
d = 128, ℓ1) is out of reach of the CPU backend here (hours per run) and is not
recorded.  The GPU box never runs this script; only the JSON travels.
"""
from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))

import refpkg  # noqa: E402

OUT = HERE / "solve_reference.json"


def run(name: str, perturbation: str):
    hello_ot = refpkg.import_reference(cpp=True)
    from hello_ot.progress import final_metrics

    x, y, a, b, cost = refpkg.solve_config(name)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    r = hello_ot.solve(x, y, source_mass=a, target_mass=b, cost=cost,
                       options=hello_ot.SolverOptions(backend="cpp", num_threads=threads, verbose="off",
                                                      cost_perturbation=perturbation))
    wall = time.perf_counter() - t0
    pfeas, dfeas, gap, kkt = final_metrics(r)
    return {"objective": float(r.objective), "primal_feasibility": pfeas, "dual_feasibility": dfeas, "gap": gap,
            "kkt": kkt, "refinement_iterations": int(r.metadata["total_refinement_iterations"]),
            "wall_s": wall, "threads": threads, "nnz": int(r.solution.values.size)}


def main():
    names = sys.argv[1:] or ["C1", "C2"]
    data = json.loads(OUT.read_text()) if OUT.exists() else {}
    for name in names:
        for pert in ("off", "auto"):
            key = f"{name}/{pert}"
            data[key] = run(name, pert)
            print(key, data[key], flush=True)
            OUT.write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
