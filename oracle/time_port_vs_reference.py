"""Time the oracle port of the potential against the reference's own PyTorch path, on CPU.

Test infrastructure. The reference is pure Python and cannot travel to the GPU box, so
the benchmark's CPU leg times the oracle port (``oracle/model_oracle.py``) on the box's
host cores. This script, run where the reference source is available, measures how the
port's speed compares with the reference's ``FlashCartPotential(use_triton=False)``
E+F+stress step on the same inputs, cores and threads, so that the benchmark can state
the correction next to its CPU rate::

    python oracle/time_port_vs_reference.py <reference>/src

Workload: the 192-atom water box with the 128-channel, rank <= 3 architecture of the
MD-scale benchmark, float32, ``torch.set_num_threads(os.cpu_count())``; one warm-up and
three timed steps each, alternated so both see the same machine state. Output:
``oracle/port_vs_reference_cpu.json``.
"""

from __future__ import annotations

import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main(ref_src: str) -> None:
    sys.path.insert(0, ROOT)
    sys.path.insert(1, ref_src)
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    from make_model_golden import _fabric_shim, _Graph

    _fabric_shim()
    from flashcart.model.flashcart import FlashCartPotential as RefPotential  # reference

    from flashcart_b200.data import neighbors, synthetic
    from flashcart_b200.model.flashcart import FlashCartPotential
    from flashcart_b200.model.presets import water_model_kwargs
    from oracle import model_oracle

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    s = synthetic.water_box(4, 4, 4, seed=0)
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    n = len(s["positions"])
    cfg = water_model_kwargs("cfg3arch", ei.shape[1] / n)
    torch.manual_seed(0)
    ref_model = RefPotential(**cfg)
    torch.manual_seed(0)
    sd = FlashCartPotential(**cfg).state_dict()
    g = synthetic.graph_from_structure(s, ei, sh, device="cpu", dtype=torch.float32)
    ref_graph = _Graph({k: g[k] for k in ("positions", "cell", "atom_types", "edge_index", "shifts", "batch",
                                          "n_atoms", "pbc")})

    def ref_step():
        ref_model.predict(ref_graph, compute_forces=True, compute_stress=True)

    def port_step():
        model_oracle.predict(sd, cfg, g)

    ref_step()
    port_step()
    t = {"reference": [], "port": []}
    for _ in range(3):
        for name, fn in (("reference", ref_step), ("port", port_step)):
            t0 = time.perf_counter()
            fn()
            t[name].append(time.perf_counter() - t0)
    med = {k: sorted(v)[len(v) // 2] for k, v in t.items()}
    rec = {"workload": f"E+F+stress of the {n}-atom water box ({ei.shape[1]} edges), 128 channels, ranks <= 3, "
                       "float32, CPU",
           "threads": cores, "reference_s_per_step": med["reference"], "port_s_per_step": med["port"],
           "port_slowdown": med["port"] / med["reference"],
           "reference": "FlashCartPotential(use_triton=False).predict of the reference source"}
    with open(os.path.join(HERE, "port_vs_reference_cpu.json"), "w") as f:
        json.dump(rec, f, indent=1)
    print(json.dumps(rec))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference/src")
