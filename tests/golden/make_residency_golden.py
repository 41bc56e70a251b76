"""Regenerate ``residency_refreal.json`` from the AMOS144/Vates sources.

Run in a container where the reference checkout is mounted::

    python tests/golden/make_residency_golden.py /path/to/reference

``mlx_streaming/tests/test_demand_dual_native.py:760-823`` holds ``RefReal``,
the reference's own pure-Python model of its native demand state machine, and
``test_cpp_matches_ref_over_random_sequence`` (826-840) drives it with
``random.Random(12345)``, cap 4, 200 requests of 1..cap ids in [0, 10). The
test module imports MLX at the top, so this script takes only the ``RefReal``
class out of the file (``ast``) and runs it. It records that sequence and a few
more (LFU off, decay on, larger caps) with the reference's outputs: the slot of
every requested id and the resident set after every request. The fixture pins
:mod:`oracle.residency` and the native manager; nothing at test time reads the
reference.
"""
from __future__ import annotations

import ast
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

# (seed, cap, lfu, decay, ids_below, steps); the first is the reference test's.
CASES = [(12345, 4, True, 0, 10, 200), (7, 4, False, 0, 10, 200), (99, 6, True, 5, 16, 300),
         (2024, 8, True, 0, 24, 300), (31, 3, True, 2, 8, 200)]


def load_refreal(ref_root: str):
    path = os.path.join(ref_root, "mlx_streaming", "tests", "test_demand_dual_native.py")
    tree = ast.parse(open(path).read())
    cls = [n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "RefReal"]
    assert len(cls) == 1, "RefReal not found"
    mod = ast.Module(body=cls, type_ignores=[])
    ns: dict = {}
    exec(compile(mod, path, "exec"), ns)
    return ns["RefReal"]


def main(ref_root: str) -> None:
    RefReal = load_refreal(ref_root)
    cases = []
    for seed, cap, lfu, decay, below, steps in CASES:
        rng = random.Random(seed)
        ref = RefReal(cap, lfu, decay)
        reqs, locals_, resident = [], [], []
        for _ in range(steps):
            flat = [rng.randint(0, below - 1) for _ in range(rng.randint(1, cap))]
            reqs.append(flat)
            locals_.append(ref.place(flat))
            resident.append(sorted(ref.e2r.items()))
        cases.append({"seed": seed, "cap": cap, "lfu": lfu, "decay": decay,
                      "num_experts": below, "requests": reqs, "local": locals_,
                      "resident": resident})
        print("case", seed, cap, lfu, decay, "final", sorted(ref.e2r))
    fixture = {"source": "mlx_streaming/tests/test_demand_dual_native.py:760-840 (RefReal)",
               "cases": cases}
    with open(os.path.join(HERE, "residency_refreal.json"), "w") as f:
        json.dump(fixture, f, separators=(",", ":"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference checkout>")
    main(sys.argv[1])
