"""Regenerate the golden fixtures in this folder from the AMOS144/Vates sources.

Run in a container where the reference checkout is mounted::

    python tests/golden/make_golden.py /path/to/reference

``mlx_streaming/core/cache/quant_kv.py`` imports ``mlx.core`` only for its
array type; ``build_block_so4`` itself is pure numpy (quant_kv.py:49-65). MLX
is not installable here, so this script loads the reference module with a
minimal numpy stand-in for ``mlx.core``/``mlx.utils``/``mlx_lm`` and runs the
reference's own rotation builder. The outputs pin :mod:`oracle.isoquant`
bit-exactly. The route-reduce fixture records the hand-computed expectation of
``mlx_streaming/tests/test_expert_major_prefill.py:89-103`` and the packing
widths of ``mlx_streaming/tests/test_kv_quant.py:64-72``.

Nothing at test time reads the reference: the tests only read the files
written here.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _install_mlx_standin():
    mlx = types.ModuleType("mlx")
    core = types.ModuleType("mlx.core")
    core.array = lambda a, dtype=None: np.asarray(a)
    utils = types.ModuleType("mlx.utils")
    utils.tree_map = lambda fn, tree, *rest: tree
    utils.tree_reduce = lambda fn, tree, init=None: init
    mlx.core = core
    mlx.utils = utils
    mlx_lm = types.ModuleType("mlx_lm")
    models = types.ModuleType("mlx_lm.models")
    cache = types.ModuleType("mlx_lm.models.cache")
    cache.create_attention_mask = lambda *a, **k: None
    sys.modules.update({"mlx": mlx, "mlx.core": core, "mlx.utils": utils,
                        "mlx_lm": mlx_lm, "mlx_lm.models": models,
                        "mlx_lm.models.cache": cache})


def main(ref_root: str) -> None:
    _install_mlx_standin()
    path = os.path.join(ref_root, "mlx_streaming", "core", "cache", "quant_kv.py")
    spec = importlib.util.spec_from_file_location("_vates_quant_kv", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    cases = [(256, 0), (256, 1), (16, 3), (256, 5), (64, 0)]
    for dim, seed in cases:
        R = np.asarray(mod.build_block_so4(dim, seed=seed), dtype=np.float32)
        blocks = np.stack([R[i:i + 4, i:i + 4] for i in range(0, dim, 4)])
        off = R.copy()
        for i in range(0, dim, 4):
            off[i:i + 4, i:i + 4] = 0
        assert not off.any(), "rotation is not block diagonal"
        np.save(os.path.join(HERE, f"so4_d{dim}_seed{seed}_blocks.npy"), blocks)
        print("so4", dim, seed, blocks.shape, float(np.abs(R).sum()))
    fixture = {
        "source": "mlx_streaming/tests/test_expert_major_prefill.py:89-103",
        "previous": [[1.0, -1.0], [2.0, -2.0]],
        "assignment_pos": [3, 0, 2],
        "weighted": [[30.0, 300.0], [10.0, 100.0], [20.0, 200.0]],
        "routes_per_token": 2,
        "expected": [[11.0, 99.0], [52.0, 498.0]],
    }
    with open(os.path.join(HERE, "route_reduce_rank_order.json"), "w") as f:
        json.dump(fixture, f, indent=1)
    widths = {
        "source": "mlx_streaming/tests/test_kv_quant.py:64-72",
        "head_dim": 256, "k_bits": 4, "v_bits": 3,
        "k_words": mod._packed_words(256, 4), "v_words": mod._packed_words(256, 3),
    }
    with open(os.path.join(HERE, "kv_packed_widths.json"), "w") as f:
        json.dump(widths, f, indent=1)
    print("ok", widths)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference checkout>")
    main(sys.argv[1])
