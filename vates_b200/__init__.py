"""vates_b200: B200-native (sm_100a) kernels for the AMOS144/Vates hot path.

- fused quantized MoE (decode/MTP-verify block, expert-major prefill),
- pool slot-table gather,
- IsoQuant K4/V3 KV cache quantize + quantized GQA attention.

Importing the package loads ``libvates_b200.so`` (built in-tree with
``python -m vates_b200.build``); without it the import fails: there is no CPU
fallback.
"""
from ._lib import lib, VbError, EXPORTED  # noqa: F401  (loads the library)

__version__ = "0.1.0"
