"""vates_b200: B200-native (sm_100a) kernels for the AMOS144/Vates hot path.

- fused quantized MoE (decode/MTP-verify block, expert-major prefill),
- pool slot-table gather,
- IsoQuant K4/V3 KV cache quantize + quantized GQA attention.

Every compute module imports ``vates_b200._lib``, which loads
``libvates_b200.so`` (built in-tree with ``python -m vates_b200.build``) and
raises if it is missing: there is no CPU fallback. The package itself loads
the library on first use of ``lib``/``VbError``/``EXPORTED`` so that the
build step can run before the library exists.
"""
__version__ = "0.1.0"


def __getattr__(name):
    if name in ("lib", "VbError", "EXPORTED", "check"):
        from . import _lib
        return getattr(_lib, name)
    raise AttributeError(name)
