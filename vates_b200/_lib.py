"""ctypes binding of ``libvates_b200.so`` (the C ABI in ``include/vates_b200.h``).

The library is built in-tree by :mod:`vates_b200.build`. There is no fallback:
if the library is missing or fails to load, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvates_b200.so")

VB_OK = 0
VB_STATUS_MISS = 1
VB_STATUS_BOUNDS = 2
VB_STATUS_TIMEOUT = 4
VB_ERR_CAPACITY = 4
VB_DECODE_ROUTE_ONLY = 1


class VbQuantPool(C.Structure):
    _fields_ = [("ptr", C.c_void_p * 9), ("slot_stride", C.c_int64 * 9),
                ("cap", C.c_int32), ("reserved", C.c_int32)]


class VbMoeDecodeArgs(C.Structure):
    _fields_ = [
        ("tokens", C.c_int32), ("hidden", C.c_int32), ("inter", C.c_int32),
        ("group", C.c_int32), ("bits", C.c_int32), ("num_experts", C.c_int32),
        ("top_k", C.c_int32), ("norm_topk", C.c_int32),
        ("norm_eps", C.c_float), ("flags", C.c_int32),
        ("x", C.c_void_p), ("router_w", C.c_void_p), ("router_bias", C.c_void_p),
        ("slot_table", C.c_void_p), ("pool", VbQuantPool), ("shared", VbQuantPool),
        ("shared_gate_w", C.c_void_p), ("residual", C.c_void_p), ("out", C.c_void_p),
        ("out_inds", C.c_void_p), ("out_scores", C.c_void_p), ("out_local", C.c_void_p),
        ("status", C.c_void_p), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("timing_events", C.c_void_p), ("trace", C.c_void_p),
    ]


class VbMoePrefillArgs(C.Structure):
    _fields_ = [
        ("tokens", C.c_int32), ("hidden", C.c_int32), ("inter", C.c_int32),
        ("group", C.c_int32), ("bits", C.c_int32), ("num_experts", C.c_int32),
        ("top_k", C.c_int32), ("norm_topk", C.c_int32),
        ("layer_cap", C.c_int32), ("max_assignments", C.c_int32),
        ("x", C.c_void_p), ("router_w", C.c_void_p), ("router_bias", C.c_void_p),
        ("slot_table", C.c_void_p), ("pool", VbQuantPool), ("shared", VbQuantPool),
        ("shared_gate_w", C.c_void_p), ("out", C.c_void_p),
        ("out_inds", C.c_void_p), ("out_scores", C.c_void_p), ("out_logits", C.c_void_p),
        ("status", C.c_void_p), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
    ]


class VbMoePrefillEpArgs(C.Structure):
    _fields_ = [("base", VbMoePrefillArgs), ("owner", C.c_void_p), ("world", C.c_int32),
                ("rank", C.c_int32), ("max_tokens_per_rank", C.c_int32),
                ("reserved", C.c_int32)]


class VbMoeRouteArgs(C.Structure):
    _fields_ = [
        ("tokens", C.c_int32), ("hidden", C.c_int32), ("num_experts", C.c_int32),
        ("top_k", C.c_int32), ("norm_topk", C.c_int32), ("reserved0", C.c_int32),
        ("x", C.c_void_p), ("router_w", C.c_void_p), ("router_bias", C.c_void_p),
        ("shared_gate_w", C.c_void_p), ("out_inds", C.c_void_p), ("out_scores", C.c_void_p),
        ("out_sgate", C.c_void_p), ("out_counts", C.c_void_p), ("out_logits", C.c_void_p),
        ("status", C.c_void_p), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
    ]


class VbMoeExpertsArgs(C.Structure):
    _fields_ = [
        ("rows", C.c_int32), ("routes", C.c_int32), ("hidden", C.c_int32), ("inter", C.c_int32),
        ("group", C.c_int32), ("bits", C.c_int32), ("num_experts", C.c_int32),
        ("reserved0", C.c_int32),
        ("x", C.c_void_p), ("route_row", C.c_void_p), ("route_expert", C.c_void_p),
        ("route_score", C.c_void_p), ("slot_table", C.c_void_p),
        ("pool", VbQuantPool), ("shared", VbQuantPool),
        ("out", C.c_void_p), ("status", C.c_void_p), ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
    ]


class VbMoeCombineArgs(C.Structure):
    _fields_ = [
        ("tokens", C.c_int32), ("hidden", C.c_int32), ("num_experts", C.c_int32),
        ("top_k", C.c_int32), ("layer_cap", C.c_int32), ("max_assignments", C.c_int32),
        ("inds", C.c_void_p), ("counts", C.c_void_p), ("y_routes", C.c_void_p),
        ("route_row", C.c_void_p), ("y_shared", C.c_void_p), ("shared_row", C.c_void_p),
        ("sgate", C.c_void_p), ("out", C.c_void_p), ("group_of_ws", C.c_void_p),
    ]


class VbEpPackArgs(C.Structure):
    _fields_ = [
        ("tokens", C.c_int32), ("top_k", C.c_int32), ("hidden", C.c_int32), ("world", C.c_int32),
        ("x", C.c_void_p), ("inds", C.c_void_p), ("scores", C.c_void_p), ("owner", C.c_void_p),
        ("send_x", C.c_void_p), ("send_meta", C.c_void_p), ("route_send_idx", C.c_void_p),
        ("dest_rows", C.c_void_p), ("dest_routes", C.c_void_p), ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
    ]


_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64
_SZ = C.c_size_t

_SIGNATURES = {
    "vb_version": (_I32, []),
    "vb_last_error": (C.c_char_p, []),
    "vb_slot_remap": (_I32, [_P, _P, _P, _I64, _I32, _P, _P, _P]),
    "vb_fused_moe_workspace_size": (_SZ, [_I32, _I32]),
    "vb_fused_moe_slots": (_I32, [_P, _P, _P, C.POINTER(VbQuantPool), _I32, _I32, _I32,
                                  _I32, _I32, _I32, _P, _P, _P, _SZ, _P]),
    "vb_fused_moe_pairs": (_I32, [_P, _P, _P, C.POINTER(VbQuantPool), _I32, _I32, _I32,
                                  _I32, _I32, _P, _P, _P, _SZ, _P]),
    "vb_moe_decode_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32]),
    "vb_moe_decode": (_I32, [C.POINTER(VbMoeDecodeArgs), _P]),
    "vb_moe_decode_noalloc": (_I32, [C.POINTER(VbMoeDecodeArgs), _P]),
    "vb_moe_prefill_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32]),
    "vb_moe_prefill": (_I32, [C.POINTER(VbMoePrefillArgs), _P]),
    "vb_moe_prefill_ep_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32, _I32, _I32]),
    "vb_moe_prefill_ep": (_I32, [C.POINTER(VbMoePrefillEpArgs), _P, _P]),
    "vb_moe_route_workspace_size": (_SZ, [_I32, _I32, _I32]),
    "vb_moe_route": (_I32, [C.POINTER(VbMoeRouteArgs), _P]),
    "vb_moe_experts_workspace_size": (_SZ, [_I32, _I32, _I32, _I32]),
    "vb_moe_experts": (_I32, [C.POINTER(VbMoeExpertsArgs), _P]),
    "vb_moe_combine": (_I32, [C.POINTER(VbMoeCombineArgs), _P]),
    "vb_ep_pack_workspace_size": (_SZ, [_I32, _I32]),
    "vb_ep_pack": (_I32, [C.POINTER(VbEpPackArgs), _P]),
    "vb_ep_unpack": (_I32, [_P, _I32, _P, _P, _I32, _P, _P, _P, _P]),
    "vb_route_reduce_workspace_size": (_SZ, [_I32, _I32]),
    "vb_route_reduce": (_I32, [_P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P,
                               _SZ, _P]),
    "vb_kv_quant_append": (_I32, [_P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                                  _I32, _P, _P, _P, _P]),
    "vb_so4_rotate": (_I32, [_P, _P, _I64, _I32, _I32, _P, _P]),
    "vb_kv_attn_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32]),
    "vb_kv_decode_attn": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32,
                                 _I32, _I32, _I32, _I32, _I32, _I32, C.c_float, _I32, _P,
                                 _P, _SZ, _P]),
    "vb_res_create": (_P, [_I32, _I32, _I32, _I32, _I32]),
    "vb_res_destroy": (None, [_P]),
    "vb_res_demand": (_I32, [_P, _I32, _P, _I32, _P, _P, _P, _P, _P]),
    "vb_res_pin": (_I32, [_P, _I32, _P, _I32, _P, _P, _P]),
    "vb_res_table": (_I32, [_P, _I32, _P]),
    "vb_res_counts": (_I32, [_P, _I32, _P]),
    "vb_res_resident": (_I32, [_P, _I32, _P, _P, _P]),
    "vb_pool_fill": (_I32, [C.POINTER(VbQuantPool), _I32, _I32, _I32, _I32, _P, _P, _I32,
                            _P]),
    "vb_blob_gather": (_I32, [_P, _I64, _P, _P, _I32, _P, _P]),
    "vb_moe_decode_resident": (_I32, [C.POINTER(VbMoeDecodeArgs), _P, _I32, _P, _I64, _I32, _P,
                                      _P]),
    "vb_kv_prefill_attn": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32,
                                  _I32, _I32, _I32, _I32, _I32, _I32, C.c_float, _I32, _P, _P,
                                  _P]),
    "vb_dequantize": (_I32, [_P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P]),
    "vb_gated_delta_step": (_I32, [_P, _P, _P, _P, _I32, _P, _P, _P, _P, _P, _P, _I32, _I32,
                                   _I32, _I32, _I32, _I32, _P]),
    "vb_gated_delta_step_at": (_I32, [_P, _P, _P, _P, _I32, _P, _P, _I32, _P, _P, _P, _I32,
                                      _I32, _I32, _I32, _I32, _I32, _P]),
    "vb_kv_quant_append_at": (_I32, [_P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I32, _P,
                                     _P, _P, _P, _P]),
    "vb_kv_decode_attn_at": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32,
                                    _I32, _P, _I32, _I32, _I32, _I32, _I32, C.c_float, _I32,
                                    _P, _I32, _P, _P, _SZ, _P]),
    "vb_kv_bf16_attn_at": (_I32, [_P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _I32, _I32,
                                  _I32, C.c_float, _I32, _P, _I32, _P, _P, _SZ, _P]),
    "vb_qlinear_workspace_size": (_SZ, [_I32, _I32, _I32]),
    "vb_qlinear": (_I32, [_P, _I32, _I32, _P, _P, _P, _I32, _I32, _I32, _P, C.c_float, _P, _P,
                          _P, _SZ, _P]),
    "vb_rms_norm": (_I32, [_P, _P, _P, _I32, _I32, C.c_float, _P, _P, _I32, _P]),
    "vb_argmax_workspace_size": (_SZ, [_I32]),
    "vb_argmax": (_I32, [_P, _I32, _I32, _P, _P, _SZ, _P]),
    "vb_embed_rows": (_I32, [_P, _I32, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P, _P]),
    "vb_gdn_prepare": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I32, _P, _P, _P, _P,
                              _P, _P, _P, _P, _P, _P, _P]),
    "vb_gdn_fused": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I32, _P, _P, _P, _P, _P,
                            _I32, _P, _P, C.c_float, _P, _P, _P]),
    "vb_gdn_gated_norm": (_I32, [_P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P, C.c_float, _P,
                                 _P]),
    "vb_attn_prepare": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _P, _P, C.c_float, _I32,
                               C.c_float, _P, _I32, _P, _P, _P, _P, _I32, _P, _P]),
    "vb_attn_prepare_quant": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _P, _P, C.c_float,
                                     _I32, C.c_float, _P, _P, _P, _P, _I32, _I32, _P, _P, _P,
                                     _I32, _P, _P, _P, _P, _P]),
    "vb_attn_gate": (_I32, [_P, _P, _I32, _I32, _I32, _P, _P]),
    "vb_mtp_fc_input": (_I32, [_P, _I32, _P, _P, _P, _I32, _I32, _P, _P, _P, C.c_float, _P, _P,
                               _P]),
    "vb_spec_accept": (_I32, [_P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _I32, _P]),
    "vb_spec_sync_inputs": (_I32, [_P, _P, _P, _P, _I32, _I32, _P, _P, _P]),
    "vb_spec_advance_mtp": (_I32, [_P, _P]),
    "vb_spec_prompt_ids": (_I32, [_P, _P, _I32, _I32, _P, _P]),
    "vb_synth_fill_u32": (_I32, [_P, _I64, C.c_uint64, _P]),
    "vb_synth_fill_pool": (_I32, [C.POINTER(VbQuantPool), _P, _P, _I32, _I32, _I32, _I32,
                                  _I32, C.c_float, C.c_float, C.c_float, _P]),
    "vb_synth_fill_scales": (_I32, [_P, _P, _I64, C.c_uint64, C.c_float, C.c_float,
                                    C.c_float, _P]),
}

# Every symbol the header declares (tests check the library exports them).
EXPORTED = tuple(_SIGNATURES)


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"vates_b200: {LIB_PATH} is missing; build it with "
            "`python -m vates_b200.build` (there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class VbError(RuntimeError):
    """A vates_b200 C-ABI call returned a non-zero status."""


def check(rc: int, what: str) -> None:
    if rc != VB_OK:
        msg = lib.vb_last_error().decode(errors="replace")
        raise VbError(f"{what} failed (status {rc}): {msg}")
