"""The C-ABI library loads, exports every declared symbol, validates arguments
and computes host-side layouts (no kernel launches: runs without a GPU)."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT


def _header_symbols():
    src = open(os.path.join(ROOT, "include", "vates_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_header_symbol():
    import vates_b200
    from vates_b200 import _lib
    syms = _header_symbols()
    assert syms, "no declarations found"
    for s in syms:
        assert hasattr(_lib.lib, s), f"library does not export {s}"
    assert set(syms) == set(_lib.EXPORTED), set(syms) ^ set(_lib.EXPORTED)
    assert _lib.lib.vb_version() >= 100


def _header_prototypes():
    """name -> parameter count of every vb_ function the header declares."""
    src = open(os.path.join(ROOT, "include", "vates_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    protos = {}
    for m in re.finditer(r"\b(vb_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", src):
        params = m.group(2).strip()
        protos[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return protos


def test_ctypes_signatures_match_header_arity():
    """Every ctypes declaration has as many arguments as the C prototype:
    a stale Python signature would pass wrong values without an error."""
    from vates_b200 import _lib
    protos = _header_prototypes()
    assert set(protos) == set(_lib.EXPORTED), set(protos) ^ set(_lib.EXPORTED)
    bad = {n: (len(_lib._SIGNATURES[n][1]), k) for n, k in protos.items()
           if len(_lib._SIGNATURES[n][1]) != k}
    assert not bad, f"ctypes vs header argument counts: {bad}"


def test_invalid_arguments_fail_without_launching():
    from vates_b200 import _lib
    a = _lib.VbMoeDecodeArgs()
    a.tokens = 9  # > 8
    rc = _lib.lib.vb_moe_decode(C.byref(a), None)
    assert rc == 1
    assert b"tokens" in _lib.lib.vb_last_error()
    rc = _lib.lib.vb_kv_decode_attn(*([None] * 8), 1, 16, 2, 1, 128, 10, 16, 64, 4, 3,
                                    0.1, 0, None, None, 0, None)
    assert rc == 1 and b"D=256" in _lib.lib.vb_last_error()
    rc = _lib.lib.vb_fused_moe_slots(None, None, None, None, 1, 1, 64, 32, 32, 7, None,
                                     None, None, 0, None)
    assert rc == 1 and b"bits" in _lib.lib.vb_last_error()
    with pytest.raises(_lib.VbError):
        _lib.check(1, "probe")


def test_workspace_sizes_monotone():
    from vates_b200 import _lib
    L = _lib.lib
    a = L.vb_moe_decode_workspace_size(1, 2048, 512, 512, 10)
    b = L.vb_moe_decode_workspace_size(8, 2048, 512, 512, 10)
    assert 0 < a < b
    assert L.vb_fused_moe_workspace_size(40, 512) == 40 * 512 * 4
    assert L.vb_route_reduce_workspace_size(17, 4) >= 17 * 4 * 4


def test_blob_layout_matches_reference_stride():
    # blob_layout.py:14-32 at H=2048, I=512, 4-bit, g64: 1,769,472 B/expert
    from vates_b200.pool import blob_layout
    segs, stride = blob_layout(2048, 512, 4, 64)
    assert stride == 1_769_472
    assert [s[0] for s in segs] == ["gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b",
                                    "down_w", "down_s", "down_b"]
    assert segs[0][3] == 524_288 and segs[1][3] == 32_768
    assert all(off % 16 == 0 for *_, off in segs)
