"""``vb_moe_decode_noalloc``: the decode block on the library's fixed scratch
array instead of a caller workspace, checked against ``vb_moe_decode``.

Collected last on purpose: it must also pass after every other test has used
the library (and alone, in a fresh process).
"""
import ctypes as C

import numpy as np
import pytest

from conftest import bf16_close
from helpers import to_np


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """Shapes whose workspace exceeds the fixed array fail with a clear error
    before anything touches the device."""
    from vates_b200 import _lib
    limit = 2 << 20  # VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES
    assert _lib.lib.vb_moe_decode_workspace_size(4, 2048, 512, 512, 10) <= limit
    assert _lib.lib.vb_moe_decode_workspace_size(8, 4096, 512, 1024, 16) > limit
    a = _lib.VbMoeDecodeArgs()
    a.tokens, a.hidden, a.inter, a.group, a.bits = 8, 4096, 512, 64, 4
    a.num_experts, a.top_k = 1024, 16
    rc = _lib.lib.vb_moe_decode_noalloc(C.byref(a), None)
    assert rc == 3  # VB_ERR_WORKSPACE
    assert "scratch" in _lib.lib.vb_last_error().decode()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_two_calls(cuda):
    import torch
    from vates_b200._lib import check, lib
    from vates_b200.pool import stream_handle
    from vates_b200.synth import config0, input_tokens

    blk, _ = config0(seed=3)
    eps = 1e-6
    for call, seed in enumerate((11, 12)):
        x = input_tokens(seed, 4)
        # existing entry point, caller workspace
        dbg_ref = blk.new_debug(4)
        st_ref = torch.zeros(1, dtype=torch.int32, device="cuda")
        ref = blk.decode(x, residual=x, debug=dbg_ref, status=st_ref, norm_eps=eps)
        # fixed-scratch entry point through the C ABI
        out = torch.full_like(x, float("nan"))
        dbg = blk.new_debug(4)
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        a = blk.decode_args(x, out, residual=x, debug=dbg, status=st, norm_eps=eps)
        a.workspace, a.workspace_bytes = None, 0
        check(lib.vb_moe_decode_noalloc(C.byref(a), stream_handle(None)),
              "vb_moe_decode_noalloc")
        torch.cuda.synchronize()
        assert int(st_ref.item()) == 0 and int(st.item()) == 0, f"call {call}: status"
        assert np.array_equal(to_np(dbg["inds"]), to_np(dbg_ref["inds"])), f"call {call}: routes"
        assert np.array_equal(to_np(dbg["scores"]), to_np(dbg_ref["scores"]))
        assert np.array_equal(to_np(dbg["local"]), to_np(dbg_ref["local"]))
        bf16_close(to_np(out), to_np(ref), what=f"noalloc call {call} vs vb_moe_decode")
