"""``vb_moe_decode_noalloc``: the decode block on the library's fixed scratch
array instead of a caller workspace, checked against ``vb_moe_decode``.

Collected last on purpose: it must also pass after every other test has used
the library (and alone, in a fresh process).
"""
import ctypes as C

import numpy as np
import pytest

from helpers import bf16_tensor, pool_to_torch, random_pool_np, to_np

NOALLOC_LIMIT = 2 << 20  # VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """Shapes whose workspace exceeds the fixed array fail with a clear error
    before anything touches the device."""
    from vates_b200 import _lib
    assert _lib.lib.vb_moe_decode_workspace_size(4, 2048, 512, 512, 10) <= NOALLOC_LIMIT
    assert _lib.lib.vb_moe_decode_workspace_size(8, 4096, 512, 1024, 16) > NOALLOC_LIMIT
    a = _lib.VbMoeDecodeArgs()
    a.tokens, a.hidden, a.inter, a.group, a.bits = 8, 4096, 512, 64, 4
    a.num_experts, a.top_k = 1024, 16
    rc = _lib.lib.vb_moe_decode_noalloc(C.byref(a), None)
    assert rc == 3  # VB_ERR_WORKSPACE
    assert "scratch" in _lib.lib.vb_last_error().decode()


def _small_block(H, E, k, seed):
    from vates_b200.moe_block import MoeBlock, Workspace
    from vates_b200.pool import QuantPool, make_table
    I = 512
    rng = np.random.default_rng(seed)
    pool = QuantPool.from_tensors(pool_to_torch(random_pool_np(rng, E, H, I)), H, I, 4, 64)
    sh = QuantPool.from_tensors(pool_to_torch(random_pool_np(rng, 1, H, I)), H, I, 4, 64)
    wsg = bf16_tensor(rng.standard_normal(H).astype(np.float32) * 0.02)
    wr = bf16_tensor(rng.standard_normal((E, H)).astype(np.float32) * 0.05)
    return MoeBlock(wr, make_table(E, {e: e for e in range(E)}), pool, sh, wsg, top_k=k,
                    workspace=Workspace())


def _noalloc_vs_workspace(blk, x, call):
    """One call of each entry point on the same inputs; the decode kernel is
    deterministic, so the outputs must be identical bit for bit."""
    import torch
    from vates_b200._lib import check, lib
    from vates_b200.moe_block import Workspace
    from vates_b200.pool import stream_handle
    T = x.shape[0]
    eps = 1e-6
    blk.workspace = Workspace()  # a fresh zero-filled workspace for the reference call
    dbg_ref = blk.new_debug(T)
    st_ref = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = blk.decode(x, residual=x, debug=dbg_ref, status=st_ref, norm_eps=eps)
    out = torch.full_like(x, float("nan"))
    dbg = blk.new_debug(T)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = blk.decode_args(x, out, residual=x, debug=dbg, status=st, norm_eps=eps)
    a.workspace, a.workspace_bytes = None, 0
    check(lib.vb_moe_decode_noalloc(C.byref(a), stream_handle(None)), "vb_moe_decode_noalloc")
    torch.cuda.synchronize()
    assert int(st_ref.item()) == 0 and int(st.item()) == 0, f"call {call}: status"
    for key in ("inds", "local"):
        assert np.array_equal(to_np(dbg[key]), to_np(dbg_ref[key])), f"call {call}: {key}"
    assert torch.equal(dbg["scores"].view(torch.int16), dbg_ref["scores"].view(torch.int16))
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {call}: output"


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_two_calls(cuda):
    from vates_b200.synth import config0, input_tokens
    blk, _ = config0(seed=3)
    for call, seed in enumerate((11, 12)):
        _noalloc_vs_workspace(blk, input_tokens(seed, 4), call)


@pytest.mark.gpu
def test_noalloc_shape_changes_between_calls(cuda):
    """Consecutive calls with different token counts and hidden sizes share
    the array: each must see its counters cleared, whatever the previous
    call left behind. A call rejected for a bad argument in between must
    leave the next call unaffected."""
    import torch
    from vates_b200._lib import lib
    from vates_b200.pool import stream_handle
    from vates_b200.synth import config0, input_tokens
    blk, _ = config0(seed=5)
    wide = _small_block(4096, 32, 4, seed=9)
    assert lib.vb_moe_decode_workspace_size(8, 4096, 512, 32, 4) <= NOALLOC_LIMIT
    rng = np.random.default_rng(3)
    seq = [(blk, 8), (blk, 1), (wide, 8), (blk, 4), (wide, 1), (blk, 8)]
    for call, (b, T) in enumerate(seq):
        x = (input_tokens(100 + call, T) if b is blk else
             bf16_tensor(rng.standard_normal((T, 4096)).astype(np.float32)))
        _noalloc_vs_workspace(b, x, call)
        if call == 2:
            out = torch.empty_like(x)
            a = b.decode_args(x, out)
            a.bits = 3  # rejected before any device work
            assert lib.vb_moe_decode_noalloc(C.byref(a), stream_handle(None)) == 1
