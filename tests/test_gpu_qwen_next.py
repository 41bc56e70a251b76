"""Qwen3-Next decode stack (GDN + IsoQuant attention + MoE + MTP verify loop)
against the CPU oracle (``oracle/qwen_next.py``).

Layers are compared teacher-forced (the oracle's input fed to the GPU layer)
over two steps, so the conv window, recurrent-state slot and cache offsets of
the second step depend on the first step's commit. Tolerance: the bf16 bar of
the MoE/attention outputs (max-abs 2e-2 scaled to the value, mean-rel 5e-3;
``conftest.bf16_close``)."""
import numpy as np
import pytest

from conftest import bf16_close
from oracle import mlx_ops as M
from oracle import qwen_next as OQ

pytestmark = pytest.mark.gpu


def _np(t):
    import torch
    return t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy()


def _bf(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(M.bf16(a))).to(torch.bfloat16).cuda()


@pytest.fixture(scope="module")
def tiny(cuda):
    from vates_b200.qwen_next import QwenNextModel, tiny_config
    cfg = tiny_config()
    return QwenNextModel(cfg, seed=4, cache_len=512, verify_len=4, drafts=3), OQ.Model(cfg, 4)


@pytest.mark.parametrize("N,K,T,norm,res", [
    (12352, 2048, 4, True, False),     # GDN in_proj, 8-group slices
    (2048, 4096, 4, False, True),      # out_proj / o_proj shape, 4-group slices
    (1000, 1024, 1, True, True),       # ragged row block
    (9216, 2048, 8, True, False),      # attention q|k|v, eight rows
    (300, 256, 3, False, False),       # one slice: direct output
])
def test_qlinear_vs_oracle(cuda, N, K, T, norm, res):
    import torch
    from vates_b200.qwen_next import QLinear, QwenNextConfig
    cfg = QwenNextConfig()
    seed = 1234 + N + K
    g = QLinear(N, K, seed, cfg)
    o = OQ.QLinear(N, K, seed, cfg.dense_scale, cfg.dense_bias_mul)
    rng = np.random.default_rng(N + T)
    x = M.bf16(rng.standard_normal((T, K)).astype(np.float32))
    w = M.bf16((1 + 0.1 * rng.standard_normal(K)).astype(np.float32)) if norm else None
    r = M.bf16(rng.standard_normal((T, N)).astype(np.float32)) if res else None
    y = torch.empty((T, N), dtype=torch.bfloat16, device="cuda")
    g(_bf(x), y, T, norm_w=_bf(w) if norm else None, eps=1e-6, residual=_bf(r) if res else None)
    ref = o(x, norm_w=w, eps=1e-6, residual=r)
    # float32 (GPU) vs float64 (oracle) sums and RMS factors: results agree to
    # one bf16 rounding, two ulps where the values straddle a binade
    bf16_close(_np(y), ref, atol=2e-3, max_ulps=2, frac_beyond=0.05, scale=r,
               what=f"qlinear {N}x{K} T={T}")
    # deterministic and replay-safe (tickets reset): a second call is identical
    y2 = torch.empty_like(y)
    g(_bf(x), y2, T, norm_w=_bf(w) if norm else None, eps=1e-6, residual=_bf(r) if res else None)
    assert torch.equal(y, y2)


def test_synthetic_weights_match_oracle(tiny):
    """The device generator and the oracle build the same model."""
    model, om = tiny
    g0, o0 = model.layers[0], om.layers[0]
    assert np.array_equal(g0.mixer.in_proj.codes.cpu().numpy().view(np.uint32), o0.in_proj.codes)
    assert np.array_equal(M.bf16_bits(_np(g0.mixer.in_proj.scales)), o0.in_proj.s)
    assert np.array_equal(M.bf16_bits(_np(g0.mixer.in_proj.biases)), o0.in_proj.b)
    assert np.array_equal(_np(g0.mixer.conv_w), o0.conv_w)
    assert np.array_equal(g0.mixer.a_log.cpu().numpy(), o0.a_log)
    assert np.array_equal(_np(g0.mixer.dt_bias), o0.dt_bias)
    assert np.array_equal(_np(g0.input_norm), o0.input_norm)
    a3, q3 = model.layers[3], om.layers[3]
    assert np.array_equal(_np(a3.mixer.k_norm), q3.k_norm)
    assert np.array_equal(a3.mixer.o_proj.codes.cpu().numpy().view(np.uint32), q3.o_proj.codes)
    assert np.array_equal(_np(model.mtp_norm), om.mtp_norm)
    assert np.array_equal(model.mtp_fc.codes.cpu().numpy().view(np.uint32), om.mtp_fc.codes)
    assert np.array_equal(_np(a3.moe.router_w), q3.moe["wr"])


def test_embed_and_argmax_exact(tiny):
    import torch
    from vates_b200._lib import check, lib
    model, om = tiny
    cfg = model.cfg
    ids = np.array([0, 5, cfg.vocab - 1, 777], np.int32)
    out = torch.empty((4, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    idt = torch.from_numpy(ids).cuda()
    check(lib.vb_embed_rows(idt.data_ptr(), 4, model.embed.codes.data_ptr(),
                            model.embed.scales.data_ptr(), model.embed.biases.data_ptr(),
                            cfg.vocab, cfg.hidden, 64, 4, out.data_ptr(), None, 0), "embed")
    torch.cuda.synchronize()
    assert np.array_equal(M.bf16_bits(_np(out)), M.bf16_bits(om.embed.embed(ids)))
    rng = np.random.default_rng(3)
    v = M.bf16(rng.standard_normal((5, 151936)).astype(np.float32))
    v[2, 100] = v[2, 7] = 50.0       # tie: the smaller index wins
    vt = _bf(v)
    res = torch.empty(5, dtype=torch.int32, device="cuda")
    ws = torch.zeros(lib.vb_argmax_workspace_size(5), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        check(lib.vb_argmax(vt.data_ptr(), 5, 151936, res.data_ptr(), ws.data_ptr(), ws.numel(), 0),
              "argmax")
        assert res.cpu().tolist() == [int(np.argmax(r)) for r in v]


def _commit_all(model, T):
    from vates_b200.qwen_next import SP_ACC, SP_POS, SP_SLOT
    st = model.buf["state"]
    st[SP_POS] += T
    st[SP_ACC] = T
    st[SP_SLOT] = T - 1


def test_layers_two_steps_vs_oracle(tiny):
    """Every decoder layer, teacher-forced, for a 4-row step and then a 3-row
    step on top of its caches: the mixer (GDN or IsoQuant attention) against
    the oracle mixer on the same input, then the MoE half against the oracle
    MoE block on the GPU's mixer output (each component on identical inputs,
    so a one-ulp difference is not amplified through the next block)."""
    import torch
    from vates_b200.qwen_next import SP_POS, _i32
    model, om = tiny
    model.reset()
    om.reset()
    cfg = model.cfg
    c = om.cfg
    rng = np.random.default_rng(11)
    b = model.buf
    for T in (4, 3):
        pos = om.pos
        for i, lay in enumerate(model.layers):
            x = M.bf16(rng.standard_normal((T, cfg.hidden)).astype(np.float32))
            L = om.layers[i]
            if L.linear:
                href = OQ.gdn_mixer(c, L, x, om.caches[i])
            else:
                href = OQ.attn_mixer(c, L, x, om.caches[i], pos, om.rk, om.rv)
            b["x0"][:T] = _bf(x)
            model._layer(lay, b["x0"], b["h"], b["x1"], T, None, _i32(b["state"], SP_POS))
            torch.cuda.synchronize()
            kind = "gdn" if L.linear else "attn"
            h = _np(b["h"][:T])
            # GDN: one bf16 rounding apart; attention: the quantized SDPA's
            # bf16 scores/probabilities differ by an ulp here and there and
            # o_proj sums them, so the max-abs 2e-2 bar applies
            bf16_close(h, href, atol=2e-3 if L.linear else 2e-2, max_ulps=2, frac_beyond=0.01,
                       scale=x, what=f"layer {i} {kind} mixer T={T}")
            ref = OQ.moe(c, L, h)
            bf16_close(_np(b["x1"][:T]), ref, atol=2e-2, max_ulps=2, frac_beyond=0.01, scale=h,
                       what=f"layer {i} moe T={T}")
        om.pos += T
        _commit_all(model, T)
    assert int(b["status"].item()) == 0


def _gdn_fused_vs_split(model, layer, steps, seed):
    """Run a GDN layer (in_proj -> core -> out_proj) with the fused core and
    with the three-kernel core from the same buffers; outputs, conv windows
    and state checkpoints must be bit-identical."""
    import torch
    from vates_b200.qwen_next import SP_ACC, SP_SLOT
    b, m, cfg = model.buf, layer.mixer, model.cfg
    rng = np.random.default_rng(seed)
    for T, acc in steps:
        if acc is not None:
            b["state"][SP_ACC] = acc
            b["state"][SP_SLOT] = acc - 1
        b["x0"][:T] = _bf(rng.standard_normal((T, cfg.hidden)).astype(np.float32))
        conv0, st0 = m.conv_buf.clone(), m.states.clone()
        model._gdn(m, layer, b["x0"], b["h"], T, None, fused=False)
        torch.cuda.synchronize()
        ref = (b["h"][:T].clone(), m.conv_buf[:3 + T].clone(), m.states[:T].clone())
        m.conv_buf.copy_(conv0)
        m.states.copy_(st0)
        model._gdn(m, layer, b["x0"], b["h"], T, None, fused=True)
        torch.cuda.synchronize()
        assert torch.equal(b["h"][:T], ref[0]), f"out T={T}"
        assert torch.equal(m.conv_buf[:3 + T], ref[1]), f"conv window T={T}"
        assert torch.equal(m.states[:T], ref[2]), f"state checkpoints T={T}"


def test_gdn_fused_equals_three_kernels(tiny):
    """One cluster launch per GDN layer core = prepare + step + gated norm,
    bit for bit, across a commit of 2 of 4 rows and a 3-row step."""
    model, _ = tiny
    model.reset()
    _gdn_fused_vs_split(model, model.layers[0], ((4, None), (3, 2), (1, 3)), 7)


def test_attn_prepare_quant_equals_unfused(tiny):
    """The input side with the IsoQuant append fused in (one launch) = bf16
    rows then two vb_kv_quant_append_at, bit for bit: queries, the K4/V3
    cache rows at positions 5..8 and 9..10, and the attention layer's
    output."""
    import torch
    from vates_b200.qwen_next import AttnLayer, SP_POS
    model, _ = tiny
    model.reset()
    b, cfg = model.buf, model.cfg
    lay = next(l for l in model.layers if isinstance(l.mixer, AttnLayer))
    m = lay.mixer
    rng = np.random.default_rng(11)
    pos_ptr = b["state"].data_ptr() + 4 * SP_POS
    for T, pos in ((4, 5), (2, 9)):
        b["state"][SP_POS] = pos
        b["x0"][:T] = _bf(rng.standard_normal((T, cfg.hidden)).astype(np.float32))
        cache0 = {k: v.clone() for k, v in m.cache.items()}
        outs = []
        for fused in (False, True):
            for k, v in cache0.items():
                m.cache[k].copy_(v)
            model.fused_append = fused
            model._attn(m, lay, b["x0"], b["h"], T, None, pos_ptr)
            torch.cuda.synchronize()
            outs.append((b["h"][:T].clone(), b["q"].clone(),
                         {k: v.clone() for k, v in m.cache.items()}))
        model.fused_append = True
        assert int(b["status"][0].item()) == 0
        assert torch.equal(outs[0][0], outs[1][0]), f"layer output T={T}"
        assert torch.equal(outs[0][1], outs[1][1]), f"queries T={T}"
        for k in ("kc", "ks", "kb", "vc", "vs", "vb"):
            assert torch.equal(outs[0][2][k], outs[1][2][k]), f"cache {k} T={T}"


def test_attn_gate_fused_equals_separate(tiny):
    """The output gate applied in the attention's combine pass = the plain
    attention output followed by vb_attn_gate, bit for bit (IsoQuant cache
    and plain bf16 cache)."""
    import torch
    from vates_b200._lib import lib, check
    from vates_b200.pool import stream_handle
    from vates_b200.qwen_next import AttnLayer, SP_POS
    model, _ = tiny
    model.reset()
    b, cfg = model.buf, model.cfg
    lay = next(l for l in model.layers if isinstance(l.mixer, AttnLayer))
    m, D, T = lay.mixer, cfg.head_dim, 3
    rng = np.random.default_rng(12)
    b["state"][SP_POS] = 6
    pos_ptr = b["state"].data_ptr() + 4 * SP_POS
    b["x0"][:T] = _bf(rng.standard_normal((T, cfg.hidden)).astype(np.float32))
    model._attn(m, lay, b["x0"], b["h"], T, None, pos_ptr)  # fills the caches and b["q"]
    torch.cuda.synchronize()
    c = m.cache
    st = stream_handle()
    plain = torch.empty((cfg.q_heads, T, D), dtype=torch.bfloat16, device="cuda")
    sep = torch.empty((T, cfg.q_heads * D), dtype=torch.bfloat16, device="cuda")
    fused = torch.empty_like(sep)
    for gate, out in ((None, plain), (b["proj"].data_ptr(), fused)):
        check(lib.vb_kv_decode_attn_at(
            b["q"].data_ptr(), c["kc"].data_ptr(), c["ks"].data_ptr(), c["kb"].data_ptr(),
            c["vc"].data_ptr(), c["vs"].data_ptr(), c["vb"].data_ptr(), model.rv.data_ptr(), 1,
            cfg.q_heads, cfg.kv_heads, T, D, pos_ptr, model.cache_len, model.cache_len, 64, 4, 3,
            D ** -0.5, 1, gate, cfg.attn_proj, out.data_ptr(), model.attn_ws.data_ptr(),
            model.attn_ws.numel(), st), "vb_kv_decode_attn_at")
    check(lib.vb_attn_gate(plain.data_ptr(), b["proj"].data_ptr(), cfg.attn_proj, T,
                           cfg.q_heads, sep.data_ptr(), st), "vb_attn_gate")
    torch.cuda.synchronize()
    assert torch.equal(fused, sep)
    # plain bf16 cache (the MTP layer's), keys = pos + pos_add + T
    kc = torch.randn((cfg.kv_heads, model.cache_len, D), device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    for gate, out in ((None, plain), (b["proj"].data_ptr(), fused)):
        check(lib.vb_kv_bf16_attn_at(
            b["q"].data_ptr(), kc.data_ptr(), vc.data_ptr(), 1, cfg.q_heads, cfg.kv_heads, T, D,
            pos_ptr, 2, model.cache_len, model.cache_len, D ** -0.5, 1, gate, cfg.attn_proj,
            out.data_ptr(), model.attn_ws.data_ptr(), model.attn_ws.numel(), st),
            "vb_kv_bf16_attn_at")
    check(lib.vb_attn_gate(plain.data_ptr(), b["proj"].data_ptr(), cfg.attn_proj, T,
                           cfg.q_heads, sep.data_ptr(), st), "vb_attn_gate")
    torch.cuda.synchronize()
    assert torch.equal(fused, sep)


def test_mtp_fc_input_equals_separate(tiny):
    """The MTP fc input in one launch = embedding rows, then the two RMS
    norms into the halves, bit for bit; an id out of range gives a zero
    embedding half and the bounds status."""
    import torch
    from vates_b200._lib import lib, check
    from vates_b200.pool import stream_handle
    model, _ = tiny
    cfg, H, T = model.cfg, model.cfg.hidden, 3
    rng = np.random.default_rng(13)
    st = stream_handle()
    e = model.embed
    ids = torch.from_numpy(rng.integers(0, cfg.vocab, T).astype(np.int32)).cuda()
    hid = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).cuda().to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    emb = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    ref = torch.empty((T, 2 * H), dtype=torch.bfloat16, device="cuda")
    got = torch.empty_like(ref)
    check(lib.vb_embed_rows(ids.data_ptr(), T, e.codes.data_ptr(), e.scales.data_ptr(),
                            e.biases.data_ptr(), cfg.vocab, H, 64, 4, emb.data_ptr(),
                            status.data_ptr(), st), "vb_embed_rows")
    check(lib.vb_rms_norm(emb.data_ptr(), None, model.mtp_norm_emb.data_ptr(), T, H, cfg.eps,
                          None, ref.data_ptr(), 2 * H, st), "vb_rms_norm")
    check(lib.vb_rms_norm(hid.data_ptr(), None, model.mtp_norm_hid.data_ptr(), T, H, cfg.eps,
                          None, ref.data_ptr() + 2 * H, 2 * H, st), "vb_rms_norm")
    check(lib.vb_mtp_fc_input(ids.data_ptr(), T, e.codes.data_ptr(), e.scales.data_ptr(),
                              e.biases.data_ptr(), cfg.vocab, H, model.mtp_norm_emb.data_ptr(),
                              hid.data_ptr(), model.mtp_norm_hid.data_ptr(), cfg.eps,
                              got.data_ptr(), status.data_ptr(), st), "vb_mtp_fc_input")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(got, ref)
    ids[1] = cfg.vocab  # out of range
    check(lib.vb_mtp_fc_input(ids.data_ptr(), T, e.codes.data_ptr(), e.scales.data_ptr(),
                              e.biases.data_ptr(), cfg.vocab, H, model.mtp_norm_emb.data_ptr(),
                              hid.data_ptr(), model.mtp_norm_hid.data_ptr(), cfg.eps,
                              got.data_ptr(), status.data_ptr(), st), "vb_mtp_fc_input")
    torch.cuda.synchronize()
    assert int(status.item()) & 2  # VB_STATUS_BOUNDS
    assert not got[1, :H].float().abs().sum().item()
    assert torch.equal(got[1, H:], ref[1, H:]) and torch.equal(got[0], ref[0])


def test_forward_logits_vs_oracle(tiny):
    """Embeddings -> 4 layers -> final norm + lm_head -> argmax, two chunks,
    free-running. Each block matches on identical inputs (test above); over a
    whole random-init model the small per-block differences compound (about
    2% of the logits), so the bar here is the mean relative error and the
    argmax wherever the oracle's top-2 margin is clear."""
    import torch
    model, om = tiny
    model.reset()
    om.reset()
    cfg = model.cfg
    rng = np.random.default_rng(5)
    for T in (4, 2):
        ids = rng.integers(0, cfg.vocab, T).astype(np.int32)
        idt = torch.from_numpy(ids).cuda()
        model.forward(idt.data_ptr(), T)
        torch.cuda.synchronize()
        ref_logits, ref_h = om.forward(ids.tolist())
        got = _np(model.buf["logits"][:T])
        err = np.abs(got - ref_logits)
        assert err.mean() / np.abs(ref_logits).mean() < 0.05, err.mean()
        preds = model.buf["preds"][:T].cpu().numpy()
        for t in range(T):
            r = ref_logits[t]
            top = np.sort(r)[-2:]
            if top[1] - top[0] > 0.2:      # a clear winner must agree
                assert preds[t] == int(np.argmax(r)), (t, preds[t], int(np.argmax(r)))
        _commit_all(model, T)


def test_mtp_head_vs_oracle(tiny):
    """MTP head rows (plain bf16 cache) at positions 0..2, then a draft at 3."""
    import torch
    from vates_b200.qwen_next import SP_MTP_POS
    model, om = tiny
    model.reset()
    om.reset()
    cfg = model.cfg
    rng = np.random.default_rng(9)
    hid = M.bf16(rng.standard_normal((3, cfg.hidden)).astype(np.float32))
    ids = rng.integers(0, cfg.vocab, 3).astype(np.int32)
    idt = torch.from_numpy(ids).cuda()
    H = model.mtp_step(idt.data_ptr(), _bf(hid), 3, 0, None)
    torch.cuda.synchronize()
    ref = om.mtp(hid, ids.tolist(), 0)
    # fc -> attention -> MoE -> norm chained (not teacher-forced in between)
    bf16_close(_np(H[:3]), ref, atol=2e-2, max_ulps=4, frac_beyond=0.02, what="mtp rows")
    model.buf["state"][SP_MTP_POS] = 3
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    H1 = model.mtp_step(idt.data_ptr() + 4, _bf(hid[1:2]), 1, 0, out.data_ptr())
    torch.cuda.synchronize()
    ref1 = om.mtp(hid[1:2], [int(ids[1])], 3)
    bf16_close(_np(H1[:1]), ref1, atol=2e-2, max_ulps=4, frac_beyond=0.02, what="mtp draft row")
    lg = om.lm_head(ref1)[0]
    top = np.sort(lg)[-2:]
    if top[1] - top[0] > 0.06:
        assert int(out.item()) == int(np.argmax(lg))


def _clear_divergence(got, ref, steps, prefill_logits):
    """Index of the first emitted token where the GPU and the oracle differ
    although the oracle's top-2 logit margin there was clear (> 0.2), else
    None. Every emitted token is the main model's argmax of one verify row:
    row j of the step for the j-th token it emits, the last prefill row for
    the first token."""
    rows = [prefill_logits]
    for s in steps:
        rows.extend(s["logits"][j] for j in range(min(s["matched"] + 1, len(s["logits"]))))
    for i, (g, r) in enumerate(zip(got, ref)):
        if g != r:
            top = np.sort(rows[i])[-2:]
            return i if top[1] - top[0] > 0.2 else None
    return None


@pytest.mark.parametrize("V,K", [(4, 3), (3, 3)])
def test_spec_generate_vs_oracle(tiny, V, K):
    """The device speculative loop (one CUDA graph per iteration) emits the
    oracle's tokens; with V = K the verify feeds x + K-1 drafts as the
    reference's batch mode, with V = K+1 it also verifies the last draft."""
    from vates_b200.qwen_next import QwenNextModel
    model, om = tiny
    if (model.V, model.K) != (V, K):
        model = QwenNextModel(model.cfg, seed=4, cache_len=512, verify_len=V, drafts=K)
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, model.cfg.vocab, 13).tolist()
    toks, stats = model.generate(prompt, 12)
    ref, steps = OQ.spec_generate(om, prompt, 12, K=K, V=V)
    assert stats["status"] == 0
    assert len(toks) == 12
    assert stats["steps"] == len(steps)
    assert _clear_divergence(list(toks), ref, steps, steps[0].get("prefill_logits")) is None, (
        list(toks), ref)


def test_spec_generate_eager_equals_graph(tiny):
    """Graph replay and eager launches give the same tokens."""
    model, _ = tiny
    prompt = list(range(30, 41))
    a, _ = model.generate(prompt, 10, use_graphs=True)
    b, _ = model.generate(prompt, 10, use_graphs=False)
    assert list(a) == list(b)


@pytest.mark.slow
def test_config4_layers_and_loop(cuda):
    """Config 4 shapes (48 layers, 512 experts, vocab 151,936): the first GDN
    and first attention layer against the oracle, then prefill + a few
    speculative iterations with a clean status word."""
    import torch
    from vates_b200.qwen_next import QwenNextConfig, QwenNextModel, SP_POS, _i32
    cfg = QwenNextConfig()
    model = QwenNextModel(cfg, seed=4, cache_len=1024)
    om = OQ.Model(cfg, 4)
    b = model.buf
    rng = np.random.default_rng(2)
    c = om.cfg
    _gdn_fused_vs_split(model, model.layers[0], ((4, None), (4, 1)), 8)
    model.reset()
    for i in (0, 3):
        x = M.bf16(rng.standard_normal((4, cfg.hidden)).astype(np.float32))
        L = om.layers[i]
        if L.linear:
            href = OQ.gdn_mixer(c, L, x, om.caches[i])
        else:
            href = OQ.attn_mixer(c, L, x, om.caches[i], 0, om.rk, om.rv)
        b["x0"][:4] = _bf(x)
        model._layer(model.layers[i], b["x0"], b["h"], b["x1"], 4, None, _i32(b["state"], SP_POS))
        torch.cuda.synchronize()
        h = _np(b["h"][:4])
        bf16_close(h, href, atol=2e-3 if L.linear else 2e-2, max_ulps=2, frac_beyond=0.01,
                   scale=x, what=f"config-4 layer {i} mixer")
        bf16_close(_np(b["x1"][:4]), OQ.moe(c, L, h), atol=2e-2, max_ulps=2, frac_beyond=0.01,
                   scale=h, what=f"config-4 layer {i} moe")
    prompt = rng.integers(0, cfg.vocab, 64).tolist()
    toks, stats = model.generate(prompt, 8)
    assert stats["status"] == 0 and len(toks) == 8
    assert all(0 <= t < cfg.vocab for t in toks)
