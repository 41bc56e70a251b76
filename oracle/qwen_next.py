"""CPU restatement of the Qwen3-Next decode stack and the MTP speculative loop
(test infrastructure).

The model is mlx-lm 0.31.3 ``models/qwen3_next.py`` (a pinned dependency of
the reference, ``uv.lock:350-352``, not vendored), restated from its published
definition, with the reference's patches:
- Gated-DeltaNet layer in verify mode: mlx_streaming/mtp/kv_cache.py:34-103
  (projection split, conv1d over [state; rows] with per-token window
  checkpoints, SiLU, q/k RMS scaling, sigmoid beta, compute_g, the recurrence
  of ``oracle.gdn``, gated RMSNorm, out_proj);
- full attention with the IsoQuant cache: core/cache/kv_quant_patch.py:26-71
  (q_proj split into query and gate, q_norm / k_norm, RoPE, SO(4) rotations,
  quantized SDPA of ``oracle.isoquant``, inverse V rotation, sigmoid gate,
  o_proj);
- decoder layer h = x + mixer(input_norm(x)); out = h + moe(post_norm(h))
  with the MoE block of ``oracle.moe``;
- the MTP head, mtp/qwen3_next_mtp.py:40-56 (plain bf16 KVCache attention,
  mx.fast.scaled_dot_product_attention in float32);
- the greedy speculative loop, mtp/generate.py:424-900 (drafter.draft, batch
  verify of [x, d1..d_{V-1}], accept_prefix 338-352, direct commit 818-853,
  drafter.sync 178-186).
MLX's dtype chain is kept: float32 inside an op, bf16 at op outputs.

Weights are rebuilt from the same seeds as ``vates_b200.qwen_next`` (counter
hash of ``oracle.synth_np`` for 4-bit linears, numpy PCG64 for dense tensors,
``synth_np.LazyLayer`` for the MoE blocks).
"""
from __future__ import annotations

import numpy as np

from . import gdn as OG
from . import isoquant as OI
from . import mlx_ops as M
from . import moe as OM
from .synth_np import LazyLayer, _mix_int, fill_scales, fill_u32

_IN_PROJ, _OUT_PROJ, _QKV, _O_PROJ, _EMBED, _LM_HEAD, _FC = range(1, 8)


def tensor_seed(seed: int, layer: int, salt: int) -> int:
    return _mix_int(_mix_int(seed, 5000 + layer), salt)


def dense_rng(seed: int, layer: int):
    return np.random.Generator(np.random.PCG64([seed, 7000 + layer]))


def norm_weight(rng, n, unit):
    if unit:
        return np.ones(n, np.float32)
    return M.bf16((1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32))


# --------------------------------------------------------------------- ops
def rms_norm(x, w, eps):
    """``mx.fast.rms_norm(x, w, eps)``: bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)."""
    x = np.asarray(x, np.float32)
    ss = (x.astype(np.float64) ** 2).sum(-1, keepdims=True).astype(np.float32)
    inv = (np.float32(1) / np.sqrt((ss / np.float32(x.shape[-1]) + np.float32(eps))
                                   .astype(np.float32))).astype(np.float32)
    y = M.bf16(x * inv)
    return y if w is None else M.bf16(y * np.asarray(w, np.float32))


class QLinear:
    """4-bit group-64 ``nn.QuantizedLinear`` (MLX quantized_matmul: float32
    accumulation, one bf16 rounding)."""

    def __init__(self, out_f, in_f, seed, scale=(0.001, 0.01), bias_mul=-7.5):
        self.out_f, self.in_f = out_f, in_f
        self._args = (seed, scale, bias_mul)
        self._data = None

    def _materialise(self):
        if self._data is None:
            seed, scale, bias_mul = self._args
            n, i = self.out_f, self.in_f
            codes = fill_u32(n * i // 8, _mix_int(seed, 0)).reshape(n, i // 8)
            s, b = fill_scales(n * i // 64, _mix_int(seed, 1), scale[0], scale[1], bias_mul)
            self._data = (codes, s.reshape(n, i // 64), b.reshape(n, i // 64))
        return self._data

    @property
    def codes(self):
        return self._materialise()[0]

    @property
    def s(self):
        return self._materialise()[1]

    @property
    def b(self):
        return self._materialise()[2]

    def rows(self, r0, r1):
        return M.dequantize(self.codes[r0:r1], self.s[r0:r1], self.b[r0:r1], self.in_f, 64, 4)

    def __call__(self, x, norm_w=None, eps=1e-6, residual=None, chunk=16384):
        x = M.bf16(np.asarray(x, np.float32))
        if norm_w is not None:
            x = rms_norm(x, norm_w, eps)
        y = np.zeros((x.shape[0], self.out_f), np.float32)
        for r0 in range(0, self.out_f, chunk):
            r1 = min(self.out_f, r0 + chunk)
            y[:, r0:r1] = M.matvec_f32(self.rows(r0, r1), x)
        y = M.bf16(y)
        if residual is not None:
            y = M.bf16(M.bf16(np.asarray(residual, np.float32)) + y)
        return y

    def embed(self, ids):
        """``nn.QuantizedEmbedding``: dequantized rows in bf16."""
        ids = np.asarray(ids, np.int64)
        return M.dequantize_bf16(self.codes[ids], self.s[ids], self.b[ids], self.in_f, 64, 4)


def silu_bf16(x):
    x = np.asarray(x, np.float32)
    return M.bf16(x * M.bf16(M.sigmoid_f32(x)))


def softplus_f32(x):
    x = np.asarray(x, np.float32)
    return (np.maximum(x, 0) + np.log1p(np.exp(-np.abs(x)))).astype(np.float32)


def rope(x, pos0, dims, base):
    """mx.fast.rope, traditional=False, over the first ``dims`` of the last
    axis; x [..., T, D] at positions pos0 + t; float32 angles."""
    x = np.asarray(x, np.float32)
    T = x.shape[-2]
    half = dims // 2
    i = np.arange(half, dtype=np.float32)
    inv = np.exp2(-(i / np.float32(half)) * np.float32(np.log2(base))).astype(np.float32)
    pos = (np.arange(T, dtype=np.float32) + np.float32(pos0))[:, None]
    th = (pos * inv[None, :]).astype(np.float32)
    c = np.cos(th.astype(np.float64)).astype(np.float32)
    s = np.sin(th.astype(np.float64)).astype(np.float32)
    x1, x2 = x[..., :half], x[..., half:dims]
    out = x.copy()
    out[..., :half] = M.bf16((x1 * c - x2 * s).astype(np.float32))
    out[..., half:dims] = M.bf16((x1 * s + x2 * c).astype(np.float32))
    return out


def sdpa_f32(q, k, v, scale, causal):
    """mx.fast.scaled_dot_product_attention on bf16 inputs: float32 math,
    bf16 output. q [Hq, L, D], k/v [Hkv, S, D]."""
    Hq, L, D = q.shape
    Hkv, S, _ = k.shape
    rep = Hq // Hkv
    out = np.zeros((Hq, L, D), np.float32)
    for h in range(Hq):
        kv = h // rep
        qs = (q[h] * np.float32(scale)).astype(np.float32)
        sc = (qs.astype(np.float64) @ k[kv].astype(np.float64).T).astype(np.float32)
        if causal:
            qi = np.arange(S - L, S)[:, None]
            sc = np.where(np.arange(S)[None, :] <= qi, sc, -np.inf)
        m = sc.max(-1, keepdims=True)
        e = np.exp(sc - m).astype(np.float32)
        p = (e / e.astype(np.float64).sum(-1, keepdims=True)).astype(np.float32)
        out[h] = (p.astype(np.float64) @ v[kv].astype(np.float64)).astype(np.float32)
    return M.bf16(out)


# --------------------------------------------------------------------- model
class Config:
    """Shapes of ``vates_b200.qwen_next.QwenNextConfig`` (plain attributes)."""

    def __init__(self, **kw):
        self.__dict__.update(kw)

    @classmethod
    def of(cls, cfg):
        return cls(**{k: getattr(cfg, k) for k in cfg.__dataclass_fields__})

    def is_linear(self, layer):
        return (layer + 1) % self.full_attention_interval != 0


class Layer:
    def __init__(self, cfg, seed, layer, linear=None):
        c = cfg
        rng = dense_rng(seed, layer)
        self.input_norm = norm_weight(rng, c.hidden, c.unit_norms)
        self.post_norm = norm_weight(rng, c.hidden, c.unit_norms)
        self.linear = c.is_linear(layer) if linear is None else linear
        ds, bm = tuple(c.dense_scale), c.dense_bias_mul
        if self.linear:
            r = c.v_heads // c.k_heads
            C = 2 * c.k_heads * c.head_k + c.v_heads * c.head_v
            self.conv_w = M.bf16(rng.uniform(-0.5, 0.5, (C, 4)).astype(np.float32))
            self.a_log = np.log(rng.uniform(1.0, 16.0, c.v_heads)).astype(np.float32)
            self.dt_bias = M.bf16(rng.uniform(0.0, 2.0, c.v_heads).astype(np.float32))
            self.norm_w = norm_weight(rng, c.head_v, c.unit_norms)
            proj = c.k_heads * (2 * c.head_k + 2 * r * c.head_v) + 2 * c.v_heads
            self.in_proj = QLinear(proj, c.hidden, tensor_seed(seed, layer, _IN_PROJ), ds, bm)
            self.out_proj = QLinear(c.hidden, c.v_heads * c.head_v,
                                    tensor_seed(seed, layer, _OUT_PROJ), ds, bm)
        else:
            proj = c.q_heads * 2 * c.head_dim + 2 * c.kv_heads * c.head_dim
            self.qkv = QLinear(proj, c.hidden, tensor_seed(seed, layer, _QKV), ds, bm)
            self.q_norm = norm_weight(rng, c.head_dim, c.unit_norms)
            self.k_norm = norm_weight(rng, c.head_dim, c.unit_norms)
            self.o_proj = QLinear(c.hidden, c.q_heads * c.head_dim,
                                  tensor_seed(seed, layer, _O_PROJ), ds, bm)
        self.moe = LazyLayer(seed, layer, c.hidden, c.inter, c.experts, c.expert_bias_mul)


class GdnCache:
    def __init__(self, cfg):
        C = 2 * cfg.k_heads * cfg.head_k + cfg.v_heads * cfg.head_v
        self.conv = np.zeros((3, C), np.float32)
        self.state = np.zeros((cfg.v_heads, cfg.head_v, cfg.head_k), np.float32)
        self.ckpt = None


class QuantKVCache:
    """Rotated, quantized K/V rows per position (AsymmetricQuantizedKVCache)."""

    def __init__(self):
        self.k, self.v = [], []     # per position: packed triples [Hkv, ...]

    def trim(self, n):
        del self.k[n:]
        del self.v[n:]


class Bf16KVCache:
    def __init__(self):
        self.k, self.v = [], []     # per position: [Hkv, D]

    def trim(self, n):
        del self.k[n:]
        del self.v[n:]


def gdn_mixer(cfg, lay: Layer, x, cache: GdnCache):
    """Verify-mode Gated-DeltaNet (kv_cache.py:34-103). Commits all rows and
    keeps per-row checkpoints (conv window, state) in ``cache.ckpt``."""
    c = cfg
    T = x.shape[0]
    Hk, Hv, Dk, Dv = c.k_heads, c.v_heads, c.head_k, c.head_v
    r = Hv // Hk
    W = 2 * Dk + 2 * r * Dv
    proj = lay.in_proj(x, norm_w=lay.input_norm, eps=c.eps)
    qkvz = proj[:, :Hk * W].reshape(T, Hk, W)
    ba = proj[:, Hk * W:Hk * W + 2 * Hv].reshape(T, Hk, 2 * r)
    q = qkvz[:, :, :Dk].reshape(T, -1)
    k = qkvz[:, :, Dk:2 * Dk].reshape(T, -1)
    v = qkvz[:, :, 2 * Dk:2 * Dk + r * Dv].reshape(T, -1)
    z = qkvz[:, :, 2 * Dk + r * Dv:].reshape(T, Hv, Dv)
    b = ba[:, :, :r].reshape(T, Hv)
    a = ba[:, :, r:].reshape(T, Hv)
    mixed = np.concatenate([q, k, v], -1)
    conv_in = np.concatenate([cache.conv, mixed], 0)                     # [3 + T, C]
    conv_ckpt = [conv_in[i + 1:i + 4].copy() for i in range(T)]
    acc = np.zeros((T, conv_in.shape[1]), np.float32)
    for j in range(4):
        acc = (acc + conv_in[j:j + T] * lay.conv_w[:, j][None, :]).astype(np.float32)
    y = silu_bf16(M.bf16(acc))
    qc = y[:, :Hk * Dk].reshape(T, Hk, Dk)
    kc = y[:, Hk * Dk:2 * Hk * Dk].reshape(T, Hk, Dk)
    vc = y[:, 2 * Hk * Dk:].reshape(T, Hv, Dv)
    qn = M.bf16(rms_norm(qc, None, 1e-6) * M.bf16(np.float32(1.0 / Dk)))
    kn = M.bf16(rms_norm(kc, None, 1e-6) * M.bf16(np.float32(Dk ** -0.5)))
    beta = M.bf16(M.sigmoid_f32(b))
    ad = M.bf16(a + lay.dt_bias[None, :])
    g = np.exp(-np.exp(lay.a_log)[None, :] * M.bf16(softplus_f32(ad))).astype(np.float32)
    yr, state, states = OG.gated_delta(qn[None], kn[None], vc[None], g[None], beta[None],
                                       cache.state[None])
    cache.ckpt = [(conv_ckpt[i], states[0, i].copy()) for i in range(T)]
    cache.conv = conv_ckpt[-1]
    cache.state = state[0]
    yr = yr[0]                                                           # [T, Hv, Dv]
    gn = M.swiglu_bf16(z, rms_norm(yr, lay.norm_w, c.eps))
    return lay.out_proj(gn.reshape(T, -1), residual=x)


def attn_mixer(cfg, lay: Layer, x, cache, pos, rk=None, rv=None, quantized=True):
    """Full attention (kv_quant_patch.py:29-71; the MTP layer: plain cache)."""
    c = cfg
    T = x.shape[0]
    D, Hq, Hkv = c.head_dim, c.q_heads, c.kv_heads
    proj = lay.qkv(x, norm_w=lay.input_norm, eps=c.eps)
    qg = proj[:, :Hq * 2 * D].reshape(T, Hq, 2 * D)
    q = qg[..., :D]
    gate = qg[..., D:].reshape(T, Hq * D)
    k = proj[:, Hq * 2 * D:Hq * 2 * D + Hkv * D].reshape(T, Hkv, D)
    v = proj[:, Hq * 2 * D + Hkv * D:].reshape(T, Hkv, D)
    q = rms_norm(q, lay.q_norm, c.eps).transpose(1, 0, 2)               # [Hq, T, D]
    k = rms_norm(k, lay.k_norm, c.eps).transpose(1, 0, 2)
    v = v.transpose(1, 0, 2)
    q = rope(q, pos, c.rope_dims, c.rope_base)
    k = rope(k, pos, c.rope_dims, c.rope_base)
    cache.trim(pos)
    if quantized:
        q = OI.rotate_last(q, rk)
        k = OI.rotate_last(k, rk)
        v = OI.rotate_last(v, rv)
        for t in range(T):
            cache.k.append(OI.kv_quantize(k[:, t], 64, 4))
            cache.v.append(OI.kv_quantize(v[:, t], 64, 3))
        kq = tuple(np.stack([e[i] for e in cache.k], 1)[None] for i in range(3))
        vq = tuple(np.stack([e[i] for e in cache.v], 1)[None] for i in range(3))
        out = OI.asym_quantized_sdpa(q[None], kq, vq, D ** -0.5, 64, 4, 3, causal=T > 1)[0]
        out = OI.rotate_last(out, np.asarray(rv, np.float32).T)
    else:
        for t in range(T):
            cache.k.append(k[:, t].copy())
            cache.v.append(v[:, t].copy())
        ks = np.stack(cache.k, 1)
        vs = np.stack(cache.v, 1)
        out = sdpa_f32(q, ks, vs, D ** -0.5, causal=T > 1)
    out = out.transpose(1, 0, 2).reshape(T, Hq * D)
    gated = M.bf16(out * M.bf16(M.sigmoid_f32(gate)))
    return lay.o_proj(gated, residual=x)


def moe(cfg, lay: Layer, h):
    if cfg.unit_norms:
        return OM.moe_block_decode(h, lay.moe, cfg.top_k, True, norm_eps=cfg.eps,
                                   residual=h)["out"]
    hn = rms_norm(h, lay.post_norm, cfg.eps)
    return OM.moe_block_decode(hn, lay.moe, cfg.top_k, True, residual=h)["out"]


class Model:
    """Main model + MTP head with their caches."""

    def __init__(self, cfg, seed=4):
        c = self.cfg = Config.of(cfg) if not isinstance(cfg, Config) else cfg
        self.seed = seed
        L = c.layers
        self.layers = [Layer(c, seed, l) for l in range(L)]
        rng = dense_rng(seed, L + 1)
        ds, bm = tuple(c.dense_scale), c.dense_bias_mul
        self.embed = QLinear(c.vocab, c.hidden, tensor_seed(seed, L, _EMBED), ds, bm)
        self.final_norm = norm_weight(rng, c.hidden, c.unit_norms)
        self.lm_head = QLinear(c.vocab, c.hidden, tensor_seed(seed, L, _LM_HEAD), ds, bm)
        self.mtp_norm_emb = norm_weight(rng, c.hidden, c.unit_norms)
        self.mtp_norm_hid = norm_weight(rng, c.hidden, c.unit_norms)
        self.mtp_fc = QLinear(c.hidden, 2 * c.hidden, tensor_seed(seed, L, _FC), ds, bm)
        self.mtp_layer = Layer(c, seed, L, linear=False)
        self.mtp_norm = norm_weight(rng, c.hidden, c.unit_norms)
        self.rk = OI.build_block_so4(c.head_dim, seed=0)
        self.rv = OI.build_block_so4(c.head_dim, seed=1)
        self.reset()

    def reset(self):
        self.caches = [GdnCache(self.cfg) if l.linear else QuantKVCache() for l in self.layers]
        self.mtp_cache = Bf16KVCache()
        self.pos = 0
        self.mtp_pos = 0

    def layer_forward(self, i, x, pos):
        lay, c = self.layers[i], self.cfg
        if lay.linear:
            h = gdn_mixer(c, lay, x, self.caches[i])
        else:
            h = attn_mixer(c, lay, x, self.caches[i], pos, self.rk, self.rv)
        return moe(c, lay, h)

    def forward(self, ids):
        """Rows ``ids`` at ``self.pos`` (all committed); returns (logits bf16
        [T, V], pre-norm hidden [T, H])."""
        x = self.embed.embed(ids)
        for i in range(len(self.layers)):
            x = self.layer_forward(i, x, self.pos)
        logits = self.lm_head(x, norm_w=self.final_norm, eps=self.cfg.eps)
        self.pos += len(ids)
        return logits, x

    def commit(self, a, T):
        """Keep the first ``a`` of the last forward's ``T`` rows
        (commit_verified_prefix: KV trim, recurrent checkpoint)."""
        self.pos -= T - a
        for cch in self.caches:
            if isinstance(cch, GdnCache):
                cch.conv, cch.state = cch.ckpt[a - 1]
            else:
                cch.trim(self.pos)

    def mtp(self, hidden, ids, pos):
        """MTP head rows at MTP position ``pos``: (normed H, logits)."""
        c = self.cfg
        emb = rms_norm(self.embed.embed(ids), self.mtp_norm_emb, c.eps)
        hid = rms_norm(hidden, self.mtp_norm_hid, c.eps)
        x = self.mtp_fc(np.concatenate([emb, hid], -1))
        lay = self.mtp_layer
        h = attn_mixer(c, lay, x, self.mtp_cache, pos, quantized=False)
        x = moe(c, lay, h)
        H = rms_norm(x, self.mtp_norm, c.eps)
        return H


def argmax(v):
    return int(np.argmax(np.asarray(v, np.float32)))


def accept_prefix(drafts, preds):
    """generate.py:338-352."""
    matched = 0
    for d, p in zip(drafts, preds):
        if int(p) != int(d):
            break
        matched += 1
    return matched


def spec_generate(model: Model, prompt, max_new, K=3, V=4):
    """Greedy MTP self-speculative decoding, batch verify with direct commit
    (generate.py:424-900; verify feeds [x, d1..d_{V-1}], V <= K + 1).
    Returns (tokens, per-step records)."""
    model.reset()
    prompt = [int(t) for t in prompt]
    logits = hid = None
    for s in range(0, len(prompt), V):
        logits, hid = model.forward(prompt[s:s + V])
    x = argmax(logits[-1])
    H_last = hid[-1:]
    produced = [x]
    steps = []
    prefill_logits = logits[-1]
    while len(produced) < max_new:
        prev_H = H_last
        drafts, h, cur = [], H_last, x
        for j in range(K):
            Hm = model.mtp(h, [cur], model.mtp_pos + j)
            d = argmax(model.lm_head(Hm)[0])
            drafts.append(d)
            h, cur = Hm, d
        model.mtp_cache.trim(model.mtp_pos)
        verify_in = [x] + drafts[:V - 1]
        vlogits, vH = model.forward(verify_in)
        preds = [argmax(r) for r in vlogits]
        matched = accept_prefix(drafts, preds)
        a = min(matched + 1, V)
        model.commit(a, V)
        if matched < V:
            new = drafts[:matched] + [preds[matched]]
        else:
            new = drafts[:V]
        x = new[-1]
        produced.extend(new)
        rH = vH[:a]
        h_seq = np.concatenate([prev_H, rH[:-1]], 0)
        model.mtp(h_seq, verify_in[:a], model.mtp_pos)
        model.mtp_pos += a
        H_last = rH[-1:]
        steps.append({"drafts": drafts, "preds": preds, "matched": matched,
                      "logits": vlogits, "prefill_logits": prefill_logits})
    return produced[:max_new], steps
