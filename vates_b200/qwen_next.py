"""Qwen3-Next decode stack with MTP speculative verify on the B200 kernels.

Host-side mirror of what the reference runs around its MoE hot path for
end-to-end decode: the mlx-lm 0.31.3 ``qwen3_next`` model (48 layers, three
Gated-DeltaNet layers then one full-attention layer, each followed by the
sparse-MoE block), as patched by the reference (IsoQuant K4/V3 cache on the
full-attention layers, core/cache/kv_quant_patch.py:26-113; per-token
recurrent checkpoints for the verify commit, mtp/kv_cache.py:16-103), the MTP
head (mtp/qwen3_next_mtp.py:21-112, mtp/drafter.py) and the greedy
speculative loop (mtp/generate.py:424-961: draft K tokens, verify, accept the
longest matching prefix, commit, sync the MTP cache).

B200 design: every sequence position (main cache length, MTP cache length,
accepted count) lives in device memory, the recurrent state and conv window
are committed by index instead of copied, and one speculative iteration
(K draft steps, the verify forward, accept, MTP sync) is captured once as a
CUDA graph and replayed; the host only reads the emitted-token counter. All
arithmetic runs in ``libvates_b200`` (no fallback).

Weights are synthetic (the benchmark's random-init model): 4-bit group-64
linears filled on the device by the counter hash of ``vb_synth_fill_u32`` /
``vb_synth_fill_scales``, dense tensors from numpy PCG64 streams, MoE layers
from :func:`vates_b200.synth.make_layer`; ``oracle/qwen_next.py`` rebuilds
the same weights on the CPU.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import check, lib
from .moe_block import MoeBlock, Workspace
from .pool import QuantPool, _mix, ptr, stream_handle
from .quant_kv import build_block_so4, so4_blocks
from .synth import make_layer

# state words (vb_spec_accept)
SP_POS, SP_MTP_POS, SP_ACC, SP_SLOT, SP_PENDING, SP_NOUT, SP_STEPS, SP_HIST = range(8)

# per-tensor seed salts
_IN_PROJ, _OUT_PROJ, _QKV, _O_PROJ, _EMBED, _LM_HEAD, _FC = range(1, 8)


@dataclass(frozen=True)
class QwenNextConfig:
    """Qwen3-Next-80B-A3B shapes (mlx-lm ``ModelArgs``), config 4 by default."""
    hidden: int = 2048
    vocab: int = 151936
    layers: int = 48
    full_attention_interval: int = 4
    q_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 256
    rope_dims: int = 64              # head_dim * partial_rotary_factor 0.25
    rope_base: float = 10_000_000.0
    eps: float = 1e-6
    k_heads: int = 16                # linear_num_key_heads
    v_heads: int = 32                # linear_num_value_heads
    head_k: int = 128
    head_v: int = 128
    experts: int = 512
    top_k: int = 10
    inter: int = 512
    group: int = 64
    bits: int = 4
    # synthetic dense weights: scales U(lo, hi), bias = bias_mul * scale
    dense_scale: tuple = (0.001, 0.01)
    dense_bias_mul: float = -7.5
    expert_bias_mul: float = -8.0    # the MoE blocks of config 0
    unit_norms: bool = True          # random-init RMSNorm weights are 1

    def is_linear(self, layer: int) -> bool:
        return (layer + 1) % self.full_attention_interval != 0

    @property
    def gdn_proj(self) -> int:       # in_proj_qkvz | in_proj_ba rows
        r = self.v_heads // self.k_heads
        return self.k_heads * (2 * self.head_k + 2 * r * self.head_v) + 2 * self.v_heads

    @property
    def conv_dim(self) -> int:
        return 2 * self.k_heads * self.head_k + self.v_heads * self.head_v

    @property
    def value_dim(self) -> int:
        return self.v_heads * self.head_v

    @property
    def attn_proj(self) -> int:      # q_proj (query | gate per head) | k_proj | v_proj
        return self.q_heads * 2 * self.head_dim + 2 * self.kv_heads * self.head_dim

    @property
    def attn_out(self) -> int:
        return self.q_heads * self.head_dim


def tiny_config(**kw) -> QwenNextConfig:
    """A small instance of the same architecture for tests."""
    base = dict(hidden=1024, vocab=2048, layers=4, q_heads=4, kv_heads=1, k_heads=2,
                v_heads=4, experts=16, top_k=4, inter=128, unit_norms=False,
                expert_bias_mul=-7.5)
    base.update(kw)
    return QwenNextConfig(**base)


def tensor_seed(seed: int, layer: int, salt: int) -> int:
    return _mix(_mix(seed, 5000 + layer), salt)


def dense_rng(seed: int, layer: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, 7000 + layer]))


def _bf16(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(device)


def norm_weight(rng, n: int, unit: bool, device) -> torch.Tensor:
    """RMSNorm weight: ones (random init), else N(1, 0.1) in bf16 (tests)."""
    if unit:
        return torch.ones(n, dtype=torch.bfloat16, device=device)
    return _bf16(1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32), device)


class QLinear:
    """A 4-bit group-64 quantized linear ``[out_features, in_features]`` and
    its split-K workspace (sized for 8 tokens, zeroed once)."""

    def __init__(self, out_features: int, in_features: int, seed: int, cfg: QwenNextConfig,
                 device="cuda"):
        self.out_features, self.in_features = out_features, in_features
        self.codes = torch.empty((out_features, in_features // 8), dtype=torch.int32,
                                 device=device)
        self.scales = torch.empty((out_features, in_features // cfg.group),
                                  dtype=torch.bfloat16, device=device)
        self.biases = torch.empty_like(self.scales)
        st = stream_handle()
        check(lib.vb_synth_fill_u32(self.codes.data_ptr(), self.codes.numel(), _mix(seed, 0), st),
              "vb_synth_fill_u32")
        lo, hi = cfg.dense_scale
        check(lib.vb_synth_fill_scales(self.scales.data_ptr(), self.biases.data_ptr(),
                                       self.scales.numel(), _mix(seed, 1), lo, hi,
                                       cfg.dense_bias_mul, st), "vb_synth_fill_scales")
        ws = lib.vb_qlinear_workspace_size(8, in_features, out_features)
        self.ws = torch.zeros(max(ws, 16), dtype=torch.uint8, device=device)

    def __call__(self, x: torch.Tensor, out: torch.Tensor, tokens: int, norm_w=None,
                 eps: float = 1e-6, residual=None, stream=None):
        check(lib.vb_qlinear(x.data_ptr(), tokens, self.in_features, self.codes.data_ptr(),
                             self.scales.data_ptr(), self.biases.data_ptr(),
                             self.out_features, 64, 4, ptr(norm_w), eps, ptr(residual),
                             out.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                             stream_handle(stream)), "vb_qlinear")
        return out


def _i32(t: torch.Tensor, i: int = 0) -> int:
    return t.data_ptr() + 4 * i


@dataclass
class GdnLayer:
    in_proj: QLinear
    conv_w: torch.Tensor
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    norm_w: torch.Tensor
    out_proj: QLinear
    conv_buf: torch.Tensor = None
    states: torch.Tensor = None


@dataclass
class AttnLayer:
    qkv: QLinear
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o_proj: QLinear
    cache: dict = field(default_factory=dict)


@dataclass
class DecoderLayer:
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    mixer: object
    moe: MoeBlock


def _make_attn(cfg, seed, layer, rng, device):
    qkv = QLinear(cfg.attn_proj, cfg.hidden, tensor_seed(seed, layer, _QKV), cfg, device)
    q_norm = norm_weight(rng, cfg.head_dim, cfg.unit_norms, device)
    k_norm = norm_weight(rng, cfg.head_dim, cfg.unit_norms, device)
    o_proj = QLinear(cfg.hidden, cfg.attn_out, tensor_seed(seed, layer, _O_PROJ), cfg, device)
    return AttnLayer(qkv, q_norm, k_norm, o_proj)


def make_decoder_layer(cfg: QwenNextConfig, seed: int, layer: int, moe_ws: Workspace,
                       device="cuda", linear: bool | None = None) -> DecoderLayer:
    """One synthetic decoder layer (weights of ``oracle.qwen_next``)."""
    rng = dense_rng(seed, layer)
    input_norm = norm_weight(rng, cfg.hidden, cfg.unit_norms, device)
    post_norm = norm_weight(rng, cfg.hidden, cfg.unit_norms, device)
    linear = cfg.is_linear(layer) if linear is None else linear
    if linear:
        conv_w = _bf16(rng.uniform(-0.5, 0.5, (cfg.conv_dim, 4)).astype(np.float32), device)
        a_log = torch.from_numpy(np.log(rng.uniform(1.0, 16.0, cfg.v_heads)).astype(np.float32)
                                 ).to(device)
        dt_bias = _bf16(rng.uniform(0.0, 2.0, cfg.v_heads).astype(np.float32), device)
        norm_w = norm_weight(rng, cfg.head_v, cfg.unit_norms, device)
        mixer = GdnLayer(QLinear(cfg.gdn_proj, cfg.hidden, tensor_seed(seed, layer, _IN_PROJ),
                                 cfg, device),
                         conv_w, a_log, dt_bias, norm_w,
                         QLinear(cfg.hidden, cfg.value_dim, tensor_seed(seed, layer, _OUT_PROJ),
                                 cfg, device))
    else:
        mixer = _make_attn(cfg, seed, layer, rng, device)
    pool = QuantPool.empty_blob(cfg.experts, cfg.hidden, cfg.inter, cfg.bits, cfg.group, device)
    moe = make_layer(seed, layer, pool, range(cfg.experts), device, cfg.hidden, cfg.inter,
                     cfg.experts, cfg.top_k, workspace=moe_ws, bias_mul=cfg.expert_bias_mul)
    return DecoderLayer(input_norm, post_norm, mixer, moe)


class QwenNextModel:
    """The main model, its MTP head and the device state of the speculative
    loop. ``max_tokens`` (<= 8) is the largest row count of one forward."""

    def __init__(self, cfg: QwenNextConfig, seed: int = 4, cache_len: int = 8192,
                 verify_len: int = 4, drafts: int = 3, device="cuda", out_cap: int = 65536):
        assert 1 <= verify_len <= drafts + 1 <= 8
        self.cfg, self.seed, self.device = cfg, seed, device
        self.V, self.K = verify_len, drafts
        self.max_t = 8
        self.cache_len = cache_len
        self.moe_ws = Workspace(device)
        self.layers = [make_decoder_layer(cfg, seed, l, self.moe_ws, device)
                       for l in range(cfg.layers)]
        L = cfg.layers
        rng = dense_rng(seed, L + 1)
        self.embed = QLinear(cfg.vocab, cfg.hidden, tensor_seed(seed, L, _EMBED), cfg, device)
        self.final_norm = norm_weight(rng, cfg.hidden, cfg.unit_norms, device)
        self.lm_head = QLinear(cfg.vocab, cfg.hidden, tensor_seed(seed, L, _LM_HEAD), cfg, device)
        # MTP head: norms, fc, one full-attention decoder layer (layer id L)
        self.mtp_norm_emb = norm_weight(rng, cfg.hidden, cfg.unit_norms, device)
        self.mtp_norm_hid = norm_weight(rng, cfg.hidden, cfg.unit_norms, device)
        self.mtp_fc = QLinear(cfg.hidden, 2 * cfg.hidden, tensor_seed(seed, L, _FC), cfg, device)
        self.mtp_layer = make_decoder_layer(cfg, seed, L, self.moe_ws, device, linear=False)
        self.mtp_norm = norm_weight(rng, cfg.hidden, cfg.unit_norms, device)
        # IsoQuant rotations (kv_quant_patch.py:92-93)
        self.rk = so4_blocks(build_block_so4(cfg.head_dim, seed=0), device)
        self.rv = so4_blocks(build_block_so4(cfg.head_dim, seed=1), device)
        # keys and values quantized into the caches by the input-side kernel
        # (vb_attn_prepare_quant); False: bf16 rows, then two appends
        self.fused_append = True
        self.out_cap = out_cap
        self._alloc_buffers()
        self.reset()
        self.graphs = {}

    # ------------------------------------------------------------------ memory
    def _alloc_buffers(self):
        cfg, dev, T = self.cfg, self.device, self.max_t
        bf, f32, i32 = torch.bfloat16, torch.float32, torch.int32
        H, D = cfg.hidden, cfg.head_dim
        cap = self.cache_len
        for lay in self.layers + [self.mtp_layer]:
            m = lay.mixer
            if isinstance(m, GdnLayer):
                m.conv_buf = torch.zeros((3 + T, cfg.conv_dim), dtype=bf, device=dev)
                m.states = torch.zeros((T, cfg.v_heads, cfg.head_v, cfg.head_k), dtype=f32,
                                       device=dev)
            elif lay is self.mtp_layer:
                m.cache = {"k": torch.zeros((cfg.kv_heads, cap, D), dtype=bf, device=dev),
                           "v": torch.zeros((cfg.kv_heads, cap, D), dtype=bf, device=dev)}
            else:
                m.cache = {
                    "kc": torch.zeros((cfg.kv_heads, cap, D * 4 // 32), dtype=i32, device=dev),
                    "ks": torch.zeros((cfg.kv_heads, cap, D // 64), dtype=bf, device=dev),
                    "kb": torch.zeros((cfg.kv_heads, cap, D // 64), dtype=bf, device=dev),
                    "vc": torch.zeros((cfg.kv_heads, cap, D * 3 // 32), dtype=i32, device=dev),
                    "vs": torch.zeros((cfg.kv_heads, cap, D // 64), dtype=bf, device=dev),
                    "vb": torch.zeros((cfg.kv_heads, cap, D // 64), dtype=bf, device=dev)}
        e = lambda *s, dt=bf: torch.zeros(s, dtype=dt, device=dev)
        self.buf = {
            "x0": e(T, H), "x1": e(T, H), "h": e(T, H), "hn": e(T, H),
            "proj": e(T, max(cfg.gdn_proj, cfg.attn_proj)),
            "gq": e(T, cfg.k_heads * cfg.head_k), "gk": e(T, cfg.k_heads * cfg.head_k),
            "gv": e(T, cfg.value_dim), "gg": e(T, cfg.v_heads, dt=f32),
            "gbeta": e(T, cfg.v_heads, dt=f32), "gy": e(T, cfg.value_dim),
            "gout": e(T, max(cfg.value_dim, cfg.attn_out)),
            "q": e(cfg.q_heads, T, D), "krow": e(cfg.kv_heads, T, D),
            "vrow": e(cfg.kv_heads, T, D), "attn": e(cfg.q_heads, T, D),
            "logits": e(T, cfg.vocab), "preds": e(T, dt=i32),
            "cat": e(T, 2 * H), "mtp_h": e(T, H), "sync_h": e(T, H), "sync_ids": e(T, dt=i32),
            "h_last": e(H), "prev_h": e(H),
            "state": e(16, dt=i32), "ids": e(self.K + 1, dt=i32), "out": e(self.out_cap, dt=i32),
            "status": e(1, dt=i32), "prompt": e(cap, dt=i32),
        }
        self.attn_ws = torch.zeros(
            lib.vb_kv_attn_workspace_size(1, cfg.q_heads, T, D, cap) + 256, dtype=torch.uint8,
            device=dev)
        self.argmax_ws = torch.zeros(max(lib.vb_argmax_workspace_size(T), 16),
                                     dtype=torch.uint8, device=dev)
        need = lib.vb_moe_decode_workspace_size(T, cfg.hidden, cfg.inter, cfg.experts,
                                                cfg.top_k)
        self.moe_ws.get(need)

    def reset(self):
        """Empty caches and loop state (before a new prompt)."""
        for lay in self.layers + [self.mtp_layer]:
            m = lay.mixer
            if isinstance(m, GdnLayer):
                m.conv_buf.zero_()
                m.states.zero_()
        self.buf["state"].zero_()
        self.buf["status"].zero_()
        self.buf["h_last"].zero_()
        self.buf["prev_h"].zero_()

    # ------------------------------------------------------------------ layers
    def _gdn(self, m: GdnLayer, lay: DecoderLayer, x, h, T, st, fused: bool = True):
        cfg, b = self.cfg, self.buf
        state = b["state"]
        m.in_proj(x, b["proj"], T, norm_w=lay.input_norm, eps=cfg.eps, stream=st)
        if fused:
            check(lib.vb_gdn_fused(b["proj"].data_ptr(), cfg.gdn_proj, T, cfg.k_heads,
                                   cfg.v_heads, cfg.head_k, cfg.head_v, m.conv_buf.data_ptr(),
                                   self.max_t, _i32(state, SP_ACC), m.conv_w.data_ptr(),
                                   m.a_log.data_ptr(), m.dt_bias.data_ptr(), m.states.data_ptr(),
                                   self.max_t, _i32(state, SP_SLOT), m.norm_w.data_ptr(), cfg.eps,
                                   b["gout"].data_ptr(), b["status"].data_ptr(),
                                   stream_handle(st)), "vb_gdn_fused")
            m.out_proj(b["gout"], h, T, residual=x, stream=st)
            return
        check(lib.vb_gdn_prepare(b["proj"].data_ptr(), cfg.gdn_proj, T, cfg.k_heads, cfg.v_heads,
                                 cfg.head_k, cfg.head_v, m.conv_buf.data_ptr(), self.max_t,
                                 _i32(state, SP_ACC), m.conv_w.data_ptr(), m.a_log.data_ptr(),
                                 m.dt_bias.data_ptr(), b["gq"].data_ptr(), b["gk"].data_ptr(),
                                 b["gv"].data_ptr(), b["gg"].data_ptr(), b["gbeta"].data_ptr(),
                                 b["status"].data_ptr(), stream_handle(st)), "vb_gdn_prepare")
        check(lib.vb_gated_delta_step_at(b["gq"].data_ptr(), b["gk"].data_ptr(),
                                         b["gv"].data_ptr(), b["gg"].data_ptr(), 0,
                                         b["gbeta"].data_ptr(), m.states.data_ptr(), self.max_t,
                                         _i32(state, SP_SLOT), None, b["gy"].data_ptr(), 1, T,
                                         cfg.k_heads, cfg.v_heads, cfg.head_k, cfg.head_v,
                                         stream_handle(st)), "vb_gated_delta_step_at")
        check(lib.vb_gdn_gated_norm(b["gy"].data_ptr(), b["proj"].data_ptr(), cfg.gdn_proj, T,
                                    cfg.k_heads, cfg.v_heads, cfg.head_k, cfg.head_v,
                                    m.norm_w.data_ptr(), cfg.eps, b["gout"].data_ptr(),
                                    stream_handle(st)), "vb_gdn_gated_norm")
        m.out_proj(b["gout"], h, T, residual=x, stream=st)

    def _attn(self, m: AttnLayer, lay: DecoderLayer, x, h, T, st, pos_ptr, mtp=False,
              pos_add=0):
        cfg, b = self.cfg, self.buf
        D = cfg.head_dim
        m.qkv(x, b["proj"], T, norm_w=lay.input_norm, eps=cfg.eps, stream=st)
        if mtp:
            c = m.cache
            check(lib.vb_attn_prepare(b["proj"].data_ptr(), cfg.attn_proj, T, cfg.q_heads,
                                      cfg.kv_heads, D, m.q_norm.data_ptr(), m.k_norm.data_ptr(),
                                      cfg.eps, cfg.rope_dims, cfg.rope_base, pos_ptr, pos_add,
                                      None, b["q"].data_ptr(), c["k"].data_ptr(),
                                      c["v"].data_ptr(), self.cache_len, b["status"].data_ptr(),
                                      stream_handle(st)), "vb_attn_prepare")
            check(lib.vb_kv_bf16_attn_at(b["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(),
                                         1, cfg.q_heads, cfg.kv_heads, T, D, pos_ptr, pos_add,
                                         self.cache_len, self.cache_len, D ** -0.5, 1,
                                         b["proj"].data_ptr(), cfg.attn_proj,
                                         b["gout"].data_ptr(), self.attn_ws.data_ptr(),
                                         self.attn_ws.numel(), stream_handle(st)),
                  "vb_kv_bf16_attn_at")
        else:
            c = m.cache
            if self.fused_append:
                check(lib.vb_attn_prepare_quant(
                    b["proj"].data_ptr(), cfg.attn_proj, T, cfg.q_heads, cfg.kv_heads, D,
                    m.q_norm.data_ptr(), m.k_norm.data_ptr(), cfg.eps, cfg.rope_dims,
                    cfg.rope_base, pos_ptr, self.rk.data_ptr(), self.rv.data_ptr(),
                    b["q"].data_ptr(), self.cache_len, 4, c["kc"].data_ptr(),
                    c["ks"].data_ptr(), c["kb"].data_ptr(), 3, c["vc"].data_ptr(),
                    c["vs"].data_ptr(), c["vb"].data_ptr(), b["status"].data_ptr(),
                    stream_handle(st)), "vb_attn_prepare_quant")
            else:
                check(lib.vb_attn_prepare(b["proj"].data_ptr(), cfg.attn_proj, T, cfg.q_heads,
                                          cfg.kv_heads, D, m.q_norm.data_ptr(),
                                          m.k_norm.data_ptr(), cfg.eps, cfg.rope_dims,
                                          cfg.rope_base, pos_ptr, 0, self.rk.data_ptr(),
                                          b["q"].data_ptr(), b["krow"].data_ptr(),
                                          b["vrow"].data_ptr(), 0, b["status"].data_ptr(),
                                          stream_handle(st)), "vb_attn_prepare")
                for src, rot, key, bits in ((b["krow"], self.rk, "k", 4),
                                            (b["vrow"], self.rv, "v", 3)):
                    check(lib.vb_kv_quant_append_at(src.data_ptr(), rot.data_ptr(), 1,
                                                    cfg.kv_heads, T, D, 64, bits, pos_ptr,
                                                    self.cache_len, c[key + "c"].data_ptr(),
                                                    c[key + "s"].data_ptr(),
                                                    c[key + "b"].data_ptr(),
                                                    b["status"].data_ptr(), stream_handle(st)),
                          "vb_kv_quant_append_at")
            check(lib.vb_kv_decode_attn_at(b["q"].data_ptr(), c["kc"].data_ptr(),
                                           c["ks"].data_ptr(), c["kb"].data_ptr(),
                                           c["vc"].data_ptr(), c["vs"].data_ptr(),
                                           c["vb"].data_ptr(), self.rv.data_ptr(), 1,
                                           cfg.q_heads, cfg.kv_heads, T, D, pos_ptr,
                                           self.cache_len, self.cache_len, 64, 4, 3, D ** -0.5,
                                           1, b["proj"].data_ptr(), cfg.attn_proj,
                                           b["gout"].data_ptr(), self.attn_ws.data_ptr(),
                                           self.attn_ws.numel(), stream_handle(st)),
                  "vb_kv_decode_attn_at")
        # (the output gate is applied by the attention's combine pass)
        m.o_proj(b["gout"], h, T, residual=x, stream=st)

    def _moe(self, lay: DecoderLayer, h, out, T, st):
        cfg, b = self.cfg, self.buf
        if cfg.unit_norms:
            lay.moe.decode(h[:T], out=out[:T], residual=h[:T], norm_eps=cfg.eps, stream=st,
                           status=b["status"])
        else:
            check(lib.vb_rms_norm(h.data_ptr(), None, lay.post_norm.data_ptr(), T, cfg.hidden,
                                  cfg.eps, None, b["hn"].data_ptr(), 0, stream_handle(st)),
                  "vb_rms_norm")
            lay.moe.decode(b["hn"][:T], out=out[:T], residual=h[:T], stream=st,
                           status=b["status"])

    def _layer(self, lay, x, h, out, T, st, pos_ptr, mtp=False, pos_add=0):
        if isinstance(lay.mixer, GdnLayer):
            self._gdn(lay.mixer, lay, x, h, T, st)
        else:
            self._attn(lay.mixer, lay, x, h, T, st, pos_ptr, mtp, pos_add)
        self._moe(lay, h, out, T, st)

    def forward(self, ids_ptr: int, T: int, stream=None):
        """Main model over T rows at the cache position in ``state[0]``:
        embeddings, 48 decoder layers, final norm + lm_head, row argmax.
        Leaves the pre-norm hidden rows in the returned buffer (the MTP
        head's input) and the argmaxes in ``buf['preds']``."""
        cfg, b = self.cfg, self.buf
        st = stream
        state = b["state"]
        x, y = b["x0"], b["x1"]
        check(lib.vb_embed_rows(ids_ptr, T, self.embed.codes.data_ptr(),
                                self.embed.scales.data_ptr(), self.embed.biases.data_ptr(),
                                cfg.vocab, cfg.hidden, 64, 4, x.data_ptr(), b["status"].data_ptr(),
                                stream_handle(st)), "vb_embed_rows")
        for lay in self.layers:
            self._layer(lay, x, b["h"], y, T, st, _i32(state, SP_POS))
            x, y = y, x
        self.lm_head(x, b["logits"], T, norm_w=self.final_norm, eps=cfg.eps, stream=st)
        check(lib.vb_argmax(b["logits"].data_ptr(), T, cfg.vocab, b["preds"].data_ptr(),
                            self.argmax_ws.data_ptr(), self.argmax_ws.numel(),
                            stream_handle(st)), "vb_argmax")
        return x

    def mtp_step(self, ids_ptr: int, hidden: torch.Tensor, T: int, pos_add: int,
                 draft_out: int | None, stream=None):
        """MTP head over T rows at MTP position ``state[1] + pos_add``
        (qwen3_next_mtp.py:40-56): returns the normed hidden H; with
        ``draft_out`` also lm_head + argmax of row 0 into that int32."""
        cfg, b = self.cfg, self.buf
        st = stream
        H = cfg.hidden
        state = b["state"]
        cat = b["cat"]
        # embedding + its norm | hidden norm, the halves of the fc input
        check(lib.vb_mtp_fc_input(ids_ptr, T, self.embed.codes.data_ptr(),
                                  self.embed.scales.data_ptr(), self.embed.biases.data_ptr(),
                                  cfg.vocab, H, self.mtp_norm_emb.data_ptr(),
                                  hidden.data_ptr(), self.mtp_norm_hid.data_ptr(), cfg.eps,
                                  cat.data_ptr(), b["status"].data_ptr(), stream_handle(st)),
              "vb_mtp_fc_input")
        x, y = b["x0"], b["x1"]
        self.mtp_fc(cat, x, T, stream=st)
        self._layer(self.mtp_layer, x, b["h"], y, T, st, _i32(state, SP_MTP_POS), mtp=True,
                    pos_add=pos_add)
        check(lib.vb_rms_norm(y.data_ptr(), None, self.mtp_norm.data_ptr(), T, H, cfg.eps, None,
                              b["mtp_h"].data_ptr(), 0, stream_handle(st)), "vb_rms_norm")
        if draft_out is not None:
            self.lm_head(b["mtp_h"], b["logits"], T, stream=st)
            check(lib.vb_argmax(b["logits"].data_ptr(), 1, cfg.vocab, draft_out,
                                self.argmax_ws.data_ptr(), self.argmax_ws.numel(),
                                stream_handle(st)), "vb_argmax")
        return b["mtp_h"]

    # ------------------------------------------------------------ loop steps
    def prefill_chunk(self, T: int, stream=None):
        """Prompt rows [pos, pos + T) of ``buf['prompt']``: ids, forward,
        commit all rows (generate.py:275-313 prefill_chunked, one chunk)."""
        b = self.buf
        st = stream_handle(stream)
        check(lib.vb_spec_prompt_ids(b["state"].data_ptr(), b["prompt"].data_ptr(),
                                     b["prompt"].numel(), T, b["ids"].data_ptr(), st),
              "vb_spec_prompt_ids")
        vh = self.forward(b["ids"].data_ptr(), T, stream)
        check(lib.vb_spec_accept(b["state"].data_ptr(), b["ids"].data_ptr(), b["preds"].data_ptr(),
                                 T, self.K, 1, vh.data_ptr(), b["h_last"].data_ptr(),
                                 b["prev_h"].data_ptr(), self.cfg.hidden, b["out"].data_ptr(),
                                 self.out_cap, st), "vb_spec_accept")

    def spec_iteration(self, stream=None):
        """One speculative step: K drafts, verify [x, d1..d_{V-1}], accept,
        MTP sync (generate.py:543-900 with drafter.draft / drafter.sync)."""
        b, cfg = self.buf, self.cfg
        st = stream_handle(stream)
        hid = b["h_last"]
        for j in range(self.K):
            hid = self.mtp_step(_i32(b["ids"], j), hid.view(1, cfg.hidden) if hid.dim() == 1
                                else hid, 1, j, _i32(b["ids"], j + 1), stream)
        vh = self.forward(b["ids"].data_ptr(), self.V, stream)
        check(lib.vb_spec_accept(b["state"].data_ptr(), b["ids"].data_ptr(), b["preds"].data_ptr(),
                                 self.V, self.K, 0, vh.data_ptr(), b["h_last"].data_ptr(),
                                 b["prev_h"].data_ptr(), cfg.hidden, b["out"].data_ptr(),
                                 self.out_cap, st), "vb_spec_accept")
        check(lib.vb_spec_sync_inputs(b["state"].data_ptr(), b["ids"].data_ptr(), vh.data_ptr(),
                                      b["prev_h"].data_ptr(), self.V, cfg.hidden,
                                      b["sync_ids"].data_ptr(), b["sync_h"].data_ptr(), st),
              "vb_spec_sync_inputs")
        self.mtp_step(b["sync_ids"].data_ptr(), b["sync_h"], self.V, 0, None, stream)
        check(lib.vb_spec_advance_mtp(b["state"].data_ptr(), st), "vb_spec_advance_mtp")

    # ----------------------------------------------------------------- graphs
    def _graph(self, key, fn):
        g = self.graphs.get(key)
        if g is None:
            # one eager run outside the capture (kernel attributes, lazy
            # init), from a snapshot restored before the capture; the side
            # stream starts after the snapshot's copies
            snap = self.snapshot()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fn(side)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            self.restore(snap)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                fn(side)
            torch.cuda.synchronize()
            self.graphs[key] = g
        return g

    def snapshot(self):
        """Device state that one eager warm-up run may change (restored
        before the capture so the first replay starts from the same point)."""
        snap = {k: self.buf[k].clone() for k in ("state", "ids", "h_last", "prev_h", "out")}
        snap["gdn"] = [(l.mixer.conv_buf.clone(), l.mixer.states.clone())
                       for l in self.layers if isinstance(l.mixer, GdnLayer)]
        return snap

    def restore(self, snap):
        for k in ("state", "ids", "h_last", "prev_h", "out"):
            self.buf[k].copy_(snap[k])
        gl = [l for l in self.layers if isinstance(l.mixer, GdnLayer)]
        for l, (c, s) in zip(gl, snap["gdn"]):
            l.mixer.conv_buf.copy_(c)
            l.mixer.states.copy_(s)

    def prefill(self, prompt_ids, use_graphs: bool = True):
        """Run the prompt through the main model in chunks of ``V`` rows;
        leaves the first generated token pending (ids[0]) and counted."""
        self.reset()
        prompt = torch.as_tensor(np.asarray(prompt_ids, np.int32))
        n = prompt.numel()
        assert 1 <= n and n + 64 <= self.cache_len, "prompt does not fit the caches"
        self.buf["prompt"][:n].copy_(prompt.pin_memory(), non_blocking=True)
        done = 0
        while done < n:
            T = min(self.V, n - done)
            if use_graphs:
                self._graph(("prefill", T), lambda s, T=T: self.prefill_chunk(T, s)).replay()
            else:
                self.prefill_chunk(T)
            done += T
        # the first generated token (generate.py:459-461): produced = [x]
        st = self.buf["state"]
        self.buf["out"][0] = self.buf["ids"][0]
        st[SP_NOUT] = 1
        return self.buf["ids"][0]

    def generate(self, prompt_ids, max_new: int, use_graphs: bool = True):
        """Greedy MTP self-speculative decoding (generate.py:424-961, batch
        verify and direct commit). Returns (tokens, stats)."""
        self.prefill(prompt_ids, use_graphs)
        torch.cuda.synchronize()
        n_out = 1
        while n_out < max_new:
            if use_graphs:
                self._graph(("iter",), lambda s: self.spec_iteration(s)).replay()
            else:
                self.spec_iteration()
            n_out = int(self.buf["state"][SP_NOUT].item())
        st = self.buf["state"].cpu().numpy()
        toks = self.buf["out"][:min(n_out, self.out_cap)].cpu().numpy()[:max_new]
        stats = {"steps": int(st[SP_STEPS]), "tokens": int(len(toks)),
                 "accept_hist": [int(v) for v in st[SP_HIST:SP_HIST + self.V + 1]],
                 "status": int(self.buf["status"].item())}
        return toks, stats
