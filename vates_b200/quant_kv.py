"""IsoQuant K4/V3 quantized KV cache on B200.

Mirror of mlx_streaming/core/cache/quant_kv.py (rotation builder, rotation,
AsymmetricQuantizedKVCache, asym_quantized_sdpa) and the rotated attention of
kv_quant_patch.py:26-71, over torch CUDA tensors. Packing, rotation and
attention run in ``libvates_b200``.

Cache storage per tensor (K or V) is the MLX quantize triple
``(codes uint32 [B,H,steps,D*bits/32], scales bf16 [B,H,steps,D/64],
biases bf16 [B,H,steps,D/64])`` grown in multiples of 256 steps
(quant_kv.py:86-125). Codes are stored as int32 tensors (same bits).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import check, lib
from .pool import ptr, stream_handle


# ----------------------------- SO(4) block rotation --------------------------

def _left_mult(q):
    w, x, y, z = q
    return np.array([[w, -x, -y, -z], [x, w, -z, y], [y, z, w, -x], [z, -y, x, w]],
                    dtype=np.float32)


def _right_conj_mult(q):
    w, x, y, z = q
    return np.array([[w, x, y, z], [-x, w, z, -y], [-y, -z, w, x], [-z, y, -x, w]],
                    dtype=np.float32)


def build_block_so4(head_dim: int, seed: int = 0, blocks_of: int = 4) -> torch.Tensor:
    """Block-diagonal rotation with one SO(4) block per 4 dims
    (quant_kv.py:49-65): per block two unit quaternions drawn (left, then
    right) as float32 normals from ``numpy.random.default_rng(seed)``; block =
    L(q_left) @ R(conj q_right). Returns a float32 CPU tensor [D, D]."""
    if head_dim % blocks_of:
        raise ValueError("head_dim must be a multiple of blocks_of")
    rng = np.random.default_rng(seed)
    R = np.zeros((head_dim, head_dim), dtype=np.float32)
    for b in range(head_dim // blocks_of):
        ql = rng.standard_normal(4).astype(np.float32)
        ql /= np.linalg.norm(ql)
        qr = rng.standard_normal(4).astype(np.float32)
        qr /= np.linalg.norm(qr)
        i = b * blocks_of
        R[i:i + blocks_of, i:i + blocks_of] = _left_mult(ql) @ _right_conj_mult(qr)
    return torch.from_numpy(R)


def so4_blocks(R: torch.Tensor, device="cuda") -> torch.Tensor:
    """The [D/4, 4, 4] diagonal blocks of a block-diagonal rotation (float32)."""
    D = R.shape[0]
    Rc = R.detach().float().cpu()
    blocks = torch.stack([Rc[i:i + 4, i:i + 4] for i in range(0, D, 4)])
    off = Rc.clone()
    for i in range(0, D, 4):
        off[i:i + 4, i:i + 4] = 0
    if off.abs().max() != 0:
        raise ValueError("rotation is not block-diagonal with 4x4 blocks")
    return blocks.contiguous().to(device)


def rotate_last(x: torch.Tensor, R, transpose: bool = False, stream=None) -> torch.Tensor:
    """``x @ R`` over the last dim in bf16 (quant_kv.py:68-70); ``R`` is a
    [D, D] block-diagonal rotation or its [D/4, 4, 4] blocks."""
    blocks = R if R.dim() == 3 else so4_blocks(R, x.device)
    xc = x.contiguous()
    assert xc.dtype == torch.bfloat16
    D = xc.shape[-1]
    out = torch.empty_like(xc)
    check(lib.vb_so4_rotate(xc.data_ptr(), blocks.data_ptr(), xc.numel() // D, D,
                            int(transpose), out.data_ptr(), stream_handle(stream)),
          "vb_so4_rotate")
    return out


def _packed_words(dim: int, bits: int) -> int:
    return dim * bits // 32


class AsymmetricQuantizedKVCache:
    """K and V quantized with separate widths (quant_kv.py:80-207)."""

    step = 256

    def __init__(self, group_size: int = 64, k_bits: int = 4, v_bits: int = 3):
        self.keys = None
        self.values = None
        self.offset = 0
        self.group_size = group_size
        self.k_bits = k_bits
        self.v_bits = v_bits

    def _init_quant(self, dim, bits, B, H, steps, device):
        return (torch.zeros((B, H, steps, _packed_words(dim, bits)), dtype=torch.int32, device=device),
                torch.zeros((B, H, steps, dim // self.group_size), dtype=torch.bfloat16, device=device),
                torch.zeros((B, H, steps, dim // self.group_size), dtype=torch.bfloat16, device=device))

    def _grow(self, B, H, n, kD, vD, device):
        prev = self.offset
        if self.keys is None or prev + n > self.keys[0].shape[-2]:
            new_steps = (self.step + n - 1) // self.step * self.step
            if self.keys is not None:
                def expand(t):
                    t = t[..., :prev, :]
                    z = torch.zeros(t.shape[:-2] + (new_steps, t.shape[-1]), dtype=t.dtype,
                                    device=t.device)
                    return torch.cat([t, z], dim=-2).contiguous()
                self.keys = tuple(expand(t) for t in self.keys)
                self.values = tuple(expand(t) for t in self.values)
            else:
                self.keys = self._init_quant(kD, self.k_bits, B, H, new_steps, device)
                self.values = self._init_quant(vD, self.v_bits, B, H, new_steps, device)

    def _append(self, triple, src, bits, blocks, prev, stream):
        B, H, n, D = src.shape
        cap = triple[0].shape[-2]
        check(lib.vb_kv_quant_append(src.data_ptr(), ptr(blocks), B, H, n, D, self.group_size,
                                     bits, prev, cap, triple[0].data_ptr(), triple[1].data_ptr(),
                                     triple[2].data_ptr(), stream_handle(stream)),
              "vb_kv_quant_append")

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor, rk=None, rv=None,
                         stream=None):
        """Append ``keys``/``values`` bf16 ``[B, H, n, D]`` (quant_kv.py:105-137).

        ``rk``/``rv`` (optional [D/4,4,4] blocks) fuse the R_k / R_v rotation of
        kv_quant_patch.py:49-55 into the append. Returns the quantized
        ``(keys, values)`` triples sliced to ``[..., :offset, :]``."""
        keys = keys.contiguous()
        values = values.contiguous()
        B, H, n, kD = keys.shape
        vD = values.shape[-1]
        prev = self.offset
        self._grow(B, H, n, kD, vD, keys.device)
        self.offset += n
        self._append(self.keys, keys, self.k_bits, rk, prev, stream)
        self._append(self.values, values, self.v_bits, rv, prev, stream)
        return (tuple(t[..., :self.offset, :] for t in self.keys),
                tuple(t[..., :self.offset, :] for t in self.values))

    def fork(self):
        """Isolated append-only view for speculative attention (quant_kv.py:139-156)."""
        clone = type(self)(self.group_size, self.k_bits, self.v_bits)
        clone.offset = self.offset
        if self.keys is not None:
            clone.keys = tuple(t[..., :self.offset, :] for t in self.keys)
            clone.values = tuple(t[..., :self.offset, :] for t in self.values)
        return clone

    @property
    def state(self):
        if self.keys is None:
            return None, None
        if self.offset == self.keys[0].shape[-2]:
            return self.keys, self.values
        return (tuple(t[..., :self.offset, :] for t in self.keys),
                tuple(t[..., :self.offset, :] for t in self.values))

    @state.setter
    def state(self, value):
        self.keys, self.values = value

    @property
    def meta_state(self):
        return tuple(map(str, (self.offset, self.group_size, self.k_bits, self.v_bits)))

    @meta_state.setter
    def meta_state(self, value):
        self.offset, self.group_size, self.k_bits, self.v_bits = map(int, value)

    def is_trimmable(self):
        return True

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n

    def empty(self):
        return self.keys is None

    @property
    def nbytes(self):
        if self.keys is None:
            return 0
        return sum(t.numel() * t.element_size() for t in (*self.keys, *self.values))


def _full(t):
    """Base storage and capacity of a (possibly sliced) cache tensor."""
    return t, t.shape[-2]


def asym_quantized_sdpa(queries, q_keys, q_values, scale, mask, group_size, k_bits,
                        v_bits, rv=None, workspace=None, stream=None):
    """Quantized GQA attention over packed K/V (quant_kv.py:212-249).

    ``queries`` bf16 ``[B, Hq, L, D]``; ``q_keys``/``q_values`` cache triples
    (views sliced to the valid length are accepted); ``mask`` is None or
    ``"causal"``. ``rv`` (optional [D/4,4,4] blocks) fuses the inverse V
    rotation of kv_quant_patch.py:67-68. Output bf16 ``[B, Hq, L, D]``.
    """
    if mask is not None and mask != "causal":
        raise ValueError("asym_quantized_sdpa: only mask=None or 'causal' is supported")
    q = queries.contiguous()
    B, Hq, L, D = q.shape
    if L > 4:  # beyond the decode kernels: the tensor-core prefill kernel
        return tiled_asymmetric_attention(q, q_keys, q_values, scale=scale, mask=mask,
                                          group_size=group_size, k_bits=k_bits, v_bits=v_bits,
                                          rv=rv, stream=stream)
    kc, ks, kb = q_keys
    vc, vs, vb = q_values
    Hkv = kc.shape[-3]
    keys = kc.shape[-2]
    # Sliced views share their base storage; the kernel indexes rows with the
    # storage capacity (stride of the head dimension).
    cap = kc.stride(-3) // kc.stride(-2)
    for t in (kc, ks, kb, vc, vs, vb):
        assert t.stride(-1) == 1 and t.stride(-3) // t.stride(-2) == cap
    need = lib.vb_kv_attn_workspace_size(B, Hq, L, D, keys)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    check(lib.vb_kv_decode_attn(q.data_ptr(), kc.data_ptr(), ks.data_ptr(), kb.data_ptr(),
                                vc.data_ptr(), vs.data_ptr(), vb.data_ptr(), ptr(rv), B, Hq, Hkv,
                                L, D, keys, cap, group_size, k_bits, v_bits, float(scale),
                                int(mask == "causal"), out.data_ptr(), workspace.data_ptr(),
                                workspace.numel(), stream_handle(stream)),
          "vb_kv_decode_attn")
    return out


def tiled_asymmetric_attention(queries, q_keys, q_values, *, scale, mask, group_size, k_bits,
                               v_bits, rv=None, status=None, stream=None):
    """Prefill attention over packed K/V (``_tiled_asymmetric_attention``,
    mlx_streaming/core/attention/expert_major.py:32-95): bf16(q*scale) K^T
    rounded to bf16, causal (``mask="causal"``, query ``i`` of ``L`` sees keys
    ``<= S-L+i``) or no mask, precise softmax, P V -> bf16 ``[B, Hq, L, D]``.
    One tcgen05 kernel for all query rows (the reference's query tiles only
    bound its score memory). ``rv`` fuses the inverse V rotation."""
    if mask is not None and mask != "causal":
        raise ValueError("tiled_asymmetric_attention: only mask=None or 'causal' is supported")
    q = queries.contiguous()
    B, Hq, L, D = q.shape
    kc, ks, kb = q_keys
    vc, vs, vb = q_values
    Hkv = kc.shape[-3]
    keys = kc.shape[-2]
    cap = kc.stride(-3) // kc.stride(-2)
    for t in (kc, ks, kb, vc, vs, vb):
        assert t.stride(-1) == 1 and t.stride(-3) // t.stride(-2) == cap
    out = torch.empty_like(q)
    check(lib.vb_kv_prefill_attn(q.data_ptr(), kc.data_ptr(), ks.data_ptr(), kb.data_ptr(),
                                 vc.data_ptr(), vs.data_ptr(), vb.data_ptr(), ptr(rv), B, Hq, Hkv,
                                 L, D, keys, cap, group_size, k_bits, v_bits, float(scale),
                                 int(mask == "causal"), out.data_ptr(), ptr(status),
                                 stream_handle(stream)),
          "vb_kv_prefill_attn")
    return out
