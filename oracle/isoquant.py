"""CPU restatement of IsoQuant K4/V3 (test infrastructure).

SO(4) block rotation (quant_kv.py:24-70), asymmetric affine-quantized KV cache
append (quant_kv.py:80-137) and quantized GQA attention
(quant_kv.py:212-249, kv_quant_patch.py:49-68).
"""
from __future__ import annotations

import numpy as np

from . import mlx_ops as M


def _quat_left(q):
    """Left-multiplication matrix of a unit quaternion (quant_kv.py:24-32)."""
    w, x, y, z = q
    return np.array([[w, -x, -y, -z],
                     [x, w, -z, y],
                     [y, z, w, -x],
                     [z, -y, x, w]], dtype=np.float32)


def _quat_right_conj(q):
    """Right-multiplication-by-conjugate matrix (quant_kv.py:35-46)."""
    w, x, y, z = q
    return np.array([[w, x, y, z],
                     [-x, w, z, -y],
                     [-y, -z, w, x],
                     [-z, y, -x, w]], dtype=np.float32)


def build_block_so4(head_dim: int, seed: int = 0, blocks_of: int = 4) -> np.ndarray:
    """Block-diagonal SO(4) rotation (quant_kv.py:49-65), float32 numpy.

    Per 4x4 block: ``qL`` then ``qR`` drawn as ``standard_normal(4)`` float32
    from ``default_rng(seed)``, normalised, block ``L(qL) @ R(conj qR)``.
    """
    assert head_dim % blocks_of == 0
    rng = np.random.default_rng(seed)
    Mx = np.zeros((head_dim, head_dim), dtype=np.float32)
    for b in range(head_dim // blocks_of):
        qL = rng.standard_normal(4).astype(np.float32)
        qL /= np.linalg.norm(qL)
        qR = rng.standard_normal(4).astype(np.float32)
        qR /= np.linalg.norm(qR)
        blk = _quat_left(qL) @ _quat_right_conj(qR)
        i = b * blocks_of
        Mx[i:i + blocks_of, i:i + blocks_of] = blk
    return Mx


def so4_blocks(R: np.ndarray) -> np.ndarray:
    """Extract the ``[D/4, 4, 4]`` diagonal blocks of a block-diagonal ``R``."""
    D = R.shape[0]
    return np.stack([R[i:i + 4, i:i + 4] for i in range(0, D, 4)])


def rotate_last(x, R) -> np.ndarray:
    """``x @ R.astype(x.dtype)`` for bf16 ``x`` (quant_kv.py:68-70).

    R is rounded to bf16; each output is the float32 sum, in ascending input
    index, of the four non-zero products of its 4x4 block, rounded to bf16
    (the zero entries of the dense matmul add exact zeros).
    """
    x = np.asarray(x, np.float32)
    D = x.shape[-1]
    Rb = M.bf16(R)
    blocks = so4_blocks(Rb)                      # [D/4, 4(in), 4(out)]
    xb = x.reshape(*x.shape[:-1], D // 4, 4)
    acc = np.zeros_like(xb)
    for i in range(4):
        acc = (acc + (xb[..., i:i + 1] * blocks[:, i, :]).astype(np.float32)).astype(np.float32)
    return M.bf16(acc.reshape(x.shape))


def kv_quantize(x, group_size: int, bits: int):
    """``mx.quantize`` of one KV tensor ``[..., D]`` (quant_kv.py:128-129)."""
    return M.mlx_affine_quantize(M.bf16(x), group_size, bits)


def kv_dequantize(packed, dim, group_size, bits):
    """float32 dequantization of a cache triple."""
    w, s, b = packed
    return M.dequantize(w, s, b, dim, group_size, bits)


def asym_quantized_sdpa(q, kq, vq, scale, group_size, k_bits, v_bits,
                        causal: bool = False):
    """``asym_quantized_sdpa`` (quant_kv.py:212-249), MLX dtype chain.

    ``q [B, Hq, L, D]`` bf16; ``kq``/``vq`` cache triples over ``Hkv`` heads.
    - ``queries * scale`` -> bf16;
    - scores = quantized_matmul(q, K^T) -> bf16 (float32 accumulation);
    - causal: query ``i`` of ``L`` sees keys ``<= S-L+i`` (string mask,
      quant_kv.py:233-239); masked scores take bf16's lowest finite value;
    - ``softmax(precise=True)`` -> bf16 probabilities;
    - out = quantized_matmul(p, V) -> bf16. Output stays in rotated V space.
    """
    q = np.asarray(q, np.float32)
    Bn, Hq, L, D = q.shape
    Kd = kv_dequantize(kq, D, group_size, k_bits)   # [B, Hkv, S, D]
    Vd = kv_dequantize(vq, D, group_size, v_bits)
    Hkv, S = Kd.shape[1], Kd.shape[2]
    rep = Hq // Hkv
    qs = M.bf16(q * np.float32(scale)).reshape(Bn, Hkv, rep, L, D)
    # float64 products and sums (BLAS matmul), rounded once to float32
    scores = np.matmul(qs.reshape(Bn, Hkv, rep * L, D).astype(np.float64),
                       np.swapaxes(Kd.astype(np.float64), -1, -2))
    scores = scores.astype(np.float32).reshape(Bn, Hkv, rep, L, S)
    scores = M.bf16(scores)
    if causal:
        qi = np.arange(S - L, S)[:, None]
        ki = np.arange(S)[None, :]
        mask = qi >= ki
        scores = np.where(mask, scores, np.float32(-3.3895313892515355e38))
    p = M.bf16(M.softmax_precise(scores))
    out = np.matmul(p.reshape(Bn, Hkv, rep * L, S).astype(np.float64), Vd.astype(np.float64))
    out = out.astype(np.float32).reshape(Bn, Hkv, rep, L, D)
    return M.bf16(out).reshape(Bn, Hq, L, D)


def attention_layer_decode(q_rot, kq, vq, Rv, scale, group_size=64, k_bits=4,
                           v_bits=3, causal=False):
    """Quantized SDPA followed by the inverse V rotation (kv_quant_patch.py:58-68)."""
    out = asym_quantized_sdpa(q_rot, kq, vq, scale, group_size, k_bits, v_bits,
                              causal=causal)
    return rotate_last(out, np.asarray(Rv, np.float32).T)
