"""numpy restatement of the MLX ops on the Vates hot path (test infrastructure).

Every function documents the reference call site it stands in for. Values of
dtype bfloat16 are carried as float32 arrays whose values are exactly
representable in bf16 (rounded with :func:`bf16`), or as raw ``uint16`` bit
patterns where the reference stores bits (``native_moe.py:57-72`` keeps scales
and biases as ``uint16`` holding bf16 bits).
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------


def bf16_bits(a) -> np.ndarray:
    """float32 -> bf16 bit pattern, round-to-nearest-even (NaN kept quiet)."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def bf16_from_bits(b) -> np.ndarray:
    """bf16 bit pattern (uint16) -> float32 value."""
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def bf16(a) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (returned as float32)."""
    return bf16_from_bits(bf16_bits(a))


def bf16_ulp(a) -> np.ndarray:
    """Size of one bf16 unit in the last place at the magnitude of ``a``."""
    a = np.abs(np.asarray(a, dtype=np.float32))
    exp = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return (2.0 ** (exp - 7)).astype(np.float32)


# ----------------------------------------------------------------------------
# MLX affine quantization format (bits in {2,3,4,5,6,8}, group in {32,64,128})
# ----------------------------------------------------------------------------


_CHUNK_ROWS = 8192  # rows per pass of the bit-matrix pack/unpack (bounds host memory)


def packed_words(dim: int, bits: int) -> int:
    """uint32 words per packed row: ``dim*bits//32`` (quant_kv.py:75-77)."""
    return dim * bits // 32


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack integer codes ``[..., dim]`` into a continuous LSB-first bitstream.

    Layout read back by the reference kernels: field ``c`` starts at bit
    ``c*bits`` of the row's little-endian uint32 word stream and straddles into
    the next word when ``shift + bits > 32`` (fused_moe.cpp:131-145,
    custom_kernel.py:170-185). This is the byte stream MLX's quantize writes
    (power-of-two widths as uint32 words, 3/5/6-bit widths as 3-byte packs).
    """
    codes = np.asarray(codes)
    *lead, dim = codes.shape
    assert (dim * bits) % 32 == 0
    nbits = dim * bits
    flat = codes.reshape(-1, dim)
    if flat.shape[0] > _CHUNK_ROWS:
        parts = [pack_codes(flat[i:i + _CHUNK_ROWS], bits)
                 for i in range(0, flat.shape[0], _CHUNK_ROWS)]
        return np.concatenate(parts).reshape(*lead, nbits // 32)
    flat = flat.astype(np.uint64)
    # Expand to a bit matrix [rows, dim*bits], LSB first per field.
    shifts = np.arange(bits, dtype=np.uint64)
    bitmat = ((flat[:, :, None] >> shifts[None, None, :]) & 1).astype(np.uint8)
    bitmat = bitmat.reshape(flat.shape[0], nbits)
    bytes_ = np.packbits(bitmat.reshape(flat.shape[0], nbits // 8, 8),
                         axis=-1, bitorder="little").reshape(flat.shape[0], nbits // 8)
    words = np.ascontiguousarray(bytes_).view("<u4")
    return words.reshape(*lead, nbits // 32).astype(np.uint32)


def unpack_codes(words: np.ndarray, dim: int, bits: int) -> np.ndarray:
    """Inverse of :func:`pack_codes`: ``[..., dim*bits/32]`` words -> codes."""
    words = np.ascontiguousarray(np.asarray(words, dtype="<u4"))
    *lead, nw = words.shape
    assert nw * 32 == dim * bits
    if bits in (2, 4, 8):
        per = 32 // bits
        shifts = (np.arange(per, dtype=np.uint32) * bits)
        codes = (words[..., None] >> shifts) & np.uint32((1 << bits) - 1)
        return codes.reshape(*lead, dim).astype(np.uint8)
    flat = words.reshape(-1, nw)
    if flat.shape[0] > _CHUNK_ROWS:
        parts = [unpack_codes(flat[i:i + _CHUNK_ROWS], dim, bits)
                 for i in range(0, flat.shape[0], _CHUNK_ROWS)]
        return np.concatenate(parts).reshape(*lead, dim)
    bytes_ = flat.view(np.uint8).reshape(flat.shape[0], nw * 4)
    bitmat = np.unpackbits(bytes_, axis=-1, bitorder="little")
    bitmat = bitmat.reshape(flat.shape[0], dim, bits).astype(np.uint32)
    codes = (bitmat << np.arange(bits, dtype=np.uint32)[None, None, :]).sum(-1)
    return codes.reshape(*lead, dim).astype(np.uint8)


def mlx_affine_quantize(w: np.ndarray, group_size: int, bits: int):
    """Restatement of MLX 0.31 ``mx.quantize(w, group_size, bits)`` (affine).

    Called by the reference at quant_kv.py:128-129 (K 4-bit, V 3-bit, g=64).
    Per group of ``group_size`` values (float32 math on the bf16 inputs):

    - ``scale = max((w_max - w_min) / n_bins, 1e-7)`` with ``n_bins = 2^bits-1``;
    - the edge with the larger magnitude anchors the grid: if ``|w_min| >
      |w_max|`` the scale stays positive and ``edge = w_min``, otherwise the
      scale is negated and ``edge = w_max``;
    - ``q0 = rint(edge / scale)``; when ``q0 != 0`` the scale becomes
      ``edge / q0`` and ``bias = edge`` (so that code ``-q0`` dequantizes to
      exactly zero); when ``q0 == 0`` the bias is 0;
    - codes ``q = clip(rint((w - bias) / scale), 0, n_bins)`` computed with the
      float32 scale/bias, then scale and bias are rounded to bf16 for storage.

    Returns ``(packed uint32 [..., D*bits/32], scales bf16-bits uint16
    [..., D/g], biases bf16-bits uint16 [..., D/g])``.
    """
    w = np.asarray(w, dtype=np.float32)
    *lead, dim = w.shape
    assert dim % group_size == 0
    g = w.reshape(-1, dim // group_size, group_size)
    n_bins = np.float32((1 << bits) - 1)
    w_max = g.max(-1)
    w_min = g.min(-1)
    mask = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / n_bins, np.float32(1e-7)).astype(np.float32)
    scale = np.where(mask, scale, -scale).astype(np.float32)
    edge = np.where(mask, w_min, w_max).astype(np.float32)
    q0 = np.rint(edge / scale).astype(np.float32)
    nz = q0 != 0
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = np.where(nz, edge / np.where(nz, q0, 1), scale).astype(np.float32)
    bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
    q = np.rint((g - bias[..., None]) / scale[..., None]).astype(np.float32)
    q = np.clip(q, 0, n_bins).astype(np.uint32)
    packed = pack_codes(q.reshape(-1, dim), bits)
    return (packed.reshape(*lead, dim * bits // 32),
            bf16_bits(scale).reshape(*lead, dim // group_size),
            bf16_bits(bias).reshape(*lead, dim // group_size))


def dequantize(words, scales_bits, biases_bits, dim: int, group_size: int,
               bits: int) -> np.ndarray:
    """``w = q*scale + bias`` in float32 (fused_moe.cpp:131-145 ``qvalue``).

    ``q*scale`` is exact in float32 for bits <= 8 and a bf16 scale, so this is
    the single-rounding value ``fma(q, scale, bias)``.
    """
    q = unpack_codes(words, dim, bits).astype(np.float32)
    s = np.repeat(bf16_from_bits(scales_bits), group_size, axis=-1)
    b = np.repeat(bf16_from_bits(biases_bits), group_size, axis=-1)
    return (q * s + b).astype(np.float32)


def dequantize_bf16(words, scales_bits, biases_bits, dim, group_size, bits):
    """Dequantized weights rounded once to bf16 (the tensor-core operand).

    The prefill path (MLX ``gather_qmm`` matrix kernel, compute.py:170 for
    S > 4) dequantizes weight tiles to the activation dtype before the MMA.
    """
    return bf16(dequantize(words, scales_bits, biases_bits, dim, group_size, bits))


# ----------------------------------------------------------------------------
# Dense ops with MLX's dtype chain (float32 inside an op, bf16 at op outputs)
# ----------------------------------------------------------------------------


def matvec_f32(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """``x @ w.T`` accumulated in float64 and rounded once to float32.

    Stands in for a float32-accumulating GPU reduction: the exact sum rounded
    once is the value every summation order approximates.
    """
    return (np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32)


def sigmoid_f32(x: np.ndarray) -> np.ndarray:
    """MLX's sigmoid: ``y = 1/(1+exp(-|x|))``, ``x<0 -> 1-y`` (float32)."""
    x = np.asarray(x, np.float32)
    y = (np.float32(1) / (np.float32(1) + np.exp(-np.abs(x)))).astype(np.float32)
    return np.where(x < 0, np.float32(1) - y, y).astype(np.float32)


def swiglu_bf16(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """mlx-lm ``SwiGLU``: ``silu(gate) * up`` = ``(gate*sigmoid(gate))*up``.

    Compiled elementwise graph (mlx-lm switch_layers / nn.silu) keeps the
    bf16 output type of every node: sigmoid, product and product with ``up``
    are each rounded to bf16 (compute.py:192; mlx-lm SwiGLU).
    """
    sig = bf16(sigmoid_f32(gate))
    a = bf16(gate * sig)
    return bf16(a * up)


def swiglu_f32(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """Native-extension SwiGLU in float32: ``g*(1/(1+exp(-g)))*u``.

    fused_moe.cpp:196-197 and custom_kernel.py:298-303.
    """
    g = np.asarray(gate, np.float32)
    sig = (np.float32(1) / (np.float32(1) + np.exp(-g))).astype(np.float32)
    return (g * sig * np.asarray(up, np.float32)).astype(np.float32)


def softmax_precise(logits: np.ndarray) -> np.ndarray:
    """``mx.softmax(x, precise=True)``: float32 max/exp/sum, times 1/sum."""
    x = np.asarray(logits, np.float32)
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m).astype(np.float32)
    s = e.astype(np.float64).sum(-1, keepdims=True).astype(np.float32)
    return (e * (np.float32(1) / s)).astype(np.float32)


def topk_desc(values: np.ndarray, k: int) -> np.ndarray:
    """Top-``k`` indices per row: larger value first, lower index on ties.

    Stands in for ``mx.argpartition(gates, kth=-k)[..., -k:]`` (block.py:323),
    whose order is unspecified; callers compare expert *sets*, and ties at the
    k-th value are resolved by lower expert id here and in the kernels.
    """
    v = np.asarray(values, np.float32)
    idx = np.arange(v.shape[-1])
    # lexsort: last key primary -> sort by (-v, idx)
    order = np.lexsort((np.broadcast_to(idx, v.shape), -v), axis=-1)
    return order[..., :k].astype(np.int32)
