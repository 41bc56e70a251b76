"""numpy replica of the benchmark's seeded synthetic model (test infrastructure).

Reproduces, on the CPU and without the CUDA library, the weights that
``vates_b200.synth`` generates: dense tensors from numpy ``PCG64`` streams
and expert weights from the counter hash of ``vb_synth_fill_u32`` /
``vb_synth_fill_scales`` (splitmix64 finaliser of ``seed ^ index``). Used by
the CPU baseline / reference arm of ``bench.py`` and by the tests that check
the device generator.
"""
from __future__ import annotations

import numpy as np

from . import mlx_ops as M

H, I, E, K = 2048, 512, 512, 10
SHARED_ID = 100_000
_M64 = (1 << 64) - 1


def _mix_int(seed: int, salt: int) -> int:
    z = (seed * 0x9E3779B97F4A7C15 + salt * 0xBF58476D1CE4E5B9 + 0x94D049BB133111EB) & _M64
    z ^= z >> 31
    return z


def expert_seed(base: int, layer: int, expert: int) -> int:
    return _mix_int(_mix_int(base, layer + 1), expert + 7)


def mix64(z):
    z = np.asarray(z, np.uint64)
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def fill_u32(n: int, seed: int) -> np.ndarray:
    key = mix64(np.uint64(seed))
    idx = np.arange(n, dtype=np.uint64)
    return (mix64(key ^ idx) >> np.uint64(32)).astype(np.uint32)


def fill_scales(n: int, seed: int, lo=0.002, hi=0.02, bias_mul=-8.0):
    key = mix64(np.uint64(seed) ^ np.uint64(0x5CA1E5))
    idx = np.arange(n, dtype=np.uint64)
    r = (mix64(key ^ idx) >> np.uint64(40)).astype(np.float32)
    u = (r * np.float32(1.0 / 16777216.0)).astype(np.float32)
    span = np.float32(np.float32(hi) - np.float32(lo))
    val = (span.astype(np.float64) * u.astype(np.float64) + np.float64(np.float32(lo))).astype(np.float32)
    s = M.bf16_bits(val)
    b = M.bf16_bits(M.bf16_from_bits(s) * np.float32(bias_mul))
    return s, b


def expert_arrays(seed: int, hidden=H, inter=I, bits=4, group=64, bias_mul=-8.0) -> dict:
    """One expert in the oracle's nine-array format (slot axis of length 1)."""
    out = {}
    for j, (name, (o, i)) in enumerate((("gate", (inter, hidden)), ("up", (inter, hidden)),
                                        ("down", (hidden, inter)))):
        w = fill_u32(o * i * bits // 32, _mix_int(seed, 3 * j)).reshape(1, o, i * bits // 32)
        s, b = fill_scales(o * (i // group), _mix_int(seed, 3 * j + 1), bias_mul=bias_mul)
        out[name + "_w"] = w
        out[name + "_s"] = s.reshape(1, o, i // group)
        out[name + "_b"] = b.reshape(1, o, i // group)
    return out


def normal_bf16(rng, shape, std):
    return M.bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def dense_layer(seed: int, layer: int, hidden=H, num_experts=E):
    """Router weight and shared-expert gate of a synthetic layer (same PCG64
    streams as ``vates_b200.synth.make_layer``)."""
    rng = np.random.Generator(np.random.PCG64([seed, layer]))
    wr = normal_bf16(rng, (num_experts, hidden), 0.02)
    wsg = normal_bf16(rng, (hidden,), 0.02)
    return wr, wsg


def input_tokens(seed: int, T: int, hidden=H):
    rng = np.random.Generator(np.random.PCG64([seed, 999_999]))
    return normal_bf16(rng, (T, hidden), 1.0)


class LazyLayer(dict):
    """Oracle layer dict whose expert pool materialises experts on demand
    (identity slot table over all experts)."""

    def __init__(self, seed: int, layer: int, hidden=H, inter=I, num_experts=E, bias_mul=-8.0):
        wr, wsg = dense_layer(seed, layer, hidden, num_experts)
        super().__init__(wr=wr, wsg=wsg, table=np.arange(num_experts, dtype=np.int32),
                         shared=expert_arrays(expert_seed(seed, layer, SHARED_ID), hidden, inter,
                                              bias_mul=bias_mul),
                         hidden=hidden, inter=inter, group=64, bits=4)
        self["pool"] = _LazyPool(seed, layer, hidden, inter, bias_mul)


class _LazyPool(dict):
    def __init__(self, seed, layer, hidden, inter, bias_mul=-8.0):
        super().__init__()
        self._args = (seed, layer, hidden, inter, bias_mul)
        self._cache = {}

    def _expert(self, e):
        if e not in self._cache:
            seed, layer, hidden, inter, bias_mul = self._args
            self._cache[e] = expert_arrays(expert_seed(seed, layer, e), hidden, inter,
                                           bias_mul=bias_mul)
        return self._cache[e]

    def __getitem__(self, key):
        return _LazyArray(self, key)

    def prefetch(self, experts):
        for e in experts:
            self._expert(int(e))


class _LazyArray:
    def __init__(self, pool, key):
        self.pool, self.key = pool, key

    def __getitem__(self, slot):
        return self.pool._expert(int(slot))[self.key][0]
