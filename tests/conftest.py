import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def bf16_steps(a, b):
    """Distance between bf16 values counted in representable bf16 steps."""
    from oracle import mlx_ops as M

    def ordered(x):
        u = M.bf16_bits(np.asarray(x, np.float32)).astype(np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u)

    return np.abs(ordered(a) - ordered(b))


def bf16_close(got, ref, atol=2e-2, mean_rel=5e-3, max_ulps=2, frac_beyond=5e-3, scale=None,
               what=""):
    """The parity bar for bf16 outputs (max-abs 2e-2, mean-rel 5e-3 in
    bf16).

    The MLX dtype chain rounds to bf16 after every op, so a float32
    summation-order difference can flip an intermediate rounding by one bf16
    ulp *of that intermediate*; when the last op adds two large terms (routed
    sum + gated shared expert, or the residual) a flip is worth one ulp of the
    larger addend. ``scale`` gives that per-element magnitude (default: the
    reference itself). The bar: every element within
    max(atol, max_ulps * ulp(scale)); at most ``frac_beyond`` of the elements
    beyond max(atol, ulp(scale)); and mean |err| / mean |ref| <= mean_rel."""
    from oracle import mlx_ops as M
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    mag = np.abs(ref) if scale is None else np.maximum(np.abs(ref), np.abs(scale))
    ulp = M.bf16_ulp(mag)
    err = np.abs(got - ref)
    hard = err > np.maximum(np.float32(atol), max_ulps * ulp)
    soft = err > np.maximum(np.float32(atol), ulp)
    rel = float(err.mean() / max(float(np.abs(ref).mean()), 1e-30))
    assert not hard.any(), (f"{what}: {int(hard.sum())} elements beyond {max_ulps} ulp; worst "
                            f"err={float(err.max()):.4g} at ref={float(ref.flat[int(err.argmax())]):.4g}")
    assert soft.mean() <= frac_beyond, (f"{what}: {int(soft.sum())} of {soft.size} elements "
                                        f"beyond 1 ulp")
    assert rel <= mean_rel, f"{what}: mean-rel {rel:.3g} > {mean_rel}"
    return float(err.max()), rel


def block_scale(ref: dict, residual=None):
    """Per-element magnitude of the last additions of the decode block."""
    s = np.maximum(np.abs(ref["routed"]), np.abs(ref["shared"]))
    s = np.maximum(s, np.abs(ref["out"]))
    if residual is not None:
        s = np.maximum(s, np.abs(np.asarray(residual, np.float32)))
    return s


def f32_close(got, ref, atol=2e-2, mean_rel=5e-3, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    err = np.abs(got - ref)
    rel = float(err.mean() / max(float(np.abs(ref).mean()), 1e-30))
    assert float(err.max()) <= atol, f"{what}: max-abs {float(err.max()):.4g} > {atol}"
    assert rel <= mean_rel, f"{what}: mean-rel {rel:.3g} > {mean_rel}"
    return float(err.max()), rel
