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


def bf16_close(got, ref, atol=2e-2, mean_rel=5e-3, max_ulps=2, frac_beyond=5e-3, what=""):
    """The parity bar for bf16 outputs (north star: max-abs 2e-2, mean-rel
    5e-3 in bf16).

    A bf16 ulp exceeds 2e-2 once |y| >= 4, and the MLX dtype chain rounds to
    bf16 at every op, so a float32 summation-order difference can flip an
    intermediate rounding. The bar is therefore: every element within
    max(atol, max_ulps bf16 ulps of the reference); at most ``frac_beyond`` of
    the elements beyond max(atol, 1 ulp); and mean |err| / mean |ref| <=
    mean_rel."""
    from oracle import mlx_ops as M
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    err = np.abs(got - ref)
    ulp = M.bf16_ulp(ref)
    hard = err > np.maximum(np.float32(atol), max_ulps * ulp)
    soft = err > np.maximum(np.float32(atol), ulp)
    rel = float(err.mean() / max(float(np.abs(ref).mean()), 1e-30))
    assert not hard.any(), (f"{what}: {int(hard.sum())} elements beyond {max_ulps} ulp; worst "
                            f"err={float(err.max()):.4g} at ref={float(ref.flat[int(err.argmax())]):.4g}")
    assert soft.mean() <= frac_beyond, f"{what}: {int(soft.sum())} elements beyond 1 ulp"
    assert rel <= mean_rel, f"{what}: mean-rel {rel:.3g} > {mean_rel}"
    return float(err.max()), rel


def f32_close(got, ref, atol=2e-2, mean_rel=5e-3, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    err = np.abs(got - ref)
    rel = float(err.mean() / max(float(np.abs(ref).mean()), 1e-30))
    assert float(err.max()) <= atol, f"{what}: max-abs {float(err.max()):.4g} > {atol}"
    assert rel <= mean_rel, f"{what}: mean-rel {rel:.3g} > {mean_rel}"
    return float(err.max()), rel
