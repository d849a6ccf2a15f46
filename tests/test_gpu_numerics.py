"""The kernels' FP32 exp, sigmoid, divide and softmax against FP64, on the input sweep and
with the 5e-7 per-element relative budget of the reference's numerics gate
(qwen38_tpu/numerics_validation.py:12-74); the SwiGLU activation against the oracle."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BUDGET = 5e-7  # numerics_validation.py:40


def _sweep():
    """numerics_validation.py:13-26: the same generators, seeds and shapes."""
    rng = np.random.default_rng(506)
    x = np.linspace(-30, 30, 2049, dtype=np.float32)
    e = np.exp(-np.abs(x.astype(np.float64)))
    denominator = np.exp2(rng.uniform(-16, 16, 2049)).astype(np.float32)
    numerator = (rng.uniform(-128, 128, 2049) * denominator).astype(np.float32)
    scores = rng.uniform(-12, 12, (8, 32)).astype(np.float32)
    scores[:, :3] = -np.inf
    shifted = scores - np.max(scores, -1, keepdims=True)
    probabilities = np.exp(shifted.astype(np.float64))
    probabilities /= np.sum(probabilities, -1, keepdims=True)
    return {
        "exp": ((x,), np.exp(x.astype(np.float64))),
        "sigmoid": ((x,), np.where(x >= 0, 1, e) / (1 + e)),
        "divide": ((numerator, denominator), numerator.astype(np.float64) / denominator.astype(np.float64)),
        "softmax": ((scores,), probabilities),
    }


@pytest.mark.parametrize("name", ["exp", "sigmoid", "divide", "softmax"])
def test_fp32_function_within_the_reference_budget(cuda_device, name):
    import torch

    from qk_b200 import numerics

    inputs, expected = _sweep()[name]
    args = [torch.from_numpy(np.ascontiguousarray(v)).to(cuda_device) for v in inputs]
    actual = getattr(numerics, name)(*args).cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(actual))
    error = np.abs(actual - expected)
    bound = BUDGET * np.abs(expected) + 1e-30
    rel = float(np.max(error / np.maximum(np.abs(expected), 1e-30)))
    worst = np.unravel_index(np.argmax(error / bound), expected.shape)
    assert np.all(error <= bound), (name, rel, worst, actual[worst], expected[worst])


def test_swiglu_activation_matches_the_oracle(cuda_device):
    import torch

    from oracle.precision import bf16_round, silu_bf16
    from qk_b200 import numerics

    rng = np.random.default_rng(19)
    x = np.concatenate([np.linspace(-40, 40, 4097, dtype=np.float32),
                        rng.normal(0, 3, 8192).astype(np.float32),
                        np.array([0.0, -0.0, 1e-30, -1e-30, 88.0, -88.0], np.float32)])
    got = numerics.silu_bf16(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    expected = silu_bf16(bf16_round(x))
    # NumPy's FP32 exp and CUDA's expf may differ by an ulp; that can move the BF16 rounding
    # of the product only where it sits on a rounding boundary: one BF16 ulp, rarely.
    diff = np.abs(got.view(np.int32).astype(np.int64) - expected.view(np.int32).astype(np.int64)) >> 16
    assert diff.max() <= 1 and np.count_nonzero(diff) <= x.size // 1000, np.count_nonzero(diff)


def test_softmax_any_axis_and_masked_columns(cuda_device):
    """softmax over a non-last axis, rows longer than a warp, fully masked columns -> 0."""
    import torch

    from oracle.precision import softmax
    from qk_b200 import numerics

    rng = np.random.default_rng(7)
    s = rng.uniform(-20, 20, (300, 5)).astype(np.float32)
    s[:17] = -np.inf
    got = numerics.softmax(torch.from_numpy(s).to(cuda_device), axis=0).cpu().numpy()
    expected = softmax(s, axis=0)
    assert np.all(got[:17] == 0)
    np.testing.assert_allclose(got, expected, rtol=2e-6, atol=0)
