"""BF16 rounding boundaries and FP32 elementary functions (oracle, test infrastructure).

Restates ``kaggle/qwen38_tpu/precision.py:7-23`` (``rounded_bf16_float32``,
``compute_cast``) and ``kaggle/qwen38_tpu/numerics.py:13-51`` (exp, divide,
sigmoid, softmax) in NumPy.
"""

import numpy as np


def bf16_round(x):
    """Round FP32 to BF16 with ties to even, result kept in FP32.

    ``precision.py:7-17``: ``(bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000``,
    NaNs are quieted by setting bit 22.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    rounded = (bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))) & np.uint32(
        0xFFFF0000
    )
    nan = (bits & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    return np.where(nan, bits | np.uint32(0x00400000), rounded).view(np.float32)


def bf16_bits(x):
    """BF16 storage bits (uint16) of ``bf16_round(x)``."""
    return (bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(bits):
    """FP32 values of BF16 storage bits."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def compute_cast(x, dtype="bf16"):
    """``precision.py:20-23``: explicit RNE boundary when the target is BF16."""
    if dtype == "bf16":
        return bf16_round(x)
    return np.asarray(x, dtype=np.float32)


def f32(x):
    return np.asarray(x, dtype=np.float32)


def exp(x):
    """``numerics.py:13-14``: accurate FP32 exp."""
    return np.exp(f32(x)).astype(np.float32)


def divide(numerator, denominator):
    """``numerics.py:17-39``.

    With an IEEE reciprocal the one-step residual correction reproduces the
    correctly rounded quotient for the operands the runtime passes; the oracle
    therefore uses IEEE FP32 division, which is also what the reference's own
    NumPy oracles use (``validation.py:47``).
    """
    with np.errstate(divide="ignore", invalid="ignore"):
        return (f32(numerator) / f32(denominator)).astype(np.float32)


def sigmoid(x):
    """``numerics.py:42-45``: ``divide(x >= 0 ? 1 : e, 1 + e)`` with ``e = exp(-|x|)``."""
    x = f32(x)
    e = exp(-np.abs(x))
    one = np.float32(1.0)
    return divide(np.where(x >= 0, one, e).astype(np.float32), (one + e).astype(np.float32))


def softmax(x, axis=-1):
    """``numerics.py:48-51``: max-subtracted exp, then divide by the sum."""
    x = f32(x)
    e = exp(x - np.max(x, axis=axis, keepdims=True))
    return divide(e, np.sum(e, axis=axis, keepdims=True, dtype=np.float32))


def silu_bf16(x):
    """``math.py:19-20`` with a BF16 operand: ``compute_cast(x * sigmoid(x), bf16)``."""
    x = f32(x)
    return bf16_round((x * sigmoid(x)).astype(np.float32))
