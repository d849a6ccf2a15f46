"""FP32 elementary functions as the kernels compute them (``qwen38_tpu/numerics.py:13-51``).

``exp``, ``divide``, ``sigmoid`` and ``softmax`` keep the reference's names and argument
meaning and run the same device helpers the kernels use (``qk_numerics``), so the
reference's FP64 validation (``numerics_validation.py:12-74``) can hold them to its 5e-7
relative budget. Inputs are CUDA tensors; the result is FP32 of the same shape.
"""

import torch

from . import _lib


def _run(op, a, b=None, row_len=0):
    a = a.to(torch.float32).contiguous()
    out = torch.empty_like(a)
    if b is not None:
        b = b.to(torch.float32).expand_as(a).contiguous()
    with torch.cuda.device(a.device):
        _lib.call("qk_numerics", op, _lib.ptr(a), _lib.ptr(b), _lib.ptr(out), a.numel(), row_len,
                  _lib.stream_handle(a.device))
    return out


def exp(x):
    return _run(_lib.QK_NUM_EXP, x)


def divide(numerator, denominator):
    return _run(_lib.QK_NUM_DIVIDE, numerator, denominator)


def sigmoid(x):
    return _run(_lib.QK_NUM_SIGMOID, x)


def softmax(x, axis=-1):
    moved = x.movedim(axis, -1)
    out = _run(_lib.QK_NUM_SOFTMAX, moved, row_len=moved.shape[-1])
    return out.movedim(-1, axis)


def silu_bf16(x):
    """The SwiGLU epilogue's activation ``bf16(g * sigmoid(g))`` of ``g = bf16(x)``
    (``math.py:19-20``)."""
    return _run(_lib.QK_NUM_SILU_BF16, x)


__all__ = ["exp", "divide", "sigmoid", "softmax", "silu_bf16"]
