"""GGUF row decoding on the GPU (``glm53_offload/gguf_quant.py:180-216``, ``qwen38_tpu/quant.py``).

``dequantize_rows(raw, qtype, row_width, dtype=None)`` keeps the reference's contract:
``raw`` is ``uint8[..., blocks_per_row, bytes_per_block]``; the result is
``[..., row_width]`` FP32 (or BF16 with the reference's RNE boundary), decoded by the
``qk_dequantize_rows`` kernel. Bit-exact with the reference decoders.
"""

import torch

from . import _lib

# (values per block, bytes per block) - gguf_quant.py:21-29 and quant.py:8
BLOCK_LAYOUTS = {
    "Q4_0": (32, 18),
    "Q4_1": (32, 20),
    "Q5_0": (32, 22),
    "Q5_1": (32, 24),
    "Q8_0": (32, 34),
    "Q4_K": (256, 144),
    "Q5_K": (256, 176),
    "Q6_K": (256, 210),
    "IQ4_NL": (32, 18),
    "F16": (1, 2),
    "BF16": (1, 2),
    "F32": (1, 4),
}

GGML_TYPE = {
    "F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8,
    "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ4_NL": 20, "BF16": 30,
}
_NAMES = {v: k for k, v in GGML_TYPE.items()}


def normalize_qtype(qtype):
    """Accept a name (``"Q6_K"``, ``"GGMLQuantizationType.Q6_K"``), an enum or a GGML number."""
    if hasattr(qtype, "name"):
        name = str(qtype.name).upper()
    elif isinstance(qtype, str):
        name = qtype.rsplit(".", 1)[-1].upper()
    else:
        try:
            name = _NAMES[int(qtype)]
        except (TypeError, ValueError, KeyError) as exc:
            raise ValueError(f"unsupported GGUF quantization type: {qtype!r}") from exc
    if name not in BLOCK_LAYOUTS:
        raise ValueError(f"unsupported GGUF quantization type: {qtype!r}")
    return name


def block_layout(qtype):
    """``(values_per_block, bytes_per_block)`` of a supported type."""
    return BLOCK_LAYOUTS[normalize_qtype(qtype)]


def dequantize_rows(raw, qtype, row_width, dtype=None):
    """Decode packed rows on the device into ``(..., row_width)`` values."""
    name = normalize_qtype(qtype)
    if not isinstance(row_width, int) or isinstance(row_width, bool):
        raise TypeError("row_width must be an integer")
    if not isinstance(raw, torch.Tensor) or raw.dtype != torch.uint8:
        got = raw.dtype if hasattr(raw, "dtype") else type(raw)
        raise TypeError(f"raw must have dtype uint8; got {got}")
    if raw.dim() < 2:
        raise ValueError("raw must have shape (..., blocks_per_row, bytes_per_block)")
    values, size = BLOCK_LAYOUTS[name]
    if raw.shape[-1] != size:
        raise ValueError(f"{name} blocks contain {size} bytes; got {raw.shape[-1]}")
    if row_width <= 0:
        raise ValueError("row_width must be a positive integer")
    nblocks = (row_width + values - 1) // values
    if raw.shape[-2] != nblocks:
        raise ValueError(f"row_width {row_width} requires {nblocks} {name} blocks; got {raw.shape[-2]}")
    if not raw.is_cuda:
        raise ValueError("raw must be a CUDA tensor")
    if dtype is None:
        dtype = torch.float32
    if dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("dtype must be float32 or bfloat16")
    raw = raw.contiguous()
    lead = tuple(raw.shape[:-2])
    rows = 1
    for n in lead:
        rows *= n
    out = torch.empty(lead + (row_width,), dtype=dtype, device=raw.device)
    with torch.cuda.device(raw.device):
        _lib.call(
            "qk_dequantize_rows",
            _lib.ptr(raw),
            GGML_TYPE[name],
            rows,
            row_width,
            _lib.QK_OUT_BF16 if dtype == torch.bfloat16 else _lib.QK_OUT_F32,
            _lib.ptr(out),
            _lib.stream_handle(raw.device),
        )
    return out
