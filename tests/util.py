"""Small helpers shared by the tests (host <-> device conversions, error metrics)."""

import numpy as np


def bf16_tensor(values, device):
    """FP32 numpy values -> BF16 torch tensor (RNE, the oracle's rounding)."""
    import torch

    from oracle.precision import bf16_bits

    bits = bf16_bits(np.asarray(values, np.float32)).view(np.int16)
    return torch.from_numpy(bits.copy()).to(device).view(torch.bfloat16)


def to_f32(tensor):
    """Any torch tensor -> FP32 numpy array (BF16 values are exact in FP32)."""
    import torch

    return tensor.detach().to(torch.float32).cpu().numpy()


def rel_err(actual, expected):
    """max |a - e| / max |e| and relative L2 error."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    scale = max(np.max(np.abs(e)), 1e-30)
    return float(np.max(np.abs(a - e)) / scale), float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))


def random_blocks(rng, rows, width, qtype):
    """Random GGUF blocks ``uint8[rows, blocks, bytes]`` of a Q5_K or Q5_1 row of ``width``
    values with finite FP16 scales (no encoder of these types is needed: any code bytes are
    legal). Q5_K: d in [1e-4, 2e-4), dmin in [0, 1e-4); Q5_1: d in [1e-3, 2e-3), m in
    [-0.03, 0)."""
    values, size = {"Q5_K": (256, 176), "Q5_1": (32, 24)}[qtype]
    blocks = (width + values - 1) // values
    raw = rng.integers(0, 256, (rows, blocks, size), dtype=np.uint8)

    def f16(lo, hi):
        return rng.uniform(lo, hi, (rows, blocks)).astype("<f2").view(np.uint8).reshape(rows, blocks, 2)

    if qtype == "Q5_K":
        raw[..., 0:2] = f16(1e-4, 2e-4)
        raw[..., 2:4] = f16(0, 1e-4)
    else:
        raw[..., 0:2] = f16(1e-3, 2e-3)
        raw[..., 2:4] = f16(-0.03, 0)
    return raw
