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
