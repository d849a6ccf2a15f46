"""Expert placement: byte-exact EP/TP splits and device-resident tiled expert tensors.

``split_expert_bytes`` keeps the reference's contract (``qwen38_tpu/parallel.py:40-61``):
raw GGUF expert bytes ``[E, bytes]`` -> ``[tensor_rank, local_expert, bytes]`` without
splitting a quantisation block. ``put_expert_bytes`` replaces ``parallel.py:64-87``: it
takes this rank's contiguous expert range (EP: experts are partitioned, tokens are
replicated) and repacks each expert into the B200 tile layout on the device.
"""

import numpy as np
import torch

from . import _lib
from .packed import TILED_TYPES as EXPERT_TYPES  # gate/up: the k-quants; down: Q6_K, Q4_K, Q8_0, Q5_1
from .packed import tiled_bytes
from .quant import BLOCK_LAYOUTS, GGML_TYPE, normalize_qtype


def split_expert_bytes(raw, kind, qtype, hidden, intermediate, tensor_parallel):
    """Every tensor rank's slice of every expert, ``uint8[tensor_parallel, E, bytes / tp]``.

    The byte contract of ``qwen38_tpu/parallel.py:40-61`` (pinned by a golden of that
    function): entry ``[t]`` is ``tensor_slice(raw, ..., t)``, so gate/up keep whole rows
    and down keeps whole quantisation blocks. The argument checks (and their messages)
    are ``tensor_slice``'s."""
    raw = np.asarray(raw)
    slices = [tensor_slice(raw, kind, qtype, hidden, intermediate, tensor_parallel, t)
              for t in range(tensor_parallel)]
    return np.stack(slices).astype(np.uint8, copy=False)


def expert_shape(kind, hidden, intermediate):
    """(rows, row_width) of one expert's projection matrix."""
    return (hidden, intermediate) if kind == "down" else (intermediate, hidden)


def local_range(num_experts, rank, world):
    if num_experts % world:
        raise ValueError("Expert count must divide expert parallel size")
    per = num_experts // world
    return rank * per, per


def tensor_slice(raw, kind, qtype, hidden, intermediate, tensor_parallel, tensor_rank):
    """Tensor rank ``tensor_rank``'s bytes of every expert in ``raw`` ``[E, bytes]`` (NumPy or
    torch): the slice ``split_expert_bytes(...)[tensor_rank]`` - gate/up rows
    ``[r * I/tp, (r + 1) * I/tp)``, down columns of the same range in whole blocks."""
    if kind not in {"gate", "up", "down"}:
        raise ValueError("Unknown expert projection")
    block, size = BLOCK_LAYOUTS[normalize_qtype(qtype)]
    if intermediate % tensor_parallel:
        raise ValueError("Intermediate channels must divide tensor parallel size")
    if not 0 <= tensor_rank < tensor_parallel:
        raise ValueError("tensor rank must lie in [0, tensor_parallel)")
    local = intermediate // tensor_parallel
    count = len(raw)
    if kind == "down":
        if local % block:
            raise ValueError("Tensor slices must contain whole down quantization blocks")
        part = raw.reshape(count, hidden, tensor_parallel, local // block, size)[:, :, tensor_rank]
    else:
        if hidden % block:
            raise ValueError("Hidden channels must contain whole quantization blocks")
        part = raw.reshape(count, tensor_parallel, local, hidden // block, size)[:, tensor_rank]
    return part.reshape(count, -1)


def put_expert_bytes(raw, kind, qtype, hidden, intermediate, *, rank=0, world=1, device=None,
                     tensor_rank=0, tensor_parallel=1):
    """This rank's experts as a device tensor ``uint8[E_local, tiled_bytes_per_expert]``.

    With ``tensor_parallel > 1`` every expert of the range is cut to tensor rank
    ``tensor_rank``'s slice of the intermediate channels (``tensor_slice``), tiled as a
    matrix of ``intermediate / tensor_parallel`` channels."""
    name = normalize_qtype(qtype)
    if name not in EXPERT_TYPES:
        raise ValueError(f"expert kernels take {EXPERT_TYPES}; got {name}")
    values, size = BLOCK_LAYOUTS[name]
    first, count = local_range(len(raw), rank, world)
    device = torch.device(device or "cuda")
    part = raw[first : first + count]
    if tensor_parallel > 1:
        full = expert_shape(kind, hidden, intermediate)
        per_full = full[0] * ((full[1] + values - 1) // values) * size
        if part.reshape(count, -1).shape[1] != per_full:
            raise ValueError(f"{kind} expert must hold {per_full} bytes; got {part.reshape(count, -1).shape[1]}")
        part = tensor_slice(part.reshape(count, -1), kind, name, hidden, intermediate, tensor_parallel, tensor_rank)
        if isinstance(part, np.ndarray):
            part = np.ascontiguousarray(part)
        else:
            part = part.contiguous()
        intermediate //= tensor_parallel
    rows, width = expert_shape(kind, hidden, intermediate)
    per_raw = rows * ((width + values - 1) // values) * size
    if isinstance(part, np.ndarray):
        if part.dtype != np.uint8:
            raise TypeError("GGUF expert bytes must have dtype uint8")
        src = torch.from_numpy(np.ascontiguousarray(part.reshape(count, -1))).to(device)
    else:
        src = part.reshape(count, -1).to(device).contiguous()
    if src.shape[1] != per_raw:
        raise ValueError(f"{kind} expert must hold {per_raw} bytes; got {src.shape[1]}")
    per_tiled = tiled_bytes(name, rows, width)
    out = torch.empty((count, per_tiled), dtype=torch.uint8, device=device)
    bad = torch.zeros(1, dtype=torch.int32, device=device)
    stream = _lib.stream_handle(device)
    with torch.cuda.device(device):
        if rows % 64 == 0:  # experts never share a 64-row tile: one launch for all
            _lib.call("qk_repack_rows", _lib.ptr(src), GGML_TYPE[name], count * rows, width,
                      _lib.ptr(out), _lib.ptr(bad), stream)
        else:
            for e in range(count):
                _lib.call("qk_repack_rows", _lib.ptr(src[e]), GGML_TYPE[name], rows, width,
                          _lib.ptr(out[e]), _lib.ptr(bad), stream)
    if int(bad.item()):
        raise ValueError(f"{name} block scales must be finite")
    return out
