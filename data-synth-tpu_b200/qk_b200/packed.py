"""Lossless tiled repack and the packed-weight projection.

Mirrors ``kaggle/packed_q6``: ``pack_q6``/``unpack_q6`` (``layout.py:49-108``) and
``q6_matmul`` (``kernel.py:98-148``), with this build's tile layout (64 rows x 256
values per tile, see ``csrc/rowtile.cuh``) instead of the TPU SoA tiles. ``pack_rows``
and ``quant_matmul`` are the type-generic forms (Q6_K, Q4_K, Q5_K, Q8_0, Q5_1).
"""

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .quant import BLOCK_LAYOUTS, GGML_TYPE, normalize_qtype

TILED_TYPES = ("Q6_K", "Q4_K", "Q5_K", "Q8_0", "Q5_1")


@dataclass(frozen=True)
class PackedWeights:
    data: torch.Tensor  # uint8 [tiled_bytes] on the device
    qtype: str
    input_features: int
    output_features: int

    @property
    def input_blocks(self):
        """GGUF blocks per row (256 values for the k-quants, 32 for Q8_0 and Q5_1)."""
        values = BLOCK_LAYOUTS[self.qtype][0]
        return (self.input_features + values - 1) // values

    def storage(self):
        original = self.output_features * self.input_blocks * BLOCK_LAYOUTS[self.qtype][1]
        size = self.data.numel()
        return dict(
            original_bytes=original,
            packed_bytes=size,
            padding_bytes=size - original,
            padding_ratio=size / original - 1,
            layout="qk_b200_tile16x256_v1",
        )


def tiled_bytes(qtype, rows, row_width):
    n = _lib.load().qk_tiled_bytes(GGML_TYPE[normalize_qtype(qtype)], rows, row_width)
    if n < 0:
        raise ValueError(f"no tiled layout for {qtype}")
    return int(n)


def _device_raw(raw, device):
    if isinstance(raw, np.ndarray):
        if raw.dtype != np.uint8:
            raise TypeError(f"GGUF input must have dtype uint8; got {raw.dtype}")
        return torch.from_numpy(np.ascontiguousarray(raw)).to(device)
    if not isinstance(raw, torch.Tensor) or raw.dtype != torch.uint8:
        raise TypeError("GGUF input must have dtype uint8")
    return raw.to(device).contiguous()


def pack_rows(raw, input_features, qtype="Q6_K", device=None):
    """Repack ``uint8[N, ceil(K/block_values), bpb]`` GGUF rows into device tiles (no arithmetic)."""
    name = normalize_qtype(qtype)
    if name not in TILED_TYPES:
        raise ValueError(f"tiled layout supports {TILED_TYPES}; got {name}")
    if type(input_features) is not int or input_features < 1:
        raise ValueError("input_features must be a positive integer")
    device = torch.device(device or "cuda")
    if isinstance(raw, np.ndarray) and raw.dtype != np.uint8:
        raise TypeError(f"GGUF {name} input must have dtype uint8")
    if isinstance(raw, torch.Tensor) and raw.dtype != torch.uint8:
        raise TypeError(f"GGUF {name} input must have dtype uint8")
    values, size = BLOCK_LAYOUTS[name]
    blocks = (input_features + values - 1) // values
    if raw.ndim != 3 or raw.shape[0] < 1 or tuple(raw.shape[1:]) != (blocks, size):
        raise ValueError(f"Expected [output_features, ceil(input_features / {values}), bytes_per_block]")
    src = _device_raw(raw, device)
    rows = int(src.shape[0])
    out = torch.empty(tiled_bytes(name, rows, input_features), dtype=torch.uint8, device=device)
    bad = torch.zeros(1, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        _lib.call("qk_repack_rows", _lib.ptr(src), GGML_TYPE[name], rows, input_features,
                  _lib.ptr(out), _lib.ptr(bad), _lib.stream_handle(device))
    if int(bad.item()):
        raise ValueError(f"{name} block scales must be finite")
    return PackedWeights(out, name, input_features, rows)


def pack_q6(raw, input_features, device=None):
    """``packed_q6.layout.pack_q6`` with the B200 tile layout."""
    return pack_rows(raw, input_features, "Q6_K", device)


def unpack_rows(packed):
    """Inverse byte transform -> ``uint8[N, ceil(K/block_values), bpb]`` on the device."""
    size = BLOCK_LAYOUTS[packed.qtype][1]
    out = torch.empty((packed.output_features, packed.input_blocks, size), dtype=torch.uint8,
                      device=packed.data.device)
    with torch.cuda.device(packed.data.device):
        _lib.call("qk_unpack_rows", _lib.ptr(packed.data), GGML_TYPE[packed.qtype],
                  packed.output_features, packed.input_features, _lib.ptr(out),
                  _lib.stream_handle(packed.data.device))
    return out


unpack_q6 = unpack_rows

# The reference's TPU input form of a Q6_K projection (packed_q6/layout.py:13-18, 49-91):
# per (64-row tile, K block) a 13,312-byte data tile and a 128-byte scale tile; the scale
# plane is padded to whole 512-byte fetch windows.
SOA_TILE_BYTES = 64 * 208
SOA_SCALE_TILE_BYTES = 64 * 2
SOA_SCALE_FETCH_BYTES = 512


def soa_plane_bytes(output_features, input_features):
    """``(data bytes, scale bytes)`` of the reference's ``PackedQ6`` planes."""
    tiles = (output_features + 63) // 64
    blocks = (input_features + 255) // 256
    scale = tiles * blocks * SOA_SCALE_TILE_BYTES
    scale = (scale + SOA_SCALE_FETCH_BYTES - 1) // SOA_SCALE_FETCH_BYTES * SOA_SCALE_FETCH_BYTES
    return tiles * blocks * SOA_TILE_BYTES, scale


def _flat_u8(plane, device):
    if isinstance(plane, np.ndarray):
        if plane.dtype != np.uint8:
            return None
        return torch.from_numpy(np.ascontiguousarray(plane).reshape(-1)).to(device)
    if not isinstance(plane, torch.Tensor) or plane.dtype != torch.uint8:
        return None
    return plane.reshape(-1).to(device).contiguous()


def from_soa(data, scales=None, input_features=None, output_features=None, device=None):
    """The reference's ``PackedQ6`` planes -> this build's tiles on the device.

    ``data``/``scales`` are the flat uint8 planes of ``packed_q6.layout.pack_q6``
    (``layout.py:49-91``), NumPy or torch; or pass a ``PackedQ6``-like object (``.data``,
    ``.scales``, ``.input_features``, ``.output_features``) as ``data``. The planes go back
    to GGUF rows on the device (``qk_q6_soa_to_rows``, the inverse of ``pack_q6``) and are
    repacked into the tile layout, all on the device and without arithmetic, so the result
    equals ``pack_q6`` of the original rows byte for byte."""
    if scales is None and hasattr(data, "scales"):
        data, scales, input_features, output_features = (
            data.data, data.scales, data.input_features, data.output_features)
    if type(input_features) is not int or input_features < 1:
        raise ValueError("input_features must be a positive integer")
    if type(output_features) is not int or output_features < 1:
        raise ValueError("output_features must be positive")
    device = torch.device(device or "cuda")
    want_data, want_scales = soa_plane_bytes(output_features, input_features)
    d = _flat_u8(data, device)
    if d is None or d.numel() != want_data or (getattr(data, "ndim", 1) != 1):
        raise ValueError("Packed Q6 dtype/shape does not match projection dimensions")
    sc = _flat_u8(scales, device)
    if sc is None or sc.numel() != want_scales or (getattr(scales, "ndim", 1) != 1):
        raise ValueError("Packed Q6 scale dtype/shape does not match projection dimensions")
    blocks = (input_features + 255) // 256
    raw = torch.empty((output_features, blocks, 210), dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        _lib.call("qk_q6_soa_to_rows", _lib.ptr(d), _lib.ptr(sc), output_features, input_features,
                  _lib.ptr(raw), _lib.stream_handle(device))
    return pack_rows(raw, input_features, "Q6_K", device)


def dequantize_packed(packed, dtype=torch.bfloat16, *, fused=False):
    """Decode tiles through the GEMM kernels' fragment decoder -> ``[N, K]``.

    ``fused=False`` reproduces the reference bit for bit (signed zeros included);
    ``fused=True`` runs the fused multiply-add form of the GEMM kernels (same values, a
    zero may carry the other sign)."""
    out = torch.empty((packed.output_features, packed.input_features), dtype=dtype,
                      device=packed.data.device)
    with torch.cuda.device(packed.data.device):
        _lib.call("qk_dequantize_tiled", _lib.ptr(packed.data), GGML_TYPE[packed.qtype],
                  packed.output_features, packed.input_features,
                  (_lib.QK_OUT_BF16 if dtype == torch.bfloat16 else _lib.QK_OUT_F32)
                  | (_lib.QK_DECODE_FUSED if fused else 0),
                  _lib.ptr(out), _lib.stream_handle(packed.data.device))
    return out


_workspaces = {}


def _workspace(device, nbytes):
    """Per-device scratch for the activation tiles (grown on demand, never shrunk)."""
    key = device.index
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def quant_matmul(x, packed):
    """FP32 ``x @ bf16(decode(W)).T`` with the weights kept packed (tcgen05 tensor core)."""
    if not isinstance(x, torch.Tensor) or x.dim() != 2 or min(x.shape) < 1 or x.dtype != torch.bfloat16:
        raise ValueError("x must be a nonempty [M,K] BF16 array")
    if x.shape[1] != packed.input_features:
        raise ValueError("Packed dtype/shape does not match projection dimensions")
    x = x.contiguous()
    out = torch.empty((x.shape[0], packed.output_features), dtype=torch.float32, device=x.device)
    need = int(_lib.load().qk_quant_gemm_workspace_bytes(x.shape[0], x.shape[1],
                                                        packed.output_features))
    ws = _workspace(x.device, need)
    with torch.cuda.device(x.device):
        _lib.call("qk_quant_gemm", _lib.ptr(x), x.shape[0], x.shape[1], _lib.ptr(packed.data),
                  GGML_TYPE[packed.qtype], packed.output_features, _lib.ptr(out), _lib.ptr(ws),
                  ws.numel(), _lib.stream_handle(x.device))
    return out


def q8_matmul(x, packed, *, output_dtype=None):
    """``qwen38_tpu/compute.py:20-34`` ``q8_matmul(x, packed, *, output_dtype=None)``: the W8A8
    integer dot over Q8_0 weights (tiles of :func:`pack_rows`), on the tcgen05 tensor core
    (kind::i8). Returns ``[M, N]`` in ``output_dtype`` (default: x's dtype, BF16)."""
    if not isinstance(x, torch.Tensor) or x.dim() != 2 or min(x.shape) < 1 or x.dtype != torch.bfloat16:
        raise ValueError("x must be a nonempty [M,K] BF16 array")
    if packed.qtype != "Q8_0" or x.shape[1] != packed.input_features:
        raise ValueError("Packed dtype/shape does not match projection dimensions")
    dtype = torch.bfloat16 if output_dtype is None else output_dtype
    if dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("output_dtype must be BF16 or FP32")
    x = x.contiguous()
    out = torch.empty((x.shape[0], packed.output_features), dtype=dtype, device=x.device)
    need = int(_lib.load().qk_q8_matmul_workspace_bytes(x.shape[0], x.shape[1], packed.output_features))
    ws = _workspace(x.device, need)
    with torch.cuda.device(x.device):
        _lib.call("qk_q8_matmul", _lib.ptr(x), x.shape[0], x.shape[1], _lib.ptr(packed.data),
                  packed.output_features, _lib.QK_OUT_BF16 if dtype == torch.bfloat16 else _lib.QK_OUT_F32,
                  _lib.ptr(out), _lib.ptr(ws), ws.numel(), _lib.stream_handle(x.device))
    return out


def q6_matmul(x, packed, scales=None, *, output_features, batch_tile=8):
    """``packed_q6.kernel.q6_matmul`` contract: FP32 ``[M, N]``; validates like the reference.

    ``packed`` is a :class:`PackedWeights` of this build's tiles, or, with ``scales``, the
    reference's flat ``PackedQ6`` data plane (``kernel.py:99``: ``q6_matmul(x, packed,
    scales, *, output_features)``), which is converted on the device first
    (:func:`from_soa`; convert once with it to keep the conversion out of a loop)."""
    if not isinstance(x, torch.Tensor) or x.dim() != 2 or min(x.shape) < 1 or x.dtype != torch.bfloat16:
        raise ValueError("x must be a nonempty [M,K] BF16 array")
    if type(output_features) is not int or output_features < 1:
        raise ValueError("output_features must be positive")
    if type(batch_tile) is not int or batch_tile < 8 or batch_tile % 8:
        raise ValueError("batch_tile must be a positive multiple of 8")
    if scales is not None:
        packed = from_soa(packed, scales, x.shape[1], output_features, x.device)
    if packed.qtype != "Q6_K" or packed.output_features != output_features or (
        packed.input_features != x.shape[1]
    ):
        raise ValueError("Packed Q6 dtype/shape does not match projection dimensions")
    return quant_matmul(x, packed)


def linear_workspace(M, K, N, device):
    """A zeroed workspace for ``qk_linear_bf16`` at these sizes (zeroed once; every call leaves
    it ready for the next)."""
    nbytes = int(_lib.load().qk_linear_bf16_workspace_bytes(M, K, N))
    if nbytes == 0:
        raise ValueError("linear_bf16 takes 1 <= M <= 256 rows and K a multiple of 64")
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def linear_bf16(x, weight, out=None, workspace=None):
    """``linear(x, weight)`` of ``qwen38_tpu/math.py:10-16`` for BF16 operands at decode batch
    sizes: ``bf16(x @ weight^T)`` with FP32 accumulation on the tensor core (x: BF16 [M, K],
    1 <= M <= 256; weight: BF16 [N, K])."""
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or x.dim() != 2 or weight.dim() != 2:
        raise TypeError("x and weight must be BF16 matrices")
    M, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError("weight must be [N, K] for x [M, K]")
    x, weight = x.contiguous(), weight.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = linear_workspace(M, K, N, x.device)
    with torch.cuda.device(x.device):
        _lib.call("qk_linear_bf16", _lib.ptr(x), M, K, _lib.ptr(weight), N, _lib.ptr(out), _lib.ptr(workspace),
                  workspace.numel(), _lib.stream_handle(x.device))
    return out
