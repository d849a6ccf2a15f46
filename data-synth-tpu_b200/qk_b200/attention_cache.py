"""Q8 KV cache on the GPU (replaces ``qwen38_tpu/attention_cache.py:15-81,152-170``).

The cache is the reference's dict: ``k``/``v`` int8 ``[B, T, kv*hd]`` and ``k_scale``/
``v_scale`` BF16 ``[B*G, T]`` (time-minor planes, ``G = kv*hd/group``,
``group = min(32, hd)``). ``write_quantized`` updates it in place (the reference donates
the cache) and returns it.
"""

from dataclasses import dataclass

import torch

from . import _lib


@dataclass(frozen=True)
class CacheConfig:
    """The ``ModelConfig`` fields the KV path reads (``config.py:11-93``)."""

    kv_heads: int = 2
    head_dim: int = 256
    query_heads: int = 16
    max_context: int = 2048
    kv_scale_gather: str = "indexed"

    def __post_init__(self):
        if type(self.max_context) is not int or not 0 < self.max_context <= 32768:
            raise ValueError("Validated context capacity must be in [1, 32768]")
        if self.kv_scale_gather not in {"indexed", "rowwise"}:
            raise ValueError("KV scale gather must be indexed or rowwise")
        if self.head_dim % self.cache_group:
            raise ValueError("KV head dimension must divide into cache quantization groups")
        if self.query_heads % self.kv_heads:
            raise ValueError("Head counts must have integer repetition factors")

    @property
    def cache_group(self):
        return min(32, self.head_dim)

    @property
    def groups(self):
        return self.kv_heads * (self.head_dim // self.cache_group)


def empty_cache(batch, c, device=None):
    device = torch.device(device or "cuda")
    width = c.kv_heads * c.head_dim
    cache = {n: torch.zeros((batch, c.max_context, width), dtype=torch.int8, device=device)
             for n in ("k", "v")}
    cache.update({n: torch.zeros((batch * c.groups, c.max_context), dtype=torch.bfloat16,
                                 device=device) for n in ("k_scale", "v_scale")})
    return cache


def _dtype_code(t):
    if t.dtype == torch.bfloat16:
        return _lib.QK_OUT_BF16
    if t.dtype == torch.float32:
        return _lib.QK_OUT_F32
    raise TypeError("expected a BF16 or FP32 tensor")


def quantize(x, group):
    """``attention_cache.py:15-23`` -> ``(int8 codes like x, bf16 scales [..., D/group])``."""
    x = x.contiguous()
    width = x.shape[-1]
    rows = x.numel() // width
    codes = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    scales = torch.empty(tuple(x.shape[:-1]) + (width // group,), dtype=torch.bfloat16,
                         device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("qk_kv_q8_quantize", _lib.ptr(x), _dtype_code(x), rows, width, group,
                  _lib.ptr(codes), _lib.ptr(scales), _lib.stream_handle(x.device))
    return codes, scales


def write_quantized(cache, key, value, indices, active, c):
    """``attention_cache.py:26-43``: quantise key/value ``[B, kv, hd]`` into row ``indices[b]``."""
    batch = key.shape[0]
    key = key.contiguous()
    value = value.to(key.dtype).contiguous()
    time = indices.to(device=key.device, dtype=torch.int32).contiguous()
    act = None if active is None else active.to(device=key.device, dtype=torch.uint8).contiguous()
    with torch.cuda.device(key.device):
        _lib.call("qk_kv_q8_append", _lib.ptr(key), _lib.ptr(value), _dtype_code(key),
                  _lib.ptr(time), _lib.ptr(act), _lib.ptr(cache["k"]), _lib.ptr(cache["v"]),
                  _lib.ptr(cache["k_scale"]), _lib.ptr(cache["v_scale"]), batch,
                  cache["k"].shape[1], c.kv_heads, c.head_dim, _lib.stream_handle(key.device))
    return cache


def gather_scale_plane(plane, indices, groups, *, method="indexed"):
    """``attention_cache.py:46-68``: ``[B*groups, T]`` plane, ``[B, S]`` indices -> ``[B, S, groups]``."""
    if indices.dim() != 2 or plane.dim() != 2 or plane.shape[0] != indices.shape[0] * groups:
        raise ValueError("Scale plane must be [batch * groups, time] for [batch, selected] indices")
    if method not in ("indexed", "rowwise"):
        raise ValueError("Scale gather method must be indexed or rowwise")
    batch, selected = indices.shape
    idx = indices.to(device=plane.device, dtype=torch.int32).contiguous()
    out = torch.empty((batch, selected, groups), dtype=plane.dtype, device=plane.device)
    with torch.cuda.device(plane.device):
        _lib.call("qk_kv_q8_gather_scales", _lib.ptr(plane.contiguous()), _lib.ptr(idx), batch,
                  selected, groups, plane.shape[1], _lib.ptr(out), _lib.stream_handle(plane.device))
    return out


def read_quantized(cache, name, indices, c, dtype, *, scale_gather=None):
    """``attention_cache.py:71-81`` -> ``[B, S, kv, hd]`` of ``compute_cast(code * scale, dtype)``."""
    scale_gather = c.kv_scale_gather if scale_gather is None else scale_gather
    if scale_gather not in ("indexed", "rowwise"):
        raise ValueError("Scale gather method must be indexed or rowwise")
    codes = cache[name]
    plane = cache[name + "_scale"]
    batch, selected = indices.shape
    idx = indices.to(device=codes.device, dtype=torch.int32).contiguous()
    out = torch.empty((batch, selected, c.kv_heads, c.head_dim), dtype=dtype, device=codes.device)
    with torch.cuda.device(codes.device):
        _lib.call("qk_kv_q8_read", _lib.ptr(codes), _lib.ptr(plane), _lib.ptr(idx), batch,
                  selected, codes.shape[1], c.kv_heads, c.head_dim,
                  _lib.QK_OUT_BF16 if dtype == torch.bfloat16 else _lib.QK_OUT_F32,
                  _lib.ptr(out), _lib.stream_handle(codes.device))
    return out


class DecodeAttention:
    """Split-KV decode attention over the Q8 cache with a cached workspace."""

    def __init__(self):
        self._ws = {}

    def __call__(self, q, cache, indices, c, *, lengths=None, valid=None, gate=None):
        if q.dtype != torch.bfloat16 or q.dim() != 3:
            raise TypeError("q must be BF16 [B, query_heads, head_dim]")
        batch, hq, hd = q.shape
        if hq != c.query_heads or hd != c.head_dim:
            raise ValueError("q must be [B, query_heads, head_dim] of the cache config")
        if (lengths is None) == (valid is None):
            raise ValueError("pass exactly one of lengths or valid")
        device = q.device
        selected = indices.shape[1]
        idx = indices.to(device=device, dtype=torch.int32).contiguous()
        lens = None if lengths is None else lengths.to(device=device, dtype=torch.int32).contiguous()
        val = None if valid is None else valid.to(device=device, dtype=torch.uint8).contiguous()
        g = None if gate is None else gate.to(torch.bfloat16).contiguous()
        need = int(_lib.load().qk_kv_q8_attention_workspace_bytes(batch, selected, hq, c.kv_heads, hd))
        key = device.index
        ws = self._ws.get(key)
        if need and (ws is None or ws.numel() < need):
            ws = torch.empty(need, dtype=torch.uint8, device=device)
            self._ws[key] = ws
        out = torch.empty((batch, hq, hd), dtype=torch.bfloat16, device=device)
        with torch.cuda.device(device):
            _lib.call("qk_kv_q8_decode_attention", _lib.ptr(q.contiguous()), _lib.ptr(cache["k"]),
                      _lib.ptr(cache["v"]), _lib.ptr(cache["k_scale"]), _lib.ptr(cache["v_scale"]),
                      _lib.ptr(idx), _lib.ptr(val), _lib.ptr(lens), _lib.ptr(g), batch, selected,
                      cache["k"].shape[1], hq, c.kv_heads, hd, _lib.ptr(out),
                      _lib.ptr(ws) if need else None, need, _lib.stream_handle(device))
        return out


decode_attention = DecodeAttention()
