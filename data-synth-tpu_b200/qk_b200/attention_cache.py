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


@dataclass(frozen=True)
class IndexerConfig:
    """The ``ModelConfig`` fields ``select_tokens`` reads (``config.py:28-38``)."""

    qsa_budget: int = 2048
    indexer_heads: int = 4
    indexer_dim: int = 128
    indexer_compress: int = 4
    rotary_dim: int = 64
    rope_theta: float = 10_000_000.0
    mrope_sections: tuple = (11, 11, 10)
    eps: float = 1e-6

    def __post_init__(self):
        if (self.indexer_heads < 1 or self.indexer_dim < self.rotary_dim or self.indexer_compress < 2
                or self.qsa_budget < self.indexer_compress or self.qsa_budget % self.indexer_compress):
            raise ValueError("Invalid sparse attention indexer dimensions or budget")  # config.py:59-65

    def rope_tables(self, device):
        """``(inv_freq FP32 [rotary/2], axis int32 [rotary/2])`` of ``math.py:231-238``: pair i turns
        by ``positions[axis[i]] * theta^(-2i/rotary)``."""
        import numpy as np

        half = self.rotary_dim // 2
        inv = np.power(np.float32(self.rope_theta),
                       -np.arange(half, dtype=np.float32) * 2 / np.float32(self.rotary_dim)).astype(np.float32)
        axis = np.zeros(half, np.int32)
        for dim, offset in ((1, 1), (2, 2)):
            idx = np.arange(offset, self.mrope_sections[dim] * 3, 3)
            axis[idx[idx < half]] = dim
        return torch.from_numpy(inv).to(device), torch.from_numpy(axis).to(device)


def empty_index_cache(batch, max_context, ic, device=None):
    """The indexer state of ``engine.py:372-380``: block keys, the open block's raw keys and
    its start position."""
    device = torch.device(device or "cuda")
    blocks = (max_context + ic.indexer_compress - 1) // ic.indexer_compress
    return {
        "index_keys": torch.zeros((batch, blocks, ic.indexer_dim), dtype=torch.bfloat16, device=device),
        "index_tail": torch.zeros((batch, ic.indexer_compress, ic.indexer_dim), dtype=torch.bfloat16, device=device),
        "index_start": torch.zeros((batch, 3), dtype=torch.int32, device=device),
    }


def select_tokens(x, w, cache, lengths, positions, active, c):
    """``attention_cache.py:84-125``: update the indexer state with this step's token and
    select the sparse attention's tokens. ``x`` BF16 ``[B, H]``; ``w`` holds ``index_k``
    ``[dim, H]``, ``index_q`` ``[heads * dim, H]``, ``index_k_norm`` / ``index_q_norm`` ``[dim]``
    (BF16); ``positions`` int32 ``[B, 3]``; ``c`` an :class:`IndexerConfig`. The cache's
    ``index_*`` entries are updated in place. Returns ``(indices, valid, cache)``."""
    batch = x.shape[0]
    device = x.device
    ratio, dim, heads = c.indexer_compress, c.indexer_dim, c.indexer_heads
    keys = cache["index_keys"]
    inv, axis = c.rope_tables(device)
    lens = lengths.to(device=device, dtype=torch.int32).contiguous()
    pos = positions.to(device=device, dtype=torch.int32).contiguous()
    act = None if active is None else active.to(device=device, dtype=torch.uint8).contiguous()
    x = x.contiguous()
    raw_k = torch.matmul(x, w["index_k"].t()).contiguous()     # linear(x, index_k), :90
    raw_q = torch.matmul(x, w["index_q"].t()).contiguous()     # linear(x, index_q), :98
    query = torch.empty((batch, heads, dim), dtype=torch.bfloat16, device=device)
    with torch.cuda.device(device):
        st = _lib.stream_handle(device)
        _lib.call("qk_qsa_update_keys", _lib.ptr(raw_k), _lib.ptr(lens), _lib.ptr(pos), _lib.ptr(act),
                  _lib.ptr(w["index_k_norm"].contiguous()), c.eps, _lib.ptr(inv), _lib.ptr(axis), c.rotary_dim,
                  batch, ratio, dim, keys.shape[1], _lib.ptr(cache["index_tail"]), _lib.ptr(cache["index_start"]),
                  _lib.ptr(keys), st)
        _lib.call("qk_qsa_query", _lib.ptr(raw_q), _lib.ptr(pos), _lib.ptr(w["index_q_norm"].contiguous()), c.eps,
                  _lib.ptr(inv), _lib.ptr(axis), c.rotary_dim, batch, heads, dim, _lib.ptr(query), st)
    indices, valid = select_tokens_from_keys(query, keys, lens, ratio=ratio, budget=c.qsa_budget)
    return indices, valid, cache


def select_tokens_from_keys(query, keys, lengths, *, ratio=4, budget=2048):
    """The selection half of ``attention_cache.py:84-125`` (``select_tokens``) once the block
    keys are current: ``query`` BF16 ``[B, indexer_heads, indexer_dim]`` (normed and rotated),
    ``keys`` BF16 ``[B, blocks, indexer_dim]``, ``lengths`` ``[B]`` -> ``(indices int32, valid
    bool)`` ``[B, K * ratio + ratio - 1]`` with ``K = min(budget // ratio, blocks)``, ready for
    :func:`decode_attention` (``valid=``)."""
    if budget < ratio or budget % ratio or ratio < 2:
        raise ValueError("Invalid sparse attention indexer dimensions or budget")
    if query.dtype != torch.bfloat16 or keys.dtype != torch.bfloat16:
        raise TypeError("query and keys must be BF16")
    batch, heads, dim = query.shape
    if keys.dim() != 3 or keys.shape[0] != batch or keys.shape[2] != dim:
        raise ValueError("keys must be [B, blocks, indexer_dim]")
    blocks = keys.shape[1]
    device = query.device
    K = min(budget // ratio, blocks)
    lens = lengths.to(device=device, dtype=torch.int32).contiguous()
    scores = torch.empty((batch, blocks), dtype=torch.float32, device=device)
    indices = torch.empty((batch, K * ratio + ratio - 1), dtype=torch.int32, device=device)
    valid = torch.empty(indices.shape, dtype=torch.uint8, device=device)
    q, k = query.contiguous(), keys.contiguous()
    with torch.cuda.device(device):
        st = _lib.stream_handle(device)
        _lib.call("qk_qsa_block_scores", _lib.ptr(q), _lib.ptr(k), _lib.ptr(lens), batch, heads, dim, blocks,
                  ratio, _lib.ptr(scores), st)
        _lib.call("qk_qsa_select", _lib.ptr(scores), _lib.ptr(lens), batch, blocks, ratio, budget,
                  _lib.ptr(indices), _lib.ptr(valid), st)
    return indices, valid.bool()


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


# ---- time-sharded cache (the reference's layout over ranks) ---------------------------
#
# The reference shards the cache's time axis over the "expert" mesh axis
# (engine.py:350-369: codes P(None, "expert", None), scale planes P(None, "expert")), so
# rank r holds cache times [r * T / world, (r + 1) * T / world). The dense decode step
# (attention_cache.py:146-149: indices = arange(T), mask = indices <= lengths) then
# reduces its softmax over the shards. Here each rank runs the split-KV kernel over its own
# times and writes an unnormalised partial (output, max, sum); the ranks all-gather the
# partials (rank order is time order) and a log-sum-exp combine finishes the output.


def time_shard(max_context, rank, world):
    """``(first time, times)`` of ``rank``'s slice of a ``max_context`` cache."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if max_context % world:
        raise ValueError("Cache time axis must divide evenly over the ranks")
    size = max_context // world
    return rank * size, size


def local_lengths(lengths, first):
    """Per-row last valid local slot: global slot ``t`` is valid iff ``t <= lengths[b]``
    (``attention_cache.py:148``), so local slot ``s`` is valid iff ``s <= lengths[b] - first``
    (negative: no valid slot in this shard)."""
    return lengths.to(torch.int32) - int(first)


def local_write_target(lengths, active, first, size, max_context):
    """Local time and active flag of the cache write of ``attention_cache.py:138-140``
    (``lengths`` clipped to ``[0, max_context - 1]``): only the rank whose slice holds the
    time writes it."""
    t = lengths.to(torch.int64).clamp(0, max_context - 1) - int(first)
    mine = (t >= 0) & (t < size)
    if active is not None:
        mine = mine & active.to(device=mine.device, dtype=torch.bool)
    return torch.where(mine, t, torch.zeros_like(t)).to(torch.int32), mine


def partial_set_floats(batch, hq, hd):
    """FP32 values of one partial set: ``batch * hq * hd`` outputs, then ``batch * hq``
    (max, sum) pairs."""
    return batch * hq * (hd + 2)


def split_partial(partial, batch, hq, hd):
    """Views ``(o [B, hq, hd], stats [B, hq, 2])`` of one flat partial set."""
    n = batch * hq * hd
    return partial[:n].view(batch, hq, hd), partial[n:].view(batch, hq, 2)


def decode_attention_partial(q, cache, indices, c, *, lengths=None, valid=None, workspace=None):
    """Split-KV decode attention over ``cache`` that stops before normalising: one flat FP32
    partial set (``split_partial`` gives its unnormalised output and (max, sum) views)."""
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
    need = int(_lib.load().qk_kv_q8_attention_workspace_bytes(batch, selected, hq, c.kv_heads, hd))
    ws = workspace
    if need and (ws is None or ws.numel() < need):
        ws = torch.empty(need, dtype=torch.uint8, device=device)
    partial = torch.empty(partial_set_floats(batch, hq, hd), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _lib.call("qk_kv_q8_decode_attention_partial", _lib.ptr(q.contiguous()), _lib.ptr(cache["k"]),
                  _lib.ptr(cache["v"]), _lib.ptr(cache["k_scale"]), _lib.ptr(cache["v_scale"]),
                  _lib.ptr(idx), _lib.ptr(val), _lib.ptr(lens), batch, selected, cache["k"].shape[1],
                  hq, c.kv_heads, hd, _lib.ptr(partial), _lib.ptr(ws) if need else None, need,
                  _lib.stream_handle(device))
    return partial


def combine_partials(parts, batch, hq, hd, gate=None):
    """Log-sum-exp merge of the ``R`` consecutive partial sets in ``parts`` (flat FP32, set
    order = time order), then the output gate (``attention_cache.py:169-170``):
    BF16 ``[B, hq, hd]``."""
    per = partial_set_floats(batch, hq, hd)
    if parts.dim() != 1 or parts.dtype != torch.float32 or parts.numel() % per:
        raise ValueError("parts must be a flat FP32 tensor of whole partial sets")
    device = parts.device
    g = None if gate is None else gate.to(torch.bfloat16).contiguous()
    out = torch.empty((batch, hq, hd), dtype=torch.bfloat16, device=device)
    with torch.cuda.device(device):
        _lib.call("qk_kv_q8_attention_combine", _lib.ptr(parts.contiguous()), parts.numel() // per,
                  batch, hq, hd, _lib.ptr(g), _lib.ptr(out), _lib.stream_handle(device))
    return out


def gather_partials(partial, group, world):
    """All ranks' partial sets, concatenated in rank order (one all-gather)."""
    if world == 1:
        return partial
    import torch.distributed as dist

    parts = torch.empty(world * partial.numel(), dtype=partial.dtype, device=partial.device)
    dist.all_gather_into_tensor(parts, partial, group=group)
    return parts


class TimeShardedAttention:
    """Decode step over a cache whose time axis is split over the ranks of ``group``.

    ``cache`` is this rank's slice (``empty_cache`` with ``max_context / world`` times);
    ``c.max_context`` is the whole context. ``write`` stores this step's key/value on the
    rank that owns time ``lengths[b]``; ``__call__`` attends over every rank's slots
    ``<= lengths[b]`` and returns the same BF16 ``[B, hq, hd]`` on every rank.
    """

    def __init__(self, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self._ws = None

    def shard(self, c):
        return time_shard(c.max_context, self.rank, self.world)

    def write(self, cache, key, value, lengths, active, c):
        first, size = self.shard(c)
        t, mine = local_write_target(lengths.to(key.device), active, first, size, c.max_context)
        return write_quantized(cache, key, value, t, mine, c)

    def __call__(self, q, cache, lengths, c, *, gate=None):
        first, size = self.shard(c)
        if cache["k"].shape[1] != size:
            raise ValueError("cache must hold this rank's max_context / world times")
        batch, hq, hd = q.shape
        indices = torch.arange(size, dtype=torch.int32, device=q.device).expand(batch, size)
        lens = lengths.to(q.device).clamp(0, c.max_context - 1)
        need = int(_lib.load().qk_kv_q8_attention_workspace_bytes(batch, size, hq, c.kv_heads, hd))
        if need and (self._ws is None or self._ws.numel() < need):
            self._ws = torch.empty(need, dtype=torch.uint8, device=q.device)
        partial = decode_attention_partial(q, cache, indices, c, lengths=local_lengths(lens, first),
                                           workspace=self._ws)
        parts = gather_partials(partial, self.group, self.world)
        return combine_partials(parts, batch, hq, hd, gate)
