"""Q8 KV cache codec, gathers and decode attention core (oracle, test infrastructure).

Restates ``kaggle/qwen38_tpu/attention_cache.py``:

* ``quantize`` ``:15-23`` - per ``group`` channels, ``s = bf16(max|x| / 127)``,
  codes ``clip(rint(x / (s == 0 ? 1 : s)), -127, 127)``;
* ``write_quantized`` ``:26-43`` - codes row at ``[b, t]``, scales into the time-minor
  plane ``[B * G, T]`` (``G = kv_heads * head_dim / group``), inactive rows unchanged;
* ``gather_scale_plane`` ``:46-68`` with the index rule of the reference's own oracle
  (``tests/test_qwen38_kv_gather.py:22-32``: negative indices wrap once, then clamp);
* ``read_quantized`` ``:71-81`` - ``compute_cast(code * scale, dtype)``;
* ``attention`` ``:159-170`` - GQA scores, BF16 boundaries, masked softmax, PV and the
  sigmoid output gate.
"""

import numpy as np

from .precision import bf16_round, divide, sigmoid, softmax


def quantize(x, group):
    """``attention_cache.py:15-23``: returns ``(int8 codes [..., D], BF16-valued scales [..., D/group])``."""
    x = np.asarray(x, np.float32)
    grouped = x.reshape(x.shape[:-1] + (-1, group))
    rounded = bf16_round((np.max(np.abs(grouped), -1) / np.float32(127)).astype(np.float32))
    divisor = np.where(rounded == 0, np.float32(1), rounded)
    codes = np.clip(np.rint(divide(grouped, divisor[..., None])), -127, 127).astype(np.int8)
    return codes.reshape(x.shape), rounded


def write_quantized(cache, key, value, indices, active, kv_heads, head_dim, group=32):
    """``attention_cache.py:26-43``, in place on NumPy arrays.

    ``cache`` holds ``k``, ``v``: int8 ``[B, T, kv*hd]``; ``k_scale``, ``v_scale``:
    BF16-valued FP32 ``[B * G, T]``. ``key``/``value``: ``[B, kv, hd]``.
    """
    batch = key.shape[0]
    groups = kv_heads * (head_dim // group)
    for name, token in (("k", key), ("v", value)):
        codes, scale = quantize(token, group)
        codes = codes.reshape(batch, -1)
        scale = scale.reshape(batch, groups)
        for b in range(batch):
            if not active[b]:
                continue
            t = int(indices[b])
            cache[name][b, t] = codes[b]
            cache[name + "_scale"][b * groups : (b + 1) * groups, t] = scale[b]
    return cache


def _time_index(t, size):
    """Index rule of ``test_qwen38_kv_gather.py:26-29``."""
    t = int(t)
    if t < 0:
        t += size
    return min(max(t, 0), size - 1)


def gather_scale_plane(plane, indices, groups):
    """``attention_cache.py:46-68`` -> ``[B, S, groups]``."""
    plane = np.asarray(plane)
    indices = np.asarray(indices)
    if indices.ndim != 2 or plane.ndim != 2 or plane.shape[0] != indices.shape[0] * groups:
        raise ValueError("Scale plane must be [batch * groups, time] for [batch, selected] indices")
    out = np.empty(indices.shape + (groups,), plane.dtype)
    for b in range(indices.shape[0]):
        for s in range(indices.shape[1]):
            t = _time_index(indices[b, s], plane.shape[1])
            out[b, s] = plane[b * groups : (b + 1) * groups, t]
    return out


def read_quantized(codes, plane, indices, kv_heads, head_dim, group=32, dtype="bf16"):
    """``attention_cache.py:71-81`` -> ``[B, S, kv, hd]`` (BF16-valued unless ``dtype='f32'``)."""
    codes = np.asarray(codes)
    indices = np.asarray(indices)
    batch, selected = indices.shape
    groups = kv_heads * (head_dim // group)
    scale = gather_scale_plane(plane, indices, groups).astype(np.float32)
    rows = np.empty((batch, selected, codes.shape[2]), np.float32)
    for b in range(batch):
        for s in range(selected):
            rows[b, s] = codes[b, _time_index(indices[b, s], codes.shape[1])]
    values = rows.reshape(batch, selected, groups, group) * scale[..., None]
    values = values.reshape(batch, selected, kv_heads, head_dim).astype(np.float32)
    return bf16_round(values) if dtype == "bf16" else values


def attention(q, keys, values, mask, gate=None):
    """Decode attention core, ``attention_cache.py:159-170``.

    ``q``: BF16-valued ``[B, hq, hd]``; ``keys``/``values``: BF16-valued
    ``[B, S, kv, hd]``; ``mask``: bool ``[B, S]``; ``gate``: optional ``[B, hq, hd]``.
    Returns BF16-valued ``[B, hq, hd]`` (before the output projection).
    """
    batch, hq, hd = q.shape
    kv = keys.shape[2]
    r = hq // kv
    qg = q.reshape(batch, kv, r, hd).astype(np.float64)
    raw = np.einsum("bkrd,btkd->bkrt", qg, keys.astype(np.float64)).astype(np.float32)
    raw = bf16_round(raw)
    score = bf16_round((raw / np.float32(np.sqrt(hd))).astype(np.float32))
    score = np.where(mask[:, None, None, :], score, np.float32(-np.inf)).astype(np.float32)
    with np.errstate(invalid="ignore"):
        prob = bf16_round(softmax(score, axis=-1))
    out = np.einsum("bkrt,btkd->bkrd", prob.astype(np.float64), values.astype(np.float64))
    out = bf16_round(out.astype(np.float32)).reshape(batch, hq, hd)
    if gate is not None:
        out = bf16_round((out * bf16_round(sigmoid(gate))).astype(np.float32))
    return out


def attention_partial(q, keys, values, mask):
    """One time shard of the decode attention (test infrastructure for the time-sharded
    path; the reference reduces ``attention_cache.py:159-168`` over the shards of
    ``engine.py:350-369`` inside SPMD). Scores as in ``attention``; then per (row, head)
    ``m = max`` valid score, ``l = sum exp(score - m)``, ``o = sum exp(score - m) * v``.
    Returns the flat FP32 partial set: ``o`` ``[B, hq, hd]`` then ``(m, l)`` ``[B, hq, 2]``."""
    batch, hq, hd = q.shape
    kv = keys.shape[2]
    r = hq // kv
    qg = q.reshape(batch, kv, r, hd).astype(np.float64)
    raw = bf16_round(np.einsum("bkrd,btkd->bkrt", qg, keys.astype(np.float64)).astype(np.float32))
    score = bf16_round((raw / np.float32(np.sqrt(hd))).astype(np.float32)).astype(np.float64)
    score = np.where(mask[:, None, None, :], score, -np.inf)
    m = np.max(score, axis=-1) if score.shape[-1] else np.full(score.shape[:-1], -np.inf)
    with np.errstate(invalid="ignore"):
        p = np.where(np.isfinite(m)[..., None], np.exp(score - m[..., None]), 0.0)
    l_sum = p.sum(-1)
    o = np.einsum("bkrt,btkd->bkrd", p, values.astype(np.float64))
    stats = np.stack([m, l_sum], -1).reshape(batch, hq, 2)
    return np.concatenate([o.reshape(-1), stats.reshape(-1)]).astype(np.float32)


def combine_partials(parts, batch, hq, hd, gate=None):
    """Log-sum-exp merge of consecutive flat partial sets (``attention_partial``) in set
    order, then BF16 and the output gate of ``attention_cache.py:169-170``."""
    per = batch * hq * (hd + 2)
    parts = np.asarray(parts, np.float64).reshape(-1, per)
    o = parts[:, : batch * hq * hd].reshape(-1, batch, hq, hd)
    st = parts[:, batch * hq * hd :].reshape(-1, batch, hq, 2)
    m_all = st[..., 0].max(0)
    with np.errstate(invalid="ignore"):
        f = np.where(np.isfinite(st[..., 0]), np.exp(st[..., 0] - m_all[None]), 0.0)
        out = (o * f[..., None]).sum(0) / (st[..., 1] * f).sum(0)[..., None]
    out = bf16_round(out.astype(np.float32))
    if gate is not None:
        out = bf16_round((out * bf16_round(sigmoid(gate))).astype(np.float32))
    return out


def qsa_scores(query, keys, lengths, ratio):
    """``attention_cache.py:100-114``: ``sum_h relu(q_h . k_t) / sqrt(dim)`` (FP32 values from an
    exact dot), ``-inf`` for blocks ``t >= (lengths + 1) // ratio``."""
    q = np.asarray(query, np.float64)
    k = np.asarray(keys, np.float64)
    dots = np.einsum("bhd,btd->bth", q, k).astype(np.float32)
    scores = (np.maximum(dots, 0).astype(np.float64).sum(-1) / np.sqrt(q.shape[-1])).astype(np.float32)
    count = (np.asarray(lengths) + 1) // ratio
    return np.where(np.arange(k.shape[1])[None, :] < count[:, None], scores, np.float32(-np.inf)).astype(np.float32)


def qsa_select(scores, lengths, ratio, budget):
    """``attention_cache.py:115-124``: ``lax.top_k`` (score descending, ties to the lower
    block), then the selected blocks' tokens and the tail tokens, invalid entries index 0."""
    scores = np.asarray(scores, np.float32)
    batch, blocks = scores.shape
    K = min(budget // ratio, blocks)
    lengths = np.asarray(lengths)
    count = (lengths + 1) // ratio
    out_i, out_v = [], []
    for b in range(batch):
        order = np.lexsort((np.arange(blocks), -scores[b].astype(np.float64)))[:K]
        tokens = (order[:, None] * ratio + np.arange(ratio)).reshape(-1)
        ok = np.repeat(order < count[b], ratio)
        tail = count[b] * ratio + np.arange(ratio - 1)
        tail_ok = np.arange(ratio - 1) < (lengths[b] + 1) % ratio
        idx = np.concatenate([tokens, tail])
        val = np.concatenate([ok, tail_ok])
        out_i.append(np.where(val, idx, 0).astype(np.int32))
        out_v.append(val)
    return np.stack(out_i), np.stack(out_v)


def qsa_rope(x, positions, inv, axis, rotary):
    """``math.py:231-243`` with three position components: ``x`` ``[B, heads, dim]``,
    ``positions`` ``[B, 3]``; pair i turns by ``positions[:, axis[i]] * inv[i]``."""
    half = rotary // 2
    angles = (np.asarray(positions, np.float32)[:, axis] * inv[None, :]).astype(np.float32)
    cs = bf16_round(np.cos(angles.astype(np.float64)).astype(np.float32))[:, None, :]
    sn = bf16_round(np.sin(angles.astype(np.float64)).astype(np.float32))[:, None, :]
    a, b = x[..., :half], x[..., half:rotary]
    rot = np.concatenate([(a * cs - b * sn).astype(np.float32), (b * cs + a * sn).astype(np.float32)], -1)
    return np.concatenate([bf16_round(rot), x[..., rotary:]], -1)


def _rms(x, gamma, eps):
    x = np.asarray(x, np.float32)
    mean = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    r = (1.0 / np.sqrt(mean + eps)).astype(np.float32)
    return bf16_round(((x * r).astype(np.float32) * np.asarray(gamma, np.float32)).astype(np.float32))


def qsa_update(state, raw_k, lengths, positions, active, k_norm, eps, inv, axis, rotary, ratio):
    """``attention_cache.py:86-97`` on NumPy state ``{index_keys [B, blocks, dim],
    index_tail [B, ratio, dim], index_start [B, 3]}`` (in place)."""
    lengths = np.asarray(lengths)
    for b in range(len(lengths)):
        slot = lengths[b] % ratio
        if active[b]:
            state["index_tail"][b, slot] = raw_k[b]
            if slot == 0:
                state["index_start"][b] = positions[b]
    pooled = bf16_round(np.mean(state["index_tail"].astype(np.float64), axis=1).astype(np.float32))
    block = qsa_rope(_rms(pooled, k_norm, eps)[:, None, :], state["index_start"], inv, axis, rotary)[:, 0]
    for b in range(len(lengths)):
        if active[b] and lengths[b] % ratio == ratio - 1:
            state["index_keys"][b, lengths[b] // ratio] = block[b]
    return state


def qsa_query(raw_q, positions, q_norm, eps, inv, axis, rotary):
    """``attention_cache.py:98-99``: rope(rms(raw_q, q_norm), positions), ``raw_q`` ``[B, heads, dim]``."""
    return qsa_rope(_rms(raw_q, q_norm, eps), positions, inv, axis, rotary)
