"""Decoder-layer glue around the hot path (oracle, test infrastructure).

NumPy restatements of ``kaggle/qwen38_tpu/math.py``:

* ``rms`` ``:27-31`` - ``compute_cast(xf * rsqrt(mean(xf^2) + eps) * gamma)``;
* ``rope`` ``:231-243`` with one position for every rotary section - the first
  ``rotary`` dims rotate in (i, i + half) pairs by ``position * inv_freq[i]`` with the
  cosine and sine rounded to BF16;
* the q/gate split and q_norm / k_norm of ``attention_cache.py:129-135``;
* the shared expert's gate ``sigmoid(linear(x, shared_router))`` of ``math.py:282-283``;

and a whole decode step of the synthetic stack (``decode_step``) built from these, the KV
oracle and the routed-FFN oracle.
"""

import numpy as np

from . import kv, moe
from .precision import bf16_round, sigmoid


def rms(x, gamma, eps):
    x = np.asarray(x, np.float32)
    mean = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    r = (1.0 / np.sqrt(mean.astype(np.float64) + eps)).astype(np.float32)
    return bf16_round(((x * r).astype(np.float32) * np.asarray(gamma, np.float32)).astype(np.float32))


def inv_freq(rotary, theta):
    half = rotary // 2
    return np.power(np.float32(theta), -np.arange(half, dtype=np.float32) * 2 / np.float32(rotary)).astype(np.float32)


def rope(x, positions, inv, rotary):
    """``x`` ``[B, heads, hd]`` BF16-valued, ``positions`` ``[B]``."""
    half = rotary // 2
    angles = (np.asarray(positions, np.float32)[:, None] * inv[None, :]).astype(np.float32)
    cs = bf16_round(np.cos(angles.astype(np.float64)).astype(np.float32))[:, None, :]
    sn = bf16_round(np.sin(angles.astype(np.float64)).astype(np.float32))[:, None, :]
    a, b = x[..., :half], x[..., half:rotary]
    rot = np.concatenate([(a * cs - b * sn).astype(np.float32), (b * cs + a * sn).astype(np.float32)], -1)
    return np.concatenate([bf16_round(rot), x[..., rotary:]], -1)


def qk_norm_rope(qkv, q_norm, k_norm, positions, hq, kvh, hd, rotary, theta, eps):
    """Fused projection rows ``[B, hq*(q|gate) + kv*k + kv*v]`` -> ``(q, gate, k, v)``."""
    B = qkv.shape[0]
    qg = qkv[:, : 2 * hq * hd].reshape(B, hq, 2 * hd)
    q, gate = qg[..., :hd], qg[..., hd:]
    k = qkv[:, 2 * hq * hd : 2 * hq * hd + kvh * hd].reshape(B, kvh, hd)
    v = qkv[:, 2 * hq * hd + kvh * hd :].reshape(B, kvh, hd)
    inv = inv_freq(rotary, theta)
    q = rope(rms(q, q_norm, eps), positions, inv, rotary)
    k = rope(rms(k, k_norm, eps), positions, inv, rotary)
    return q, gate, k, v


def shared_gate(h, shared_router):
    """``bf16(sigmoid(bf16(h . w)))`` per row."""
    dot = bf16_round((np.asarray(h, np.float64) @ np.asarray(shared_router, np.float64)).astype(np.float32))
    return bf16_round(sigmoid(dot))


def linear(x, w):
    """``compute_cast(x @ w^T)`` with exact accumulation, math.py:10-16."""
    return bf16_round((np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32))


def decode_step(x, layers, caches, indices, positions, cfg):
    """One decode step of the synthetic stack (the layer order of ``qk_b200.decoder``).

    ``layers``: per layer a dict of FP32-valued weights (``w_qkv``, ``w_o``, norms,
    ``router``, ``shared_router``) and raw GGUF expert bytes ``gate``/``up``/``down``
    ``[experts + 1, bytes]`` (the last one the shared expert); ``caches``: per layer the
    KV oracle's cache dict, updated in place. Returns the new BF16-valued ``x``."""
    hq, kvh, hd = cfg.query_heads, cfg.kv_heads, cfg.head_dim
    x = bf16_round(np.asarray(x, np.float32))
    for L, cache in zip(layers, caches):
        h = rms(x, L["attn_norm"], cfg.eps)
        qkv = linear(h, L["w_qkv"])
        q, gate, k, v = qk_norm_rope(qkv, L["q_norm"], L["k_norm"], positions, hq, kvh, hd, cfg.rotary_dim,
                                     cfg.rope_theta, cfg.eps)
        kv.write_quantized(cache, k, v, positions, np.ones(len(positions), bool), kvh, hd)
        keys = kv.read_quantized(cache["k"], cache["k_scale"], indices, kvh, hd)
        values = kv.read_quantized(cache["v"], cache["v_scale"], indices, kvh, hd)
        mask = np.arange(indices.shape[1])[None, :] <= np.asarray(positions)[:, None]
        o = kv.attention(q, keys, values, mask, gate)
        x = bf16_round((x + linear(o.reshape(len(x), -1), L["w_o"])).astype(np.float32))
        h2 = rms(x, L["ffn_norm"], cfg.eps)
        ids, w, _ = moe.routes(h2, L["router"], cfg.top_k)
        ids = np.concatenate([ids, np.full((len(x), 1), cfg.experts, np.int32)], 1)
        w = np.concatenate([w, shared_gate(h2, L["shared_router"])[:, None]], 1)
        y = moe.expert_ffn(L["gate"], L["up"], L["down"], h2, ids, w, gate_type=cfg.qtype, up_type=cfg.qtype,
                           down_type=cfg.qtype, hidden=cfg.hidden, intermediate=cfg.intermediate)
        x = bf16_round((x + y).astype(np.float32))
    return x


def checked_argmax(logits):
    """``run.py:46-55``: ``(argmax, count of non-finite)`` per row; NumPy's argmax takes the
    first maximum and treats NaN as the maximum, as ``jnp.argmax`` does."""
    logits = np.asarray(logits, np.float32)
    return np.stack([np.argmax(logits, -1), np.sum(~np.isfinite(logits), -1)], -1).astype(np.int32)
