"""Decoder-layer glue around the hot path (oracle, test infrastructure).

NumPy restatements of ``kaggle/qwen38_tpu/math.py``:

* ``rms`` ``:27-31`` - ``compute_cast(xf * rsqrt(mean(xf^2) + eps) * gamma)``;
* ``rope`` ``:231-243`` with one position for every rotary section - the first
  ``rotary`` dims rotate in (i, i + half) pairs by ``position * inv_freq[i]`` with the
  cosine and sine rounded to BF16;
* the q/gate split and q_norm / k_norm of ``attention_cache.py:129-135``;
* the shared expert's gate ``sigmoid(linear(x, shared_router))`` of ``math.py:282-283``;
* ``checked_argmax`` of ``run.py:46-55``.

The decoder stack's GPU test checks each stage of a layer with these, the KV oracle and the
routed-FFN oracle.
"""

import numpy as np

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


def checked_argmax(logits):
    """``run.py:46-55``: ``(argmax, count of non-finite)`` per row; NumPy's argmax takes the
    first maximum and treats NaN as the maximum, as ``jnp.argmax`` does."""
    logits = np.asarray(logits, np.float32)
    return np.stack([np.argmax(logits, -1), np.sum(~np.isfinite(logits), -1)], -1).astype(np.int32)
