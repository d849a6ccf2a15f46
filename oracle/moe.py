"""Routed-expert FFN, router top-k and packed projection oracles (test infrastructure).

* ``routes`` restates the router part of ``routes_and_shared``
  (``kaggle/qwen38_tpu/math.py:277-281``).
* ``expert_ffn`` restates the single-device semantics of ``expert_parallel.local``
  (``kaggle/qwen38_tpu/experts.py:61-131``), equal to ``grouped_expert_parallel``
  (``kaggle/qwen38_tpu/grouped_experts.py:185-292``) at tp=1: per active expert, in
  ascending expert order, ``y = bf16(bf16(silu(bf16(x Wg^T)) * bf16(x Wu^T)) Wd^T)``,
  ``out += f32(y) * f32(route)``; finally ``bf16(out)``.
* ``projection`` restates ``packed_q6/reference.py:44-48`` (``projection_reference``).
* ``q8_matmul`` restates the W8A8 integer dot ``numpy_q8_matmul``
  (``kaggle/qwen38_tpu/compute.py:52-65``), the ``int8_q8`` expert policy's Q8_0 projection
  (``compute.py:20-34``, used by ``experts.py:85-99``).
"""

import numpy as np

from .gguf import dequantize_rows
from .precision import bf16_round, divide, sigmoid, softmax


def _dot(a, b, accumulate):
    """``a @ b.T`` of FP32-valued operands: exact FP64 accumulation, or FP32 BLAS."""
    if accumulate == "f64":
        return (a.astype(np.float64) @ b.astype(np.float64).T).astype(np.float32)
    return (a.astype(np.float32) @ b.astype(np.float32).T).astype(np.float32)


def routes(x, router_weight, top_k, active=None, *, logits=None):
    """``math.py:277-281``: FP32 logits, softmax, ``lax.top_k`` (ties to the lower
    index), renormalise with ``numerics.divide``, zero inactive rows, cast to BF16.

    Returns ``(ids int32[T, k], weights float32[T, k] holding BF16 values, probs)``.
    """
    if logits is None:
        logits = _dot(np.asarray(x, np.float32), np.asarray(router_weight, np.float32), "f64")
    probs = softmax(np.asarray(logits, np.float32), axis=-1)
    ids = np.argsort(-probs, axis=-1, kind="stable")[:, :top_k].astype(np.int32)
    top = np.take_along_axis(probs, ids, axis=-1)
    total = np.zeros(top.shape[0], np.float32)
    for j in range(top_k):  # sequential FP32 sum, the order the kernel uses
        total = (total + top[:, j]).astype(np.float32)
    weights = divide(top, total[:, None])
    if active is not None:
        weights = np.where(np.asarray(active, bool)[:, None], weights, np.float32(0))
    return ids, bf16_round(weights), probs


def route_weights(ids, weights, num_experts, first=0):
    """Per-expert route weight ``[E_local, B]`` (``experts.py:66-73``), BF16-valued."""
    ids = np.asarray(ids)
    weights = np.asarray(weights, np.float32)
    out = np.zeros((num_experts, ids.shape[0]), np.float32)
    for j in range(ids.shape[1]):
        local = ids[:, j] - first
        ok = (local >= 0) & (local < num_experts)
        out[local[ok], np.nonzero(ok)[0]] += weights[ok, j]
    return bf16_round(out)


def expert_weights(raw, qtype, rows, width):
    """BF16 weights of one projection of one expert, ``[rows, width]`` as FP32 values."""
    return bf16_round(dequantize_rows(np.asarray(raw).reshape(rows, -1, _bpb(qtype)), qtype, width))


def _bpb(qtype):
    from .gguf import BLOCK_LAYOUTS

    return BLOCK_LAYOUTS[qtype][1]


def q8_matmul(x, packed):
    """``compute.py:52-65`` (``numpy_q8_matmul``): FP32 ``[rows, outputs]`` of a W8A8 dot.

    ``x``: FP32-valued ``[rows, K]``; ``packed``: Q8_0 blocks ``uint8[outputs, K / 32, 34]``.
    Per 32-value group g the activations are quantised to int8 with the FP32 scale
    ``max|x| / 127`` (``x / scale`` rounded half to even, clipped to +-127; a zero scale
    divides by 1), the int32 dot with the weight codes is taken exactly, and the groups are
    added in order: ``out += (f32(partial) * act_scale) * weight_scale``."""
    packed = np.asarray(packed, np.uint8)
    scale = np.ascontiguousarray(packed[..., :2]).view("<f2").reshape(packed.shape[:2]).astype(np.float32)
    weights = np.ascontiguousarray(packed[..., 2:]).view(np.int8).astype(np.int64)
    grouped = np.asarray(x, np.float32).reshape(x.shape[0], -1, 32)
    act_scale = (np.max(np.abs(grouped), -1) / np.float32(127)).astype(np.float32)
    codes = np.clip(np.rint(grouped / np.where(act_scale == 0, np.float32(1), act_scale)[..., None]),
                    -127, 127).astype(np.int64)
    out = np.zeros((x.shape[0], packed.shape[0]), np.float32)
    for group in range(weights.shape[1]):
        partial = (codes[:, group] @ weights[:, group].T).astype(np.float32)
        out = (out + (partial * act_scale[:, group, None]).astype(np.float32) * scale[:, group][None, :]).astype(
            np.float32)
    return out


def expert_forward(x, wg, wu, wd, accumulate="f64", down_q8=None):
    """One expert's SwiGLU on BF16-valued rows; returns BF16-valued ``y``. With ``down_q8``
    (the expert's raw Q8_0 down blocks ``[hidden, I / 32, 34]``) the down projection is the
    ``int8_q8`` policy's W8A8 dot (``experts.py:96-107``) instead of the BF16 one."""
    g = bf16_round(_dot(x, wg, accumulate))
    u = bf16_round(_dot(x, wu, accumulate))
    act = bf16_round((bf16_round(g * sigmoid(g)) * u).astype(np.float32))
    if down_q8 is not None:
        return bf16_round(q8_matmul(act, down_q8))
    return bf16_round(_dot(act, wd, accumulate))


def expert_ffn(
    gate,
    up,
    down,
    x,
    ids,
    weights,
    *,
    gate_type,
    up_type,
    down_type,
    hidden,
    intermediate,
    first_expert=0,
    accumulate="f64",
    partial=False,
    compute="bf16",
):
    """Routed FFN over this rank's experts ``[first_expert, first_expert + E_local)``.

    ``gate``/``up``: raw GGUF bytes ``[E_local, intermediate * row_bytes(hidden)]``;
    ``down``: ``[E_local, hidden * row_bytes(intermediate)]``. ``x``: BF16-valued
    ``[B, hidden]``; ``ids``/``weights``: ``[B, k]``. Returns BF16-valued ``[B, hidden]``,
    or the FP32 partial sum when ``partial`` (the value the EP all-reduce adds).
    ``compute="int8_q8"`` computes a Q8_0 down projection as the W8A8 dot (``q8_matmul``).
    """
    x = bf16_round(np.asarray(x, np.float32))
    count = np.asarray(gate).shape[0]
    route = route_weights(ids, weights, count, first_expert)
    out = np.zeros((x.shape[0], hidden), np.float32)
    for e in range(count):
        rows = np.nonzero(route[e])[0]
        if rows.size == 0:
            continue
        wg = expert_weights(gate[e], gate_type, intermediate, hidden)
        wu = expert_weights(up[e], up_type, intermediate, hidden)
        w8 = compute == "int8_q8" and down_type == "Q8_0"
        wd = None if w8 else expert_weights(down[e], down_type, hidden, intermediate)
        q8 = np.asarray(down[e]).reshape(hidden, -1, 34) if w8 else None
        y = expert_forward(x[rows], wg, wu, wd, accumulate, down_q8=q8)
        contribution = (y * route[e, rows][:, None]).astype(np.float32)
        out[rows] = (out[rows] + contribution).astype(np.float32)
    return out if partial else bf16_round(out)


def projection(x, raw, input_features):
    """``packed_q6/reference.py:44-48``: FP64 dot of BF16-rounded x and weights, to FP32."""
    xb = bf16_round(np.asarray(x, np.float32))
    w = bf16_round(dequantize_rows(raw, "Q6_K", input_features))
    return (xb.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
