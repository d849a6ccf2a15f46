"""GGUF block decoders and the build's deterministic encoders (oracle, test infrastructure).

Decoders restate ``kaggle/glm53_offload/gguf_quant.py:63-177`` (Q4_K, Q5_K, Q6_K,
Q8_0, F16, BF16, F32) and ``kaggle/qwen38_tpu/quant.py:15-55`` (Q4_0, Q4_1, Q5_0,
Q5_1, IQ4_NL). The Q6_K position rule is the scalar one of
``kaggle/packed_q6/reference.py:11-32``. Input is the raw little-endian GGUF payload
viewed as ``uint8[..., blocks_per_row, bytes_per_block]``; output is FP32
``[..., row_width]`` (the decoded padding of a partial last block is cropped).

The reference has no Q6_K/Q4_K quantiser (``gguf_quant.py:1-12`` "never quantizes";
gguf-py 0.19.0 raises NotImplementedError for both). ``encode_q6_k`` and
``encode_q4_k`` below are this build's own deterministic encoders, used only to
make synthetic weights; parity is defined on the decode of their bytes.
``encode_q8_0`` restates the reference's ``pack_q8`` (``qwen38_tpu/compute.py:41-49``).
"""

import numpy as np

# (values per block, bytes per block), GGML type sizes (gguf_quant.py:21-29, quant.py:8).
BLOCK_LAYOUTS = {
    "Q4_0": (32, 18),
    "Q4_1": (32, 20),
    "Q5_0": (32, 22),
    "Q5_1": (32, 24),
    "Q8_0": (32, 34),
    "Q4_K": (256, 144),
    "Q5_K": (256, 176),
    "Q6_K": (256, 210),
    "IQ4_NL": (32, 18),
    "F16": (1, 2),
    "BF16": (1, 2),
    "F32": (1, 4),
}

# GGML type numbers, also used across the C ABI (include/qk_b200.h).
GGML_TYPE = {
    "F32": 0,
    "F16": 1,
    "Q4_0": 2,
    "Q4_1": 3,
    "Q5_0": 6,
    "Q5_1": 7,
    "Q8_0": 8,
    "Q4_K": 12,
    "Q5_K": 13,
    "Q6_K": 14,
    "IQ4_NL": 20,
    "BF16": 30,
}

IQ4_VALUES = np.array(
    (-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113), np.float32
)


def block_layout(qtype):
    return BLOCK_LAYOUTS[qtype]


def _f16(lo, hi):
    bits = lo.astype(np.uint16) | (hi.astype(np.uint16) << np.uint16(8))
    return bits.view(np.float16).astype(np.float32)


def _i8(b):
    return b.view(np.int8).astype(np.int32)


def _q6_k_index():
    """Per output position p of a Q6_K block: (ql byte, nibble shift, qh byte, qh shift, scale).

    ``packed_q6/reference.py:21-29``: half = p // 128, quarter = (p % 128) // 32,
    lane = p % 32; low nibble from ``ql[half*64 + (quarter % 2)*32 + lane]`` shifted by
    ``4*(quarter // 2)``; high two bits from ``qh[half*32 + lane] >> 2*quarter``;
    signed sub-scale ``scales[p // 16]``.
    """
    p = np.arange(256)
    half, quarter, lane = p // 128, (p % 128) // 32, p % 32
    return (
        half * 64 + (quarter % 2) * 32 + lane,
        4 * (quarter // 2),
        128 + half * 32 + lane,
        2 * quarter,
        192 + p // 16,
    )


_Q6 = _q6_k_index()


def _q4_k_scales(raw):
    """6-bit sub-block scales and mins of Q4_K/Q5_K (``gguf_quant.py:118-135``)."""
    s = raw[..., 4:16].astype(np.int32)
    sc = np.empty(raw.shape[:-1] + (8,), np.int32)
    mn = np.empty_like(sc)
    for j in range(4):
        sc[..., j] = s[..., j] & 63
        mn[..., j] = s[..., j + 4] & 63
        sc[..., j + 4] = (s[..., j + 8] & 15) | ((s[..., j] >> 6) << 4)
        mn[..., j + 4] = (s[..., j + 8] >> 4) | ((s[..., j + 4] >> 6) << 4)
    return sc, mn


def decode_blocks(raw, qtype):
    """Decode ``uint8[..., nblk, bpb]`` into FP32 ``[..., nblk * values_per_block]``."""
    raw = np.asarray(raw)
    if raw.dtype != np.uint8:
        raise TypeError(f"raw must have dtype uint8; got {raw.dtype}")
    values, size = BLOCK_LAYOUTS[qtype]
    if raw.ndim < 2 or raw.shape[-1] != size:
        raise ValueError(f"{qtype} blocks contain {size} bytes; got {raw.shape[-1:]}")
    lead, nblk = raw.shape[:-2], raw.shape[-2]
    if qtype == "F32":
        out = np.ascontiguousarray(raw).view("<f4").astype(np.float32)
    elif qtype == "F16":
        out = _f16(raw[..., 0], raw[..., 1])
    elif qtype == "BF16":
        bits = (raw[..., 0].astype(np.uint32) | (raw[..., 1].astype(np.uint32) << 8)) << 16
        out = bits.view(np.float32)
    elif qtype == "Q8_0":
        d = _f16(raw[..., 0], raw[..., 1])
        out = d[..., None] * _i8(raw[..., 2:]).astype(np.float32)
    elif qtype == "Q6_K":
        lo_i, lo_s, hi_i, hi_s, sc_i = _Q6
        lo = (raw[..., lo_i].astype(np.int32) >> lo_s) & 15
        hi = (raw[..., hi_i].astype(np.int32) >> hi_s) & 3
        q = ((lo | (hi << 4)) - 32).astype(np.float32)
        sc = _i8(raw[..., sc_i]).astype(np.float32)
        d = _f16(raw[..., 208], raw[..., 209])
        out = (d[..., None] * sc) * q  # gguf_quant.py:171 order: (d * scale) * q
    elif qtype in ("Q4_K", "Q5_K"):
        d = _f16(raw[..., 0], raw[..., 1])[..., None]
        dmin = _f16(raw[..., 2], raw[..., 3])[..., None]
        sc, mn = _q4_k_scales(raw)
        p = np.arange(256)
        j, i = p // 32, p % 32
        if qtype == "Q4_K":
            q = (raw[..., 16 + (j // 2) * 32 + i].astype(np.int32) >> (4 * (j % 2))) & 15
        else:
            lo = (raw[..., 48 + (j // 2) * 32 + i].astype(np.int32) >> (4 * (j % 2))) & 15
            hi = (raw[..., 16 + i].astype(np.int32) >> j) & 1
            q = lo | (hi << 4)
        scale = sc[..., j].astype(np.float32)
        mins = mn[..., j].astype(np.float32)
        out = (d * scale) * q.astype(np.float32) - dmin * mins  # gguf_quant.py:154-157
    elif qtype in ("Q4_0", "Q4_1", "Q5_0", "Q5_1", "IQ4_NL"):
        affine = qtype in ("Q4_1", "Q5_1")
        base = 4 if affine else 2
        five = qtype.startswith("Q5")
        low = raw[..., base + (4 if five else 0) :].astype(np.int32)
        q = np.concatenate((low & 15, low >> 4), axis=-1)
        if five:
            f = raw[..., base : base + 4].astype(np.uint32)
            bits = f[..., 0] | (f[..., 1] << 8) | (f[..., 2] << 16) | (f[..., 3] << 24)
            q = q | (((bits[..., None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.int32) << 4)
        d = _f16(raw[..., 0], raw[..., 1])[..., None]
        if qtype == "IQ4_NL":
            qf = IQ4_VALUES[q]
        elif affine:
            qf = q.astype(np.float32)
        else:
            qf = (q - (16 if five else 8)).astype(np.float32)
        out = d * qf
        if affine:
            out = out + _f16(raw[..., 2], raw[..., 3])[..., None]
    else:
        raise ValueError(f"unsupported GGUF quantization type: {qtype!r}")
    return np.asarray(out, np.float32).reshape(lead + (nblk * values,))


def dequantize_rows(raw, qtype, row_width):
    """``gguf_quant.dequantize_rows`` (numpy backend): decode then crop to ``row_width``."""
    values, _ = BLOCK_LAYOUTS[qtype]
    nblk = (row_width + values - 1) // values
    raw = np.asarray(raw)
    if raw.ndim < 2 or raw.shape[-2] != nblk:
        raise ValueError(f"row_width {row_width} requires {nblk} {qtype} blocks")
    return decode_blocks(raw, qtype)[..., :row_width]


# ---------------------------------------------------------------------------------------
# Encoders (synthetic weights only)
# ---------------------------------------------------------------------------------------


def _f16_bytes(values):
    return np.asarray(values, np.float32).astype("<f2").view(np.uint8).reshape(
        np.shape(values) + (2,)
    )


def encode_q8_0(weights):
    """``compute.py:41-49`` (``pack_q8``): per 32 values, FP16 ``absmax/127`` + int8 codes."""
    w = np.asarray(weights, np.float32)
    rows = w.reshape(w.shape[:-1] + (-1, 32))
    scale = (np.max(np.abs(rows), -1) / np.float32(127)).astype("<f2")
    codes = np.clip(np.rint(rows / np.where(scale == 0, 1, scale)[..., None]), -127, 127)
    return np.concatenate(
        (scale.view(np.uint8).reshape(scale.shape + (2,)), codes.astype(np.int8).view(np.uint8)),
        axis=-1,
    )


def encode_q6_k(weights):
    """Deterministic Q6_K encoder: symmetric 6-bit codes, int8 sub-scales, FP16 super-scale.

    Per 16-value sub-block j: ``s_j = max|x| / 31``. ``d = fp16(max_j s_j / 127)``,
    ``sc_j = clip(rint(s_j / d), -128, 127)``, ``q = clip(rint(x / (d * sc_j)), -32, 31)``.
    Rows must be whole 256-value blocks.
    """
    w = np.asarray(weights, np.float32)
    if w.shape[-1] % 256:
        raise ValueError("Q6_K rows must hold whole 256-value blocks")
    x = w.reshape(-1, 256)
    sub = np.abs(x.reshape(-1, 16, 16)).max(-1) / np.float32(31)
    d = (sub.max(-1) / np.float32(127)).astype(np.float16)
    df = d.astype(np.float32)
    safe = np.where(df == 0, np.float32(1), df)
    sc = np.where(df[:, None] == 0, 0, np.clip(np.rint(sub / safe[:, None]), -128, 127)).astype(
        np.int32
    )
    step = (df[:, None] * sc.astype(np.float32)).repeat(16, axis=1)
    q = np.where(step == 0, 0, np.clip(np.rint(x / np.where(step == 0, 1, step)), -32, 31))
    # u[n, half, quarter, lane]; ql[half*64 + (quarter%2)*32 + lane] holds quarters q and
    # q+2 as low/high nibbles, qh[half*32 + lane] holds the 2-bit tops of all 4 quarters.
    u = (q + 32).astype(np.uint8).reshape(-1, 2, 4, 32)
    raw = np.zeros((x.shape[0], 210), np.uint8)
    raw[:, :128] = ((u[:, :, 0:2] & 15) | ((u[:, :, 2:4] & 15) << 4)).reshape(-1, 128)
    top = u >> 4
    raw[:, 128:192] = (top[:, :, 0] | (top[:, :, 1] << 2) | (top[:, :, 2] << 4) | (top[:, :, 3] << 6)).reshape(-1, 64)
    raw[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    raw[:, 208:210] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
    return raw.reshape(w.shape[:-1] + (w.shape[-1] // 256, 210))


def encode_q4_k(weights):
    """Deterministic Q4_K encoder: asymmetric 4-bit codes with 6-bit scales and mins.

    Per 32-value sub-block j: ``lo = min(min x, 0)``, ``hi = max x``,
    ``scale_j = (hi - lo) / 15``, ``min_j = -lo``. ``d = fp16(max scale_j / 63)``,
    ``dmin = fp16(max min_j / 63)``, 6-bit ``sc_j = rint(scale_j / d)``,
    ``m_j = rint(min_j / dmin)``, ``q = clip(rint((x + dmin*m_j) / (d*sc_j)), 0, 15)``.
    """
    w = np.asarray(weights, np.float32)
    if w.shape[-1] % 256:
        raise ValueError("Q4_K rows must hold whole 256-value blocks")
    x = w.reshape(-1, 8, 32)
    lo = np.minimum(x.min(-1), 0)
    hi = x.max(-1)
    scale = (hi - lo) / np.float32(15)
    mins = -lo
    d = (scale.max(-1) / np.float32(63)).astype(np.float16)
    dmin = (mins.max(-1) / np.float32(63)).astype(np.float16)
    df, dmf = d.astype(np.float32)[:, None], dmin.astype(np.float32)[:, None]
    sc = np.where(df == 0, 0, np.clip(np.rint(scale / np.where(df == 0, 1, df)), 0, 63))
    mn = np.where(dmf == 0, 0, np.clip(np.rint(mins / np.where(dmf == 0, 1, dmf)), 0, 63))
    sc, mn = sc.astype(np.int32), mn.astype(np.int32)
    step = (df * sc.astype(np.float32))[..., None]
    off = (dmf * mn.astype(np.float32))[..., None]
    q = np.where(step == 0, 0, np.clip(np.rint((x + off) / np.where(step == 0, 1, step)), 0, 15))
    q = q.astype(np.int32)
    n = x.shape[0]
    raw = np.zeros((n, 144), np.uint8)
    raw[:, 0:2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
    raw[:, 2:4] = dmin.astype("<f2").view(np.uint8).reshape(-1, 2)
    s = np.zeros((n, 12), np.int32)
    for j in range(4):
        s[:, j] |= sc[:, j] & 63
        s[:, j + 4] |= mn[:, j] & 63
        s[:, j + 8] = (sc[:, j + 4] & 15) | ((mn[:, j + 4] & 15) << 4)
        s[:, j] |= (sc[:, j + 4] >> 4) << 6
        s[:, j + 4] |= (mn[:, j + 4] >> 4) << 6
    raw[:, 4:16] = s
    for c in range(4):
        raw[:, 16 + c * 32 : 16 + (c + 1) * 32] = q[:, 2 * c] | (q[:, 2 * c + 1] << 4)
    return raw.reshape(w.shape[:-1] + (w.shape[-1] // 256, 144))


def encode(weights, qtype):
    if qtype == "Q6_K":
        return encode_q6_k(weights)
    if qtype == "Q4_K":
        return encode_q4_k(weights)
    if qtype == "Q8_0":
        return encode_q8_0(weights)
    raise ValueError(f"no encoder for {qtype}")


def legal_q6_k_fixture(outputs, inputs, seed=3826):
    """Random legal Q6_K bytes with signed/extreme sub-scales and finite block scales.

    Same generator as ``packed_q6/reference.py:51-57`` (``fixture``), so the reference's
    golden projections can be regenerated bit-for-bit.
    """
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, (outputs, (inputs + 255) // 256, 210), dtype=np.uint8)
    scales = rng.choice(np.array([-0.003, -0.001, 0, 0.001, 0.003], dtype="<f2"), raw.shape[:2])
    raw[:, :, 208:210] = scales.view(np.uint8).reshape(*raw.shape[:2], 2)
    return raw
