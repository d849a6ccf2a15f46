"""NumPy statement of the B200 tiled weight layout (oracle for the repack kernels).

This is the build's own lossless byte layout (the reference's analogue is the TPU SoA
repack ``kaggle/packed_q6/layout.py:49-108``, which groups 64 rows x 256 values into
separate ql/qh/scale/d regions). Here a tile is 64 rows x one 256-value block, tiles are
ordered ``[row_tile][k_block]`` and rows are zero-padded to a multiple of 64. Inside a
tile the first ``16 * C`` bytes of every row's (re-packed) block are stored as
``[chunk c][row r][16 B]`` (``C = 13`` for Q6_K, ``C = 9`` for Q4_K), and Q6_K appends the
rows' FP16 scales as ``[row][2 B]`` (block bytes 208..209). A decode thread of the
tensor-core kernels reads chunk ``c`` of its row ``r`` at ``(c*64 + r)*16``.

Q4_K blocks keep their GGUF bytes. Q8_0 (32-value blocks of an FP16 scale and 32 int8
codes) groups the 8 blocks of a 256-value column into one 272-byte super-block: chunk 0 is
the 8 scales (``[block][2 B]``), chunks 1..16 the 256 codes in position order; blocks past
the row's end are zero. Q5_K blocks keep their GGUF bytes (11 chunks: d, dmin and scales;
the 32 high-bit bytes; the 128 nibble bytes). Q5_1 (32-value blocks of FP16 d and m, a 32-bit
high-bit word and 16 nibble bytes) groups 8 blocks into one 192-byte super-block: chunks 0-1
the (d, m) pairs of blocks 0-3 and 4-7, chunks 2-3 their high-bit words, chunks 4..11 the
blocks' nibble bytes; blocks past the row's end are zero. Q6_K blocks re-pack the 6-bit
codes losslessly: sub-block
``j`` (values ``16j .. 16j+15``) becomes three little-endian words ``W0, W1, W2`` at bytes
``12j .. 12j+11``; byte ``i`` of ``Wn`` holds code ``4n + i`` in bits 0..5 and bits
``2n .. 2n+1`` of code ``12 + i`` in bits 6..7. Bytes 192..207 are the sub-scales.
"""

import numpy as np

TILE_ROWS = 64
# Q8_0 and Q5_1: the 8-block super-block
BLOCK_BYTES = {"Q6_K": 210, "Q4_K": 144, "Q8_0": 272, "Q5_K": 176, "Q5_1": 192}
CHUNKS = {"Q6_K": 13, "Q4_K": 9, "Q8_0": 17, "Q5_K": 11, "Q5_1": 12}
TILE_BYTES = {q: TILE_ROWS * b for q, b in BLOCK_BYTES.items()}


def padded_rows(rows):
    return (rows + TILE_ROWS - 1) // TILE_ROWS * TILE_ROWS


def tiled_bytes(qtype, rows, row_width):
    nblk = (row_width + 255) // 256
    return padded_rows(rows) // TILE_ROWS * nblk * TILE_BYTES[qtype]


def _q6_codes(raw):
    """6-bit codes ``[..., 256]`` of Q6_K blocks (position rule of packed_q6/reference.py:21-27)."""
    p = np.arange(256)
    half, quarter, lane = p // 128, (p % 128) // 32, p % 32
    lo = (raw[..., half * 64 + (quarter % 2) * 32 + lane] >> (4 * (quarter // 2))) & 15
    hi = (raw[..., 128 + half * 32 + lane] >> (2 * quarter)) & 3
    return (lo | (hi << 4)).astype(np.uint8)


def _q6_from_codes(u):
    """Inverse of :func:`_q6_codes` -> ql/qh bytes ``[..., 192]``."""
    p = np.arange(256)
    half, quarter, lane = p // 128, (p % 128) // 32, p % 32
    out = np.zeros(u.shape[:-1] + (192,), np.uint8)
    lo_idx = half * 64 + (quarter % 2) * 32 + lane
    hi_idx = 128 + half * 32 + lane
    for pos in range(256):  # small fixtures only
        out[..., lo_idx[pos]] |= ((u[..., pos] & 15) << (4 * (quarter[pos] // 2))).astype(np.uint8)
        out[..., hi_idx[pos]] |= ((u[..., pos] >> 4) << (2 * quarter[pos])).astype(np.uint8)
    return out


def repack_q6_codes(raw):
    """GGUF Q6_K bytes ``[..., 210]`` -> re-packed bytes ``[..., 210]`` (codes, sub-scales, d)."""
    raw = np.asarray(raw, np.uint8)
    u = _q6_codes(raw).reshape(raw.shape[:-1] + (16, 16))  # [..., sub-block, value]
    words = np.zeros(raw.shape[:-1] + (16, 3, 4), np.uint8)
    for n in range(3):
        words[..., n, :] = u[..., 4 * n : 4 * n + 4] | (((u[..., 12:16] >> (2 * n)) & 3) << 6)
    out = raw.copy()
    out[..., :192] = words.reshape(raw.shape[:-1] + (192,))
    return out


def unrepack_q6_codes(packed):
    """Inverse of :func:`repack_q6_codes`."""
    packed = np.asarray(packed, np.uint8)
    words = packed[..., :192].reshape(packed.shape[:-1] + (16, 3, 4))
    u = np.zeros(packed.shape[:-1] + (16, 16), np.uint8)
    for n in range(3):
        u[..., 4 * n : 4 * n + 4] = words[..., n, :] & 63
        u[..., 12:16] |= ((words[..., n, :] >> 6) & 3) << (2 * n)
    out = packed.copy()
    out[..., :192] = _q6_from_codes(u.reshape(packed.shape[:-1] + (256,)))
    return out


def _q8_super(raw):
    """Q8_0 ``uint8[rows, nblk32, 34]`` -> super-blocks ``uint8[rows, ceil(nblk32 / 8), 272]``."""
    rows, nblk32, _ = raw.shape
    nsup = (nblk32 + 7) // 8
    full = np.zeros((rows, nsup * 8, 34), np.uint8)
    full[:, :nblk32] = raw
    full = full.reshape(rows, nsup, 8, 34)
    return np.concatenate([full[..., :2].reshape(rows, nsup, 16), full[..., 2:].reshape(rows, nsup, 256)], -1)


def _q8_blocks(sup, nblk32):
    """Inverse of :func:`_q8_super`."""
    rows, nsup, _ = sup.shape
    out = np.zeros((rows, nsup, 8, 34), np.uint8)
    out[..., :2] = sup[..., :16].reshape(rows, nsup, 8, 2)
    out[..., 2:] = sup[..., 16:].reshape(rows, nsup, 8, 32)
    return out.reshape(rows, nsup * 8, 34)[:, :nblk32]


def _q51_super(raw):
    """Q5_1 ``uint8[rows, nblk32, 24]`` -> super-blocks ``uint8[rows, ceil(nblk32 / 8), 192]``."""
    rows, nblk32, _ = raw.shape
    nsup = (nblk32 + 7) // 8
    full = np.zeros((rows, nsup * 8, 24), np.uint8)
    full[:, :nblk32] = raw
    full = full.reshape(rows, nsup, 8, 24)
    return np.concatenate([full[..., :4].reshape(rows, nsup, 32), full[..., 4:8].reshape(rows, nsup, 32),
                           full[..., 8:].reshape(rows, nsup, 128)], -1)


def _q51_blocks(sup, nblk32):
    """Inverse of :func:`_q51_super`."""
    rows, nsup, _ = sup.shape
    out = np.zeros((rows, nsup, 8, 24), np.uint8)
    out[..., :4] = sup[..., :32].reshape(rows, nsup, 8, 4)
    out[..., 4:8] = sup[..., 32:64].reshape(rows, nsup, 8, 4)
    out[..., 8:] = sup[..., 64:].reshape(rows, nsup, 8, 16)
    return out.reshape(rows, nsup * 8, 24)[:, :nblk32]


def tile(raw, qtype):
    """``uint8[rows, nblk, bpb]`` (Q8_0: ``[rows, nblk32, 34]``, Q5_1: ``[rows, nblk32, 24]``)
    -> flat tiled bytes."""
    raw = np.asarray(raw, np.uint8)
    if qtype == "Q8_0":
        if raw.shape[-1] != 34:
            raise ValueError("Q8_0 blocks contain 34 bytes")
        raw = _q8_super(raw)
    elif qtype == "Q5_1":
        if raw.shape[-1] != 24:
            raise ValueError("Q5_1 blocks contain 24 bytes")
        raw = _q51_super(raw)
    rows, nblk, size = raw.shape
    if size != BLOCK_BYTES[qtype]:
        raise ValueError(f"{qtype} blocks contain {BLOCK_BYTES[qtype]} bytes")
    if qtype == "Q6_K":
        raw = repack_q6_codes(raw)
    full = np.zeros((padded_rows(rows), nblk, size), np.uint8)
    full[:rows] = raw
    t = full.reshape(-1, TILE_ROWS, nblk, size).transpose(0, 2, 1, 3)  # [G, kb, row, B]
    g = t.shape[0]
    c = CHUNKS[qtype]
    body = t[..., : 16 * c].reshape(g, nblk, TILE_ROWS, c, 16).transpose(0, 1, 3, 2, 4)
    parts = [body.reshape(g, nblk, -1)]
    if qtype == "Q6_K":
        parts.append(t[..., 208:210].reshape(g, nblk, -1))
    return np.concatenate(parts, axis=-1).reshape(-1)


def untile(tiled, qtype, rows, row_width):
    """Inverse of :func:`tile` -> ``uint8[rows, nblk, bpb]``."""
    nblk = (row_width + 255) // 256
    g = padded_rows(rows) // TILE_ROWS
    size, c = BLOCK_BYTES[qtype], CHUNKS[qtype]
    t = np.asarray(tiled, np.uint8).reshape(g, nblk, TILE_BYTES[qtype])
    out = np.zeros((g, nblk, TILE_ROWS, size), np.uint8)
    body = t[..., : 16 * c * TILE_ROWS].reshape(g, nblk, c, TILE_ROWS, 16).transpose(0, 1, 3, 2, 4)
    out[..., : 16 * c] = body.reshape(g, nblk, TILE_ROWS, 16 * c)
    if qtype == "Q6_K":
        out[..., 208:210] = t[..., 16 * c * TILE_ROWS :].reshape(g, nblk, TILE_ROWS, 2)
    raw = out.transpose(0, 2, 1, 3).reshape(-1, nblk, size)[:rows]
    if qtype == "Q8_0":
        return _q8_blocks(raw, (row_width + 31) // 32)
    if qtype == "Q5_1":
        return _q51_blocks(raw, (row_width + 31) // 32)
    return unrepack_q6_codes(raw) if qtype == "Q6_K" else raw


def soa_to_rows(data, scales, outputs, inputs):
    """The reference's SoA planes of a Q6_K projection back to GGUF rows
    ``uint8[outputs, ceil(inputs / 256), 210]``: ``packed_q6/layout.py:93-108`` (``unpack_q6``).

    Per (64-row tile, K block) the data tile holds the rows' bytes ``[0, 128)`` as
    ``[row][128]``, ``[128, 192)`` as ``[row][64]``, ``[192, 208)`` as ``[row][16]``; the
    scale plane holds bytes ``[208, 210)`` as ``[tile][block][row][2]``."""
    blocks = (inputs + 255) // 256
    tiles = (outputs + TILE_ROWS - 1) // TILE_ROWS
    d = np.asarray(data, np.uint8).reshape(tiles, blocks, TILE_ROWS * 208)
    raw = np.empty((tiles, blocks, TILE_ROWS, 210), np.uint8)
    offset = 0
    for first, last in ((0, 128), (128, 192), (192, 208)):
        width = last - first
        raw[..., first:last] = d[..., offset:offset + TILE_ROWS * width].reshape(tiles, blocks, TILE_ROWS, width)
        offset += TILE_ROWS * width
    raw[..., 208:210] = np.asarray(scales, np.uint8)[:tiles * blocks * TILE_ROWS * 2].reshape(
        tiles, blocks, TILE_ROWS, 2)
    return raw.transpose(0, 2, 1, 3).reshape(tiles * TILE_ROWS, blocks, 210)[:outputs]
