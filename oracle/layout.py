"""NumPy statement of the B200 tiled weight layout (oracle for the repack kernels).

This is the build's own lossless byte layout (the reference's analogue is the TPU SoA
repack ``kaggle/packed_q6/layout.py:49-108``, which groups 64 rows x 256 values into
separate ql/qh/scale/d regions). Here a tile is 128 rows x one 256-value block, tiles are
ordered ``[row_tile][k_block]`` and rows are zero-padded to a multiple of 128. Inside a
tile the first ``16 * C`` bytes of every row's block are stored as ``[chunk c][row r][16 B]``
(``C = 13`` for Q6_K: block bytes 0..207; ``C = 9`` for Q4_K: the whole 144-byte block), and
Q6_K appends the rows' FP16 scales as ``[row][2 B]`` (block bytes 208..209). Thread ``r`` of
the tensor-core kernels' decode warps reads chunk ``c`` of its row at ``(c*128 + r)*16``.
"""

import numpy as np

TILE_ROWS = 128
BLOCK_BYTES = {"Q6_K": 210, "Q4_K": 144}
CHUNKS = {"Q6_K": 13, "Q4_K": 9}
TILE_BYTES = {q: TILE_ROWS * b for q, b in BLOCK_BYTES.items()}


def padded_rows(rows):
    return (rows + TILE_ROWS - 1) // TILE_ROWS * TILE_ROWS


def tiled_bytes(qtype, rows, row_width):
    nblk = (row_width + 255) // 256
    return padded_rows(rows) // TILE_ROWS * nblk * TILE_BYTES[qtype]


def tile(raw, qtype):
    """``uint8[rows, nblk, bpb]`` -> flat tiled bytes."""
    raw = np.asarray(raw, np.uint8)
    rows, nblk, size = raw.shape
    if size != BLOCK_BYTES[qtype]:
        raise ValueError(f"{qtype} blocks contain {BLOCK_BYTES[qtype]} bytes")
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
    return out.transpose(0, 2, 1, 3).reshape(-1, nblk, size)[:rows]
