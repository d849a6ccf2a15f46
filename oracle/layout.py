"""NumPy statement of the B200 tiled weight layout (oracle for the repack kernels).

This is the build's own lossless byte layout (the reference's analogue is the TPU
SoA repack ``kaggle/packed_q6/layout.py:49-108``, which groups 64 rows x 256 values
into separate ql/qh/scale/d regions). Here a tile is 16 rows x one 256-value block,
tiles are ordered ``[row_strip][k_block]`` and rows are zero-padded to a multiple of
16. Inside a tile, bytes are ordered so that lane ``l = 4*g + c`` of a warp reads its
MMA fragment's bytes with 16-byte loads (g = row within an 8-row half, c = column
quad). The kernel-side mapping is documented in ``csrc/tiles.cuh``.

Q6_K tile (3360 B = 16 x 210):
  [0, 2048)     ql: 4 x 512 B, sub-region u = 2*rh + part; unit (g, c) = 16 B =
                ql[row][h*64 + part*32 + lg*16 : +16] with h = c >> 1, lg = c & 1,
                row = 8*rh + g
  [2048, 3072)  qh: 2 x 512 B, sub-region rh; unit (g, c) = qh[row][16c : 16c + 16]
  [3072, 3328)  sub-scales: unit (g, c) = 8 B = [row g: sc[h*8 + lg + 2q], q=0..3,
                row g+8: the same four]
  [3328, 3360)  d: unit g = 4 B = [d(row g), d(row g+8)]

Q4_K tile (2304 B = 16 x 144):
  [0, 2048)     qs: 4 x 512 B, sub-region u = 2*rh + half; unit (g, c) = 16 B =
                qs[row][32c + 16*half : +16]
  [2048, 2304)  header: 16 x 16 B, row r -> the block's bytes [0, 16) (d, dmin, scales)
"""

import numpy as np

TILE_ROWS = 16
TILE_BYTES = {"Q6_K": 3360, "Q4_K": 2304}
BLOCK_BYTES = {"Q6_K": 210, "Q4_K": 144}


def padded_rows(rows):
    return (rows + TILE_ROWS - 1) // TILE_ROWS * TILE_ROWS


def tiled_bytes(qtype, rows, row_width):
    nblk = (row_width + 255) // 256
    return padded_rows(rows) // TILE_ROWS * nblk * TILE_BYTES[qtype]


def _pad(raw, qtype):
    raw = np.asarray(raw, np.uint8)
    rows, nblk, size = raw.shape
    if size != BLOCK_BYTES[qtype]:
        raise ValueError(f"{qtype} blocks contain {BLOCK_BYTES[qtype]} bytes")
    full = np.zeros((padded_rows(rows), nblk, size), np.uint8)
    full[:rows] = raw
    # [strip, rh, g, kblk, bytes]
    return full.reshape(-1, 2, 8, nblk, size).transpose(0, 3, 1, 2, 4)  # [strip, kblk, rh, g, B]


def tile(raw, qtype):
    """``uint8[rows, nblk, bpb]`` -> flat tiled bytes."""
    t = _pad(raw, qtype)
    strips, nblk = t.shape[:2]
    out = np.zeros((strips, nblk, TILE_BYTES[qtype]), np.uint8)
    c = np.arange(4)
    if qtype == "Q6_K":
        h, lg = c >> 1, c & 1
        ql = t[..., 0:128]
        for rh in range(2):
            for part in range(2):
                u = 2 * rh + part
                starts = h * 64 + part * 32 + lg * 16  # [4]
                idx = starts[:, None] + np.arange(16)[None, :]  # [c, 16]
                units = ql[:, :, rh][..., idx]  # [strip, kblk, g, c, 16]
                out[:, :, u * 512 : (u + 1) * 512] = units.reshape(strips, nblk, 512)
            qh = t[:, :, rh, :, 128:192]  # [strip, kblk, g, 64] == (g, c, 16) order
            out[:, :, 2048 + rh * 512 : 2048 + (rh + 1) * 512] = qh.reshape(strips, nblk, 512)
        sc = t[..., 192:208]  # [strip, kblk, rh, g, 16]
        sel = (h * 8 + lg)[:, None] + 2 * np.arange(4)[None, :]  # [c, q]
        lo = sc[:, :, 0][..., sel]  # [strip, kblk, g, c, 4]
        hi = sc[:, :, 1][..., sel]
        units = np.concatenate((lo, hi), axis=-1)  # [strip, kblk, g, c, 8]
        out[:, :, 3072:3328] = units.reshape(strips, nblk, 256)
        d = np.stack((t[:, :, 0, :, 208:210], t[:, :, 1, :, 208:210]), axis=3)  # [s,k,g,2,2]
        out[:, :, 3328:3360] = d.reshape(strips, nblk, 32)
    elif qtype == "Q4_K":
        qs = t[..., 16:144]
        for rh in range(2):
            for half in range(2):
                u = 2 * rh + half
                idx = (32 * c + 16 * half)[:, None] + np.arange(16)[None, :]
                units = qs[:, :, rh][..., idx]
                out[:, :, u * 512 : (u + 1) * 512] = units.reshape(strips, nblk, 512)
        head = t[..., 0:16]  # [strip, kblk, rh, g, 16] -> row order rh*8+g
        out[:, :, 2048:2304] = head.reshape(strips, nblk, 256)
    else:
        raise ValueError(f"no tiled layout for {qtype}")
    return out.reshape(-1)


def untile(tiled, qtype, rows, row_width):
    """Inverse of :func:`tile` -> ``uint8[rows, nblk, bpb]``."""
    nblk = (row_width + 255) // 256
    strips = padded_rows(rows) // TILE_ROWS
    size = BLOCK_BYTES[qtype]
    t = np.asarray(tiled, np.uint8).reshape(strips, nblk, TILE_BYTES[qtype])
    full = np.zeros((strips, nblk, 2, 8, size), np.uint8)
    c = np.arange(4)
    if qtype == "Q6_K":
        h, lg = c >> 1, c & 1
        for rh in range(2):
            for part in range(2):
                u = 2 * rh + part
                units = t[:, :, u * 512 : (u + 1) * 512].reshape(strips, nblk, 8, 4, 16)
                for ci in range(4):
                    start = h[ci] * 64 + part * 32 + lg[ci] * 16
                    full[:, :, rh, :, start : start + 16] = units[:, :, :, ci]
            full[:, :, rh, :, 128:192] = t[:, :, 2048 + rh * 512 : 2048 + (rh + 1) * 512].reshape(
                strips, nblk, 8, 64
            )
        units = t[:, :, 3072:3328].reshape(strips, nblk, 8, 4, 8)
        for ci in range(4):
            for q in range(4):
                j = h[ci] * 8 + lg[ci] + 2 * q
                full[:, :, 0, :, 192 + j] = units[:, :, :, ci, q]
                full[:, :, 1, :, 192 + j] = units[:, :, :, ci, 4 + q]
        d = t[:, :, 3328:3360].reshape(strips, nblk, 8, 2, 2)
        full[:, :, 0, :, 208:210] = d[:, :, :, 0]
        full[:, :, 1, :, 208:210] = d[:, :, :, 1]
    elif qtype == "Q4_K":
        for rh in range(2):
            for half in range(2):
                u = 2 * rh + half
                units = t[:, :, u * 512 : (u + 1) * 512].reshape(strips, nblk, 8, 4, 16)
                for ci in range(4):
                    start = 16 + 32 * ci + 16 * half
                    full[:, :, rh, :, start : start + 16] = units[:, :, :, ci]
        full[:, :, :, :, 0:16] = t[:, :, 2048:2304].reshape(strips, nblk, 2, 8, 16)
    else:
        raise ValueError(f"no tiled layout for {qtype}")
    raw = full.transpose(0, 2, 3, 1, 4).reshape(strips * 16, nblk, size)
    return raw[:rows]
