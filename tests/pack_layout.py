"""numpy restatement of the tile-packed q4_0 layout (e4b_q40_pack_tiles,
include/e4b_b200.h) and of the lane mapping it serves, shared by the CPU
layout test and the GPU byte-for-byte test.

Piece (r16, q) of a rows x IN matrix (rows % 16 == 0, IN % 256 == 0) sits at
(r16 * IN/256 + q) * 2304: the 16 rows' 8 f16 block scales as [row][block]
(256 bytes), then [block half h][row r][lane t] uint4s whose word j is the
32-bit word lane t of the MMA fragment reads from block 4h + j of row r.
"""
import numpy as np

PIECE = 2304


def lane_bytes(block: int, t: int) -> list:
    """Offsets inside an 18-byte GGUF q4_0 block of the 4 nibble bytes lane t
    reads: odd blocks bytes 2 + 4t .. 5 + 4t; even blocks 4 + 4t .. 7 + 4t for
    t < 3 and {2, 3, 16, 17} for t = 3 (the fragment-order element sets of
    batch.xfo_perm: j = 4t..4t+3, 2+4t..5+4t or {0, 1, 14, 15}, and j + 16)."""
    if block & 1:
        return [2 + 4 * t + k for k in range(4)]
    if t < 3:
        return [4 + 4 * t + k for k in range(4)]
    return [2, 3, 16, 17]


def pack_q40(w: np.ndarray, rows: int, n_in: int) -> np.ndarray:
    """The packed copy of rows x n_in GGUF q4_0 bytes (uint8, same size)."""
    nq, rb = n_in // 256, n_in // 32 * 18
    src = np.asarray(w, np.uint8).reshape(rows, rb)
    out = np.zeros((rows // 16, nq, PIECE), np.uint8)
    for r16 in range(rows // 16):
        for q in range(nq):
            piece = out[r16, q]
            for r in range(16):
                row = src[16 * r16 + r]
                for k in range(8):
                    b = 8 * q + k
                    piece[16 * r + 2 * k:16 * r + 2 * k + 2] = row[18 * b:18 * b + 2]
                for kh in range(2):
                    for t in range(4):
                        for j in range(4):
                            b = 8 * q + 4 * kh + j
                            blk = row[18 * b:18 * b + 18]
                            o = 256 + ((kh * 16 + r) * 4 + t) * 16 + 4 * j
                            piece[o:o + 4] = blk[lane_bytes(b, t)]
    return out.reshape(-1)
