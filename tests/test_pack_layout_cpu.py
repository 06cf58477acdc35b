"""The tile-packed q4_0 layout (tests/pack_layout.py, the restatement the GPU
test checks e4b_q40_pack_tiles against byte for byte) carries every weight of
the GGUF rows exactly once, where the MMA lanes read it: each piece's scales
are the blocks' f16 scales, and each lane word's nibbles are the elements of
the fragment-order set batch.xfo_perm assigns to that lane (low nibble element
j, high nibble element j + 16)."""
import numpy as np
import pytest

from pack_layout import PIECE, lane_bytes, pack_q40


def _lane_elements(block: int, t: int) -> list:
    """Element indices j (< 16) lane t covers in a block, in fragment order's
    definition (batch.xfo_perm): odd blocks 4t..4t+3; even blocks 2+4t..5+4t,
    or {0, 1, 14, 15} for t = 3."""
    if block & 1:
        return [4 * t + k for k in range(4)]
    if t < 3:
        return [2 + 4 * t + k for k in range(4)]
    return [0, 1, 14, 15]


@pytest.mark.parametrize("rows,n_in", [(16, 256), (48, 512), (32, 2816)])
def test_packed_pieces_hold_every_weight_where_lanes_read_it(rows, n_in):
    rng = np.random.default_rng(rows + n_in)
    nb = n_in // 32
    w = rng.integers(0, 256, rows * nb * 18, dtype=np.uint8)
    packed = pack_q40(w, rows, n_in)
    assert packed.size == w.size
    src = w.reshape(rows, nb, 18)
    pieces = packed.reshape(rows // 16, n_in // 256, PIECE)
    seen = np.zeros((rows, nb, 32), np.int32)
    for r16 in range(rows // 16):
        for q in range(n_in // 256):
            piece = pieces[r16, q]
            for r in range(16):
                row = 16 * r16 + r
                for k in range(8):
                    b = 8 * q + k
                    assert bytes(piece[16 * r + 2 * k:16 * r + 2 * k + 2]) == bytes(src[row, b, :2])
                for kh in range(2):
                    for t in range(4):
                        for j in range(4):
                            b = 8 * q + 4 * kh + j
                            o = 256 + ((kh * 16 + r) * 4 + t) * 16 + 4 * j
                            word = piece[o:o + 4]
                            for byte, e in zip(word, _lane_elements(b, t)):
                                # GGUF q4_0: byte 2 + e holds element e (low) and e + 16 (high)
                                assert byte == src[row, b, 2 + e]
                                seen[row, b, e] += 1
                                seen[row, b, e + 16] += 1
    assert np.all(seen == 1)


def test_lane_byte_sets_partition_each_block():
    """The four lanes of a block read its 16 nibble bytes once each."""
    for block in (0, 1):
        got = sorted(o for t in range(4) for o in lane_bytes(block, t))
        assert got == list(range(2, 18))


def test_lane_sets_match_fragment_order(e4b):
    """_lane_elements is the lane assignment batch.xfo_perm stores the
    activations in: element j (and j + 16) of block b sits in lane t's 8 halves."""
    n = 256
    pos = e4b.batch.xfo_perm(n)
    for i in range(n):
        b, j = divmod(i, 32)
        t = (int(pos[i]) - 32 * b) // 8
        assert j % 16 in _lane_elements(b, t), (i, b, j, t)
