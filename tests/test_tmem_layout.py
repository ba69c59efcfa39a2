"""CPU check of the batch-1 kernel's tensor-memory tile layout.

decode_program.cu's mover copies each landed GEMV tile (8 weight rows x 2048
fp16 columns, row-major in its shared-memory stage) into a 64-column TMEM slot
with 8 tcgen05.cp.128x256b: copy (half h, piece c) reads the stage from byte
h * 16384 + c * 256 through a K-major no-swizzle descriptor (8-row groups 1024
bytes apart, K-adjacent 16-byte core-matrix rows 128 bytes apart) into slot
columns h * 32 + c * 8 .. + 8.  Each consumer warp then reads 32 columns of its
TMEM lane quarter and assumes that lane l holds, for v = 0..7, columns
512 (l / 8) + 64 v + 8 (l % 8) + [0, 8) of one tile row.  This test replays
the copies' addressing in numpy and checks that assumption for every warp.
"""
import numpy as np


def _cp_source_bytes(base: int, lane: int) -> np.ndarray:
    """Byte offsets in the stage of the 16 fp16 values tcgen05.cp.128x256b
    puts in TMEM lane `lane` (row `lane` of the described 128 x 16 matrix)."""
    e = np.arange(16)
    return base + (lane // 8) * 1024 + (e // 8) * 128 + (lane % 8) * 16 + (e % 8) * 2


def test_tmem_slot_holds_the_columns_each_consumer_lane_assumes():
    rows, cols = 8, 2048
    tile = np.arange(rows * cols, dtype=np.int64).reshape(rows, cols)  # value = its own index
    flat = tile.reshape(-1)
    slot = np.zeros((128, 64 * 2), dtype=np.int64)  # [lane][fp16 half of 64 32-bit columns]
    for h in range(2):
        for c in range(4):
            base = h * 16384 + c * 256
            col0 = h * 32 + c * 8  # 32-bit column; each holds two fp16 values
            for lane in range(128):
                slot[lane, 2 * col0:2 * col0 + 16] = flat[_cp_source_bytes(base, lane) // 2]
    for w in range(8):  # consumer warp w: lane quarter (w + 1) % 4, column half w / 4
        q, h = (w + 1) & 3, w >> 2
        rwt = q + 4 * h
        for l in range(32):
            got = slot[32 * q + l, 64 * h:64 * h + 64]  # tcgen05.ld 32x32b.x32 of its 32 columns
            want = np.concatenate([tile[rwt, 512 * (l >> 3) + 64 * v + 8 * (l & 7) + np.arange(8)]
                                   for v in range(8)])
            np.testing.assert_array_equal(got, want, err_msg=f"warp {w} lane {l}")
    # every element of the tile is in the slot exactly once
    assert np.array_equal(np.sort(slot.reshape(-1)), np.arange(rows * cols))
