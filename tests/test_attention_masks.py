"""The attention kernel's index arithmetic (csrc/attention.cu), restated and
checked exhaustively on the CPU against the reference's key window
(attWorker, src/main.zig:2440-2444: row i sees keys [max(0, i - 64),
min(L, i + 65)) on sliding layers, all L keys on global ones).

Restated from the kernel: a CTA takes 64 query rows starting at q0 and
visits key tiles [kt0, kt1) of 64 keys; a tile is masked only when it
crosses the sequence end or a window edge, and then a score (row qi, key
kj) survives iff kj - lo, taken as unsigned, is at most hi - lo, where
[lo, hi] is the row's visible range (an empty range masks the row). For
every length and row the keys that survive must be exactly the reference's,
each once."""
import numpy as np
import pytest

QB = KB = 64
U32 = np.uint64(0xFFFFFFFF)


def kernel_visible(L, w, q0):
    """bool[64 rows][L keys]: the scores the kernel keeps for rows q0..q0+63."""
    klo, khi = (max(0, q0 - w), min(L, q0 + QB - 1 + w + 1)) if w >= 0 else (0, L)
    kt0, kt1 = klo // KB, (khi + KB - 1) // KB
    rows = q0 + np.arange(QB)
    keep = np.zeros((QB, L), dtype=np.int32)
    for kt in range(kt0, kt1):
        tlo, thi = kt * KB, kt * KB + KB - 1
        need_mask = thi >= L or (w >= 0 and (q0 + QB - 1 - tlo > w or thi - q0 > w))
        keys = np.arange(tlo, tlo + KB)
        if not need_mask:
            ok = np.ones((QB, KB), dtype=bool)
        else:
            if w >= 0:
                lo = np.maximum(0, rows - w)
                hi = np.minimum(L - 1, rows + w)
            else:
                lo = np.zeros(QB, dtype=np.int64)
                hi = np.full(QB, L - 1, dtype=np.int64)
            empty = hi < lo
            r = np.where(empty, 0, hi - lo).astype(np.uint64)
            d = (keys[None, :] - lo[:, None]).astype(np.int64).astype(np.uint64) & U32
            ok = ~empty[:, None] & (d <= r[:, None])
        in_seq = keys < L
        keep[:, keys[in_seq]] += ok[:, in_seq]
        # a key past the sequence end (another sequence's row, or zero fill) is never kept
        assert not ok[:, ~in_seq][rows < L].any(), (L, w, q0, kt)
    return keep


def reference_visible(L, w, q0):
    rows = q0 + np.arange(QB)[:, None]
    keys = np.arange(L)[None, :]
    if w < 0:
        return np.ones((QB, L), dtype=bool) & (rows < L)
    return (keys >= np.maximum(0, rows - w)) & (keys < np.minimum(L, rows + w + 1)) & (rows < L)


LENGTHS = list(range(1, 260)) + [319, 320, 321, 383, 384, 385, 511, 512, 513, 700, 1023, 1024, 1025]


@pytest.mark.parametrize("w", [64, -1, 0, 1, 63, 65, 200])
def test_kept_scores_equal_reference_window(w):
    for L in LENGTHS:
        for q0 in range(0, L, QB):
            got = kernel_visible(L, w, q0)
            ref = reference_visible(L, w, q0)
            valid = (q0 + np.arange(QB)) < L  # rows past the end are computed but never stored
            assert (got[valid] <= 1).all(), (L, w, q0, "a key visited twice")
            np.testing.assert_array_equal(got[valid].astype(bool), ref[valid], err_msg="L=%d w=%d q0=%d" % (L, w, q0))


def test_tiles_per_block_at_the_bench_length():
    """At 180 tokens a sliding layer visits 7 key tiles per (sequence, head)
    and a global one 9: the tile counts the kernel's timing model uses."""
    def tiles(L, w):
        n = 0
        for q0 in range(0, L, QB):
            klo, khi = (max(0, q0 - w), min(L, q0 + QB - 1 + w + 1)) if w >= 0 else (0, L)
            n += (khi + KB - 1) // KB - klo // KB
        return n
    assert tiles(180, 64) == 7 and tiles(180, -1) == 9
