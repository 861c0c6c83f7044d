"""RoPE as the QKV projection's epilogue applies it (csrc/gemm.cu, EPI_QKV),
restated on the CPU: the embedding kernel (csrc/norm.cu) copies each
token's 32 (cos, sin) pairs from the position-indexed table into
frequency-major rows, rope_tok[i][t] = (cos f, sin f, cos f+1, sin f+1) for
f = 2i; the epilogue rotates a head in two passes of 16 frequencies, column
16*hq + d with column 32 + 16*hq + d by rope_tok[8*hq + d/2]. The result
must be the reference's rotate_half rotation (ropeApply, src/main.zig:
2512-2519): x'[d] = x[d] cos_d - x[d+32] sin_d, x'[d+32] = x[d+32] cos_d +
x[d] sin_d for d < 32, with the table's values."""
import numpy as np

D_HEAD, HALF = 64, 32


def table(max_pos, theta=160000.0):
    inv = (1.0 / np.power(np.float32(theta), np.arange(32, dtype=np.float32) / np.float32(32))).astype(np.float32)
    f = (inv[None, :] * np.arange(max_pos, dtype=np.float32)[:, None]).astype(np.float32)
    return np.stack([np.cos(f), np.sin(f)], axis=-1).astype(np.float32)  # [pos][32][2]


def rope_tok_rows(tab, positions):
    """[16][T][4]: what the embedding kernel writes (lane i copies float4 i of
    the token's 256-byte table row)."""
    flat = tab[positions].reshape(len(positions), 16, 4)  # float2 pairs (2i, 2i+1) as one float4
    return np.ascontiguousarray(flat.transpose(1, 0, 2))


def epilogue_rotate(head, cs):
    """head: [64] one token's q or k head; cs: [16][4] its rope_tok rows."""
    out = head.copy()
    for hq in range(2):
        x0 = head[16 * hq:16 * hq + 16].copy()
        x1 = head[HALF + 16 * hq:HALF + 16 * hq + 16].copy()
        for d in range(0, 16, 2):
            c0, s0, c1, s1 = cs[8 * hq + d // 2]
            a0, b0, a1, b1 = x0[d], x1[d], x0[d + 1], x1[d + 1]
            x0[d], x1[d] = a0 * c0 - b0 * s0, b0 * c0 + a0 * s0
            x0[d + 1], x1[d + 1] = a1 * c1 - b1 * s1, b1 * c1 + a1 * s1
        out[16 * hq:16 * hq + 16] = x0
        out[HALF + 16 * hq:HALF + 16 * hq + 16] = x1
    return out


def reference_rotate(head, tab_row):
    c, s = tab_row[:, 0], tab_row[:, 1]
    x, y = head[:HALF], head[HALF:]
    return np.concatenate([x * c - y * s, y * c + x * s]).astype(np.float32)


def test_epilogue_rotation_matches_rotate_half():
    rng = np.random.Generator(np.random.PCG64(5))
    tab = table(4096)
    # packed sequences: positions restart at 0 in every sequence
    lens = [1, 63, 64, 65, 180, 1000, 2047]
    positions = np.concatenate([np.arange(L) for L in lens])
    rows = rope_tok_rows(tab, positions)
    for t in rng.choice(len(positions), size=400, replace=False):
        head = rng.standard_normal(D_HEAD).astype(np.float32)
        got = epilogue_rotate(head, rows[:, t, :])
        ref = reference_rotate(head, tab[positions[t]])
        np.testing.assert_array_equal(got, ref)


def test_rope_tok_rows_are_the_table_rows():
    tab = table(512)
    positions = np.array([0, 1, 2, 511, 7, 0, 300])
    rows = rope_tok_rows(tab, positions)
    assert rows.shape == (16, len(positions), 4)
    for t, p in enumerate(positions):
        for i in range(16):
            np.testing.assert_array_equal(rows[i, t], [tab[p, 2 * i, 0], tab[p, 2 * i, 1],
                                                       tab[p, 2 * i + 1, 0], tab[p, 2 * i + 1, 1]])
