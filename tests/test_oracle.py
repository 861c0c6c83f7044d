"""The CPU oracle, pinned against the reference's own checks.

* Golden fixtures: tests/golden/*.json hold the output of the reference's
  tools/refcheck.py (an independent f64 recompute of the whole network) on
  the seeded synthetic checkpoint; see tests/golden/make_golden.py.
* --selftest known-answer checks (src/main.zig:420-536): the packed GEMM
  against f64 on the model's shapes (relative error < 1e-4), expv against
  f64 exp (< 1e-6) and geluv against the scalar gelu (< 1e-5).
"""
import numpy as np
import pytest

from conftest import golden_cases, row_rel

CASES = golden_cases()


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_refcheck(name, oracle_model):
    g = CASES[name]
    r = oracle_model.forward(np.array(g["ids"]), np.array(g["markers"]), g["qtype"], want_stats=True,
                             want_hidden=True)
    # refcheck.py's own acceptance (refcheck.py:281-294) ...
    for tag, ref in g["tags"].items():
        got = r["stats"][tag]
        dmax = max(abs(got[i] - ref[i]) for i in range(3))
        serr = abs(got[3] - ref[3]) / max(1.0, abs(ref[3]))
        aerr = abs(got[4] - ref[4]) / max(1.0, abs(ref[4]))
        assert dmax < 5e-3 and serr < 1e-3 and aerr < 1e-3, (tag, dmax, serr, aerr)
        # ... and the agreement the reference reports for itself (~1e-5, README.md:129, 356)
        assert dmax < 1e-4 and serr < 1e-4 and aerr < 1e-5, (tag, dmax, serr, aerr)
    np.testing.assert_allclose(r["logits"], g["logits"], atol=1e-5)
    np.testing.assert_allclose(r["act"], g["act"], atol=1e-5)
    if g["logits"]:
        p = np.exp(r["logits"] - r["logits"].max())
        p /= p.sum()
        np.testing.assert_allclose(p, g["probs"], atol=1e-6)
    for k, row in g["hidden_rows"].items():
        assert row_rel(r["hidden"][int(k)], np.array(row)) < 1e-5


def test_oracle_full_hidden_matches_refcheck(oracle_model):
    import os
    from conftest import GOLDEN
    g = CASES["c1_L64"]
    ref = np.load(os.path.join(GOLDEN, "c1_L64_hidden.npy"))
    r = oracle_model.forward(np.array(g["ids"]), np.array(g["markers"]), g["qtype"], want_hidden=True)
    assert row_rel(r["hidden"], ref) < 1e-5


def _splitmix_uniform(seed, n):
    # U(-1, 1) from a counter-based hash (the reference seeds 0x5eed, main.zig:429)
    from laya_zig_b200.synth import _splitmix64, _GOLD
    with np.errstate(over="ignore"):
        h = _splitmix64((np.uint64(seed) + np.arange(n, dtype=np.uint64)) * _GOLD)
    return ((h >> np.uint64(40)).astype(np.float64) / float(1 << 24) * 2.0 - 1.0).astype(np.float32)


@pytest.mark.parametrize("rows,n,k", [(1, 768, 768), (63, 2304, 768), (63, 768, 1152), (63, 3072, 768),
                                      (63, 768, 768), (64, 768, 1152), (1, 768, 3072)])
def test_oracle_gemm_selftest(rows, n, k):
    from laya_zig_b200.synth import f32_to_bf16_bits, bf16_bits_to_f32
    from oracle import oracle
    x = _splitmix_uniform(0x5eed, rows * k).reshape(rows, k)
    wb = f32_to_bf16_bits(_splitmix_uniform(0x5eed + 1, n * k)).reshape(n, k)
    out = oracle.linear16(x, wb)
    ref = x.astype(np.float64) @ bf16_bits_to_f32(wb).astype(np.float64).T
    cols = np.arange(0, n, 29)  # every 29th column, as the reference checks
    rel = np.abs(out[:, cols] - ref[:, cols]) / np.maximum(1.0, np.abs(ref[:, cols]))
    assert rel.max() < 1e-4


def test_oracle_expv_geluv_selftest():
    from oracle import oracle
    base = np.arange(-8000, 8001, dtype=np.float32) * np.float32(0.001)
    lanes = (base[:, None] + np.arange(8, dtype=np.float32)[None, :] * np.float32(0.00017)).astype(np.float32)
    x = lanes.ravel()
    e = oracle.expv(x).astype(np.float64)
    we = np.exp(x.astype(np.float64))
    assert (np.abs(e - we) / we).max() < 1e-6
    gv = oracle.geluv(x).astype(np.float64)
    gs = oracle.gelu(x).astype(np.float64)
    assert (np.abs(gv - gs) / np.maximum(0.05, np.abs(gs))).max() < 1e-5


def test_oracle_rejects_bad_input(oracle_model):
    with pytest.raises(ValueError):
        oracle_model.forward(np.array([2, 256000, 1]), np.array([1]), 0)
    with pytest.raises(ValueError):
        oracle_model.forward(np.array([2, 5, 1]), np.array([3]), 0)
    with pytest.raises(ValueError):
        oracle_model.forward(np.array([2, 5, 1]), np.array([1]), 3)


def test_oracle_missing_tensor(weights):
    from oracle import oracle
    w = dict(weights)
    del w["encoder.layers.5.mlp.Wi.weight"]
    with pytest.raises(ValueError, match="missing tensor: encoder.layers.5.mlp.Wi.weight"):
        oracle.model_from_bf16(w)
