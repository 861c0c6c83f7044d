"""Full-size configurations.

* Long context: one 8192-token decision with 16 markers at random positions,
  global attention every third layer; checked directly against the oracle
  (about a minute of CPU on 8 cores).
* Throughput buckets: a 32,768-token bucket of 128-512-token decisions (the
  largest bucket of the sweep). Checked by size-independent properties: each
  sequence's results are bit-identical to its own single-sequence pass (the
  packing never mixes sequences), and a sample matches the oracle.
* Around the tcgen05 attention threshold: 2,047-2,300-token sequences in
  one batch with a short one, each bit-identical to its own single pass
  (where every block of the mma.sync grid has no work) and checked against
  the oracle.
"""
import numpy as np
import pytest

from conftest import row_rel

pytestmark = pytest.mark.gpu


def test_long_context_8192(gpu_model, oracle_model):
    """Random tokens at the 16 markers (the decision of tests/golden/
    separated.json), so its option logits are well separated and the
    argmax is asserted without a margin clause."""
    import json
    import os
    from conftest import GOLDEN
    from laya_zig_b200 import synth
    from test_gpu_forward import _compare
    seed = json.load(open(os.path.join(GOLDEN, "separated.json")))["c4"]["seed"]
    d = synth.long_decision(8192, 16, seed=seed, option_tokens=True)
    g = gpu_model.forward(d.ids, d.qtype, d.markers, want_hidden=True)
    r = oracle_model.forward(d.ids, d.markers, d.qtype, want_hidden=True)
    assert int(np.argmax(g.logits)) == int(np.argmax(r["logits"]))
    err = _compare(g, r, "L=8192")
    s = np.sort(r["logits"].astype(np.float64))
    print("long-context errors", err, "top-two margin %.3e" % (s[-1] - s[-2]))
    assert s[-1] - s[-2] >= 10 * err["logits"]


def test_full_bucket_packing_invariance(gpu_model, oracle_model):
    from laya_zig_b200 import synth
    sw = synth.sweep_decisions(400, seed=4)
    buckets = synth.bucket(sw, 32768)
    bucket = max(buckets, key=lambda b: sum(len(sw[i].ids) for i in b))  # packed to the cap
    batch = [sw[i] for i in bucket]
    assert 30000 < sum(len(d.ids) for d in batch) <= 32768
    outs = gpu_model.forward_batch(batch, want_pooled=True)
    for j in [0, len(batch) // 2, len(batch) - 1]:
        d = batch[j]
        s = gpu_model.forward(d.ids, d.qtype, d.markers)
        np.testing.assert_array_equal(s.logits, outs[j].logits)
        np.testing.assert_array_equal(s.act, outs[j].act)
        np.testing.assert_array_equal(s.pooled, outs[j].pooled)
        r = oracle_model.forward(d.ids, d.markers, d.qtype)
        assert row_rel(outs[j].pooled, r["pooled"]) <= 2e-2
        assert np.abs(outs[j].act - r["act"]).max() <= 1e-3


def test_long_batch_threshold_and_ragged_tiles(gpu_model, oracle_model):
    """Sequences around the tcgen05 kernel's threshold in one batch with a
    short one: 2,047 tokens (mma.sync), 2,048 (tcgen05, whole key tiles),
    2,049 (tcgen05, a last key tile of one key and a last query tile of one
    row), 2,300 (partial tiles). Each against the oracle, and each
    bit-identical to its own single-sequence pass: the kernel is chosen per
    sequence, never per batch."""
    from laya_zig_b200 import gpu, synth
    rng = np.random.Generator(np.random.PCG64(41))
    batch = [synth._decision(rng, L, sorted(rng.choice(np.arange(1, L - 1), 4, replace=False).tolist()), L % 3,
                             option_tokens=True)
             for L in (300, 2047, 2048, 2049, 2300)]
    outs = gpu_model.forward_batch(batch, want_pooled=True, want_hidden=True)
    for d, g in zip(batch, outs):
        s = gpu_model.forward(d.ids, d.qtype, d.markers)
        np.testing.assert_array_equal(s.logits, g.logits)
        np.testing.assert_array_equal(s.act, g.act)
        np.testing.assert_array_equal(s.pooled, g.pooled)
        r = oracle_model.forward(d.ids, d.markers, d.qtype, want_hidden=True)
        assert row_rel(g.hidden, r["hidden"]) <= 2e-2, len(d.ids)
        assert np.abs(gpu.option_probs(g.logits, 0) - gpu.option_probs(r["logits"], 0)).max() <= 1e-3
        assert np.abs(g.act - r["act"]).max() <= 1e-3
