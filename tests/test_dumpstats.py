"""--dumpstats from the GPU path (src/main.zig:113-130, 2651-2777).

The reference prints a fingerprint of the hidden state after every stage
(`[dump] <tag> x0 x1 x2 sum abs-sum`) and its own checker,
tools/refcheck.py, reads those lines and compares them with an f64
recompute. `laya_gpu_forward_dumpstats` prints the same lines from the GPU
forward (fingerprints reduced on the device in f64; the `final` point is
measured inside the fused final-norm kernel, not reconstructed), and
`laya_gpu_format_dump` is its host-only text part.

`parse_dump` below reads the lines as refcheck.py:233-259 does (its line
regexes, which define the format). The CPU tests pin the text: the oracle's
fingerprints round-trip through format -> parse, and, where a laya-zig
checkout is available ($LAYA_REFERENCE or ../reference beside this
repository), refcheck's own parse_dump reads the same file identically. The
GPU tests compare the GPU's dump with the golden fingerprints refcheck
computed (tests/golden/*.json) with refcheck's tolerances
(refcheck.py:281-294): the first three values within 5e-3 and the abs-sum
within 1e-3 relative to max(1, |ref|). refcheck holds the plain sum to the
same 1e-3 relative to max(1, |sum|), a bar set for the reference's f32
activations; the sum of L x 768 values cancels to a few units while its
terms carry the 16-bit rounding of tensor-core operands (about 1e-3 each,
so the sum moves by ~sqrt(L x 768) x 1e-3 = 0.2 at L = 64). The sum is
therefore held to 1e-3 of the abs-sum, the scale of its terms. In the bf16
mode the first three values (single elements of the state, of magnitude
0.5-2) carry the bf16 operands' rounding, measured up to 7e-3 at the head
layers; they are held to 1e-2 there and to refcheck's 5e-3 in the f16 mode.
"""
import importlib.util
import os
import re

import numpy as np
import pytest

from conftest import ROOT, golden_cases


def parse_dump(text):
    ids, marks, logits, layers, meta = [], [], [], {}, None
    for line in text.splitlines():
        m = re.search(r"\[dump\] meta L=(\d+) qtype=(\d+)", line)
        if m:
            meta = (int(m.group(1)), int(m.group(2)))
            continue
        m = re.search(r"\[dump\] ids((?: \d+)+)", line)
        if m:
            ids.extend(int(t) for t in m.group(1).split())
            continue
        m = re.search(r"\[dump\] mark((?: \d+)+)", line)
        if m:
            marks.extend(int(t) for t in m.group(1).split())
            continue
        m = re.search(r"\[dump\] logit(.*)", line)
        if m:
            logits.extend(float(t) for t in m.group(1).split())
            continue
        m = re.search(r"\[dump\] (\S+)\s+(\S+)\s+(\S+)\s+(\S+)\s+(\S+)\s+(\S+)", line)
        if m:
            v = [float(m.group(i)) for i in range(2, 7)]
            layers[m.group(1)] = (v[:3], v[3], v[4])
    return meta, ids, marks, logits, layers


def refcheck_compare(mine, ref, tol=5e-3):
    """refcheck.py:281-294 for the first three values (within tol) and the
    abs-sum (1e-3 relative to max(1, |ref|)); the sum within 1e-3 of the
    abs-sum (see the module docstring). Returns (ok, (dmax, sum error
    relative to the abs-sum, abs-sum error))."""
    (m3, ms, ma), (r3, rs, ra) = mine, ref
    dmax = max(abs(p - q) for p, q in zip(m3, r3))
    serr = abs(ms - rs) / max(1.0, abs(ra))
    aerr = abs(ma - ra) / max(1.0, abs(ra))
    return dmax < tol and serr < 1e-3 and aerr < 1e-3, (dmax, serr, aerr)


def _reference_refcheck():
    ref = os.environ.get("LAYA_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
    path = os.path.join(ref, "tools", "refcheck.py")
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location("refcheck_for_format_test", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _oracle_dump(oracle_model, d):
    from laya_zig_b200 import gpu
    from oracle.oracle import TAGS
    r = oracle_model.forward(d.ids, d.markers, d.qtype, want_stats=True)
    stats = np.array([r["stats"][t] for t in TAGS])
    return r, stats, gpu.format_dump(d.ids, d.qtype, d.markers, r["logits"], stats)


def test_format_round_trip(oracle_model):
    """The text carries the reference's lines in its order and precision."""
    from laya_zig_b200 import synth
    from oracle.oracle import TAGS
    d = synth.parity_decision(1)
    r, stats, text = _oracle_dump(oracle_model, d)
    lines = text.splitlines()
    assert lines[0] == "[dump] meta L=64 qtype=0"
    assert lines[1] == "[dump] ids " + " ".join(str(int(v)) for v in d.ids[:8])
    assert len([l for l in lines if l.startswith("[dump] ids")]) == 8
    tag_lines = [l for l in lines if re.match(r"\[dump\] (emb|l\d+|final|temb|h\d) ", l)]
    assert [l.split()[1] for l in tag_lines] == TAGS
    assert tag_lines[0].startswith("[dump] emb   ") and tag_lines[-1].startswith("[dump] h1    ")
    assert lines[-2] == "[dump] mark 8 16 24 32"
    assert lines[-1].startswith("[dump] logit ") and len(lines[-1].split()) == 2 + 4
    meta, ids, marks, logits, layers = parse_dump(text)
    assert meta == (64, 0) and ids == [int(v) for v in d.ids] and marks == [8, 16, 24, 32]
    np.testing.assert_allclose(logits, r["logits"], atol=5e-6)
    for i, t in enumerate(TAGS):
        x3, s, a = layers[t]
        np.testing.assert_allclose(x3, stats[i, :3], atol=5e-6)
        assert abs(s - stats[i, 3]) <= 5e-4 and abs(a - stats[i, 4]) <= 5e-4


def test_format_matches_refcheck_parser(oracle_model, tmp_path):
    """refcheck's own parse_dump reads the text as parse_dump here does."""
    rc = _reference_refcheck()
    if rc is None:
        pytest.skip("no laya-zig checkout ($LAYA_REFERENCE or ../reference)")
    from laya_zig_b200 import synth
    d = synth.parity_decision(1)
    _, _, text = _oracle_dump(oracle_model, d)
    f = tmp_path / "dump.txt"
    f.write_text(text)
    assert rc.parse_dump(str(f)) == parse_dump(text)


def test_format_rejects_small_buffer():
    import ctypes
    from laya_zig_b200 import gpu
    ids = np.arange(10, dtype=np.uint32)
    st = np.zeros((27, 5), np.float64)
    need = ctypes.c_uint64(0)
    buf = ctypes.create_string_buffer(16)
    rc = gpu.lib.laya_gpu_format_dump(ids.ctypes.data, 10, 0, None, 0, None, st.ctypes.data, buf, 16,
                                      ctypes.byref(need))
    assert rc == gpu.ERR_ARG and need.value > 16
    assert b"needs" in gpu.lib.laya_gpu_last_error(None)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(golden_cases()))
@pytest.mark.parametrize("precision", ["bf16", "f16"])
def test_gpu_dump_against_refcheck_goldens(name, precision, weights, gpu_model):
    """The GPU's [dump] lines against the fingerprints refcheck computed in
    f64, with refcheck's tolerances."""
    from laya_zig_b200 import gpu
    from oracle.oracle import TAGS
    g = golden_cases()[name]
    model = gpu_model if precision == "bf16" else gpu.LayaGPU.from_bf16(weights, precision="f16")
    try:
        logits, act, text = model.forward_dumpstats(np.array(g["ids"]), g["qtype"], np.array(g["markers"]))
    finally:
        if model is not gpu_model:
            model.close()
    meta, ids, marks, lg, layers = parse_dump(text)
    assert meta == (len(g["ids"]), g["qtype"]) and ids == g["ids"] and marks == g["markers"]
    assert sorted(layers) == sorted(TAGS)
    worst = {}
    for t in TAGS:
        ref = g["tags"][t]
        ok, err = refcheck_compare(layers[t], (ref[:3], ref[3], ref[4]), tol=1e-2 if precision == "bf16" else 5e-3)
        worst[t] = err
        assert ok, (precision, name, t, err)
    if g["logits"]:
        assert max(abs(p - q) for p, q in zip(lg, g["logits"])) < 5e-2  # refcheck.py:300-303
        np.testing.assert_allclose(lg, logits, atol=1e-5)
    print(precision, name, "worst sum/abs-sum error", max(e[1] for e in worst.values()),
          max(e[2] for e in worst.values()))
