#!/usr/bin/env python
"""Generate the golden forward-pass fixtures from the reference's own checker.

The reference ships an independent, stdlib-only recompute of the whole
network, `tools/refcheck.py` (f64 Python floats, `math.erf`/`math.exp`). This
script imports it from the reference checkout, writes the seeded synthetic
weights of `laya_zig_b200.synth` as an F16 `model.safetensors` (the only
dtype the reference's matrix loader accepts, src/main.zig:1352), and runs
refcheck's own functions on a few decisions:

    embeddings + norm -> encoder_layer x22 -> final norm -> type embedding
    -> head_layer x2 -> scorer per marker                     (refcheck.py:265-322)

The act/escalate head is not part of refcheck.py; it is restated below from
src/main.zig:2787-2814 with refcheck's own helpers (`softmax`, `gelu`,
`matvec`) in the same f64 arithmetic.

For every case it stores, as JSON, the reference's `[dump]` fingerprints per
tag (first three values, sum, abs-sum; src/main.zig:113-121), the logits,
the untempered option probabilities, the act pair, and the final hidden rows
at [CLS], the markers and the last token; the complete final hidden state of
the parity case is stored as float32 .npy.

Usage (needs a laya-zig checkout; takes several minutes of CPython):
    python tests/golden/make_golden.py --reference <path to the laya-zig checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import multiprocessing as mp
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from laya_zig_b200 import safetensors, synth  # noqa: E402

WEIGHT_SEED = 0


def cases():
    """name -> (Decision, weight seed). Kept small: refcheck is pure Python."""
    c1 = synth.parity_decision(1)
    rng = np.random.Generator(np.random.PCG64(11))
    short = synth._decision(rng, 9, [3, 6], 2)
    rng = np.random.Generator(np.random.PCG64(12))
    window = synth._decision(rng, 150, [10, 40, 70], 1)
    return {"c1_L64": c1, "edge_L9_K2": short, "edge_L150_K3": window}


def load_refcheck(reference: str):
    path = os.path.join(reference, "tools", "refcheck.py")
    spec = importlib.util.spec_from_file_location("refcheck", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def write_checkpoint(path: str) -> None:
    w = synth.make_weights(WEIGHT_SEED)
    safetensors.write(path, {k: ("F16", synth.bf16_to_f16_bits(v)) for k, v in w.items()})


def fingerprint(x):
    flat = [t for row in x for t in row]
    return [flat[0], flat[1], flat[2], math.fsum(flat), math.fsum(abs(t) for t in flat)]


def act_head(rc, st, pooled, logits):
    """src/main.zig:2787-2814 in f64 with refcheck's helpers."""
    K = len(logits)
    p = rc.softmax(logits) if K else []
    kk = float(max(K, 2))
    ent = 0.0
    for v in p:
        if v > 1e-12:
            ent -= v * math.log(v)
    ent /= math.log(kk)
    t0 = t1 = 0.0
    for v in p:
        if v > t0:
            t1 = t0
            t0 = v
        elif v > t1:
            t1 = v
    feats = [t0, t0 - t1, ent, kk / 255.0]
    act_in = list(pooled) + feats
    h = rc.matvec(st, "act_head.0.weight", act_in)
    b0 = st.get("act_head.0.bias")
    h = [rc.gelu(t + b0[i]) for i, t in enumerate(h)]
    a = rc.matvec(st, "act_head.2.weight", h)
    b2 = st.get("act_head.2.bias")
    a = [t + b2[i] for i, t in enumerate(a)]
    return rc.softmax(a), feats


def run_case(args):
    name, reference, ckpt, outdir = args
    rc = load_refcheck(reference)
    dec = cases()[name]
    ids = [int(t) for t in dec.ids]
    marks = [int(t) for t in dec.markers]
    st = rc.Safetensors(ckpt)
    tags = {}
    x = [list(r) for r in st.rows("encoder.embeddings.tok_embeddings.weight", rc.D, ids)]
    x = [rc.layernorm(row, st.get("encoder.embeddings.norm.weight")) for row in x]
    tags["emb"] = fingerprint(x)
    for l in range(rc.NL):
        x = rc.encoder_layer(st, x, l)
        tags["l%d" % l] = fingerprint(x)
        st.drop("encoder.layers.%d." % l)
    x = [rc.layernorm(row, st.get("encoder.final_norm.weight")) for row in x]
    tags["final"] = fingerprint(x)
    te = st.rows("type_emb.weight", rc.D, [dec.qtype])[0]
    x = [[t + te[d] for d, t in enumerate(row)] for row in x]
    tags["temb"] = fingerprint(x)
    for l in range(2):
        x = rc.head_layer(st, x, l)
        tags["h%d" % l] = fingerprint(x)
    logits = [rc.scorer(st, x[m]) for m in marks]
    probs = rc.softmax(logits) if logits else []
    act, feats = act_head(rc, st, x[0], logits)
    rows = sorted(set([0] + marks + [len(ids) - 1]))
    out = {
        "case": name,
        "generator": "tests/golden/make_golden.py via the reference's tools/refcheck.py",
        "weights": {"generator": "laya_zig_b200.synth.make_weights", "seed": WEIGHT_SEED},
        "L": len(ids), "qtype": dec.qtype, "ids": ids, "markers": marks,
        "tags": tags, "logits": logits, "probs": probs, "act": act, "feats": feats,
        "hidden_rows": {str(r): x[r] for r in rows},
    }
    with open(os.path.join(outdir, name + ".json"), "w") as f:
        json.dump(out, f)
    if name == "c1_L64":
        np.save(os.path.join(outdir, name + "_hidden.npy"), np.asarray(x, dtype=np.float32))
    return name


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to a laya-zig checkout (holds tools/refcheck.py)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--cases", default=",".join(cases().keys()))
    args = ap.parse_args()
    tmp = tempfile.mkdtemp(prefix="laya_golden_")
    ckpt = os.path.join(tmp, "model.safetensors")
    write_checkpoint(ckpt)
    names = args.cases.split(",")
    ctx = mp.get_context("spawn")
    with ctx.Pool(len(names)) as pool:
        for done in pool.imap_unordered(run_case, [(n, args.reference, ckpt, args.out) for n in names]):
            print("done", done, flush=True)
    os.remove(ckpt)
    os.rmdir(tmp)


if __name__ == "__main__":
    main()
