#!/usr/bin/env python
"""Generate tests/golden/separated.json: decisions whose option logits are
well separated, so that the argmax option is asserted on every one of them.

With seeded random weights, decisions whose markers are all [MASK] have
near-uniform option logits (top-two margins down to 1e-4), and their order
is decided by rounding: 16-bit tensor-core operands cannot reproduce it,
and neither can any arithmetic other than the reference's own f32 chain.
This script draws decisions of the parity shapes with a random token at
each marker (`synth.*(option_tokens=True)`, the analogue of the distinct
option text after each <mask>), runs the oracle, and keeps those whose
top-two logit margin is at least MIN_MARGIN, ten times or more the largest
logit error the bf16 forward shows. Only seeds and kept indices are stored;
the tests regenerate the decisions with laya_zig_b200.synth and compare the
GPU with the oracle on every kept decision.

    python tests/golden/make_separated.py            (about two minutes on 8 cores)
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from laya_zig_b200 import synth  # noqa: E402
from oracle import oracle  # noqa: E402

MIN_MARGIN = 1e-2


def margin(logits) -> float:
    s = np.sort(np.asarray(logits, np.float64))
    return float(s[-1] - s[-2])


def main():
    m = oracle.model_from_bf16(synth.make_weights(0))
    out = {"min_margin": MIN_MARGIN, "weights_seed": 0}

    c1 = []
    for seed in range(100, 140):
        d = synth.parity_decision(seed, option_tokens=True)
        mg = margin(m.forward(d.ids, d.markers, d.qtype)["logits"])
        if mg >= MIN_MARGIN:
            c1.append({"seed": seed, "margin": mg})
        if len(c1) == 8:
            break
    out["c1"] = c1

    seed, drawn = 42, 96
    batch = synth.snake_batch(drawn, seed=seed, option_tokens=True)
    kept, mgs = [], []
    for i, d in enumerate(batch):
        mg = margin(m.forward(d.ids, d.markers, d.qtype)["logits"])
        if mg >= MIN_MARGIN and len(kept) < 64:
            kept.append(i)
            mgs.append(mg)
    out["c3"] = {"seed": seed, "drawn": drawn, "kept": kept, "margins": mgs}

    for seed in range(3, 12):
        d = synth.long_decision(8192, 16, seed=seed, option_tokens=True)
        mg = margin(m.forward(d.ids, d.markers, d.qtype)["logits"])
        print("c4 seed %d margin %.3e" % (seed, mg), flush=True)
        if mg >= MIN_MARGIN:
            out["c4"] = {"seed": seed, "margin": mg}
            break
    with open(os.path.join(HERE, "separated.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("c1 %d kept; c3 %d of %d kept (min margin %.3e); c4 seed %s" % (
        len(c1), len(kept), drawn, min(mgs), out.get("c4", {}).get("seed")))


if __name__ == "__main__":
    main()
