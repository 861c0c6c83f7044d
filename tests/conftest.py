import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def pytest_sessionstart(session):
    """On a fresh checkout liblaya_gpu.so (kept out of git) is not there yet
    and the package refuses to import without it; build it once, in-tree,
    before any test imports the package (nvcc cross-compiles sm_100a on a
    host without a GPU)."""
    import subprocess
    lib = os.path.join(ROOT, "laya_zig_b200", "liblaya_gpu.so")
    if not os.path.exists(lib):
        subprocess.run([sys.executable, "-m", "laya_zig_b200.build"], cwd=ROOT, check=True)


@pytest.fixture(scope="session")
def weights():
    from laya_zig_b200 import synth
    return synth.make_weights(0)


@pytest.fixture(scope="session")
def oracle_model(weights):
    from oracle import oracle
    return oracle.model_from_bf16(weights)


@pytest.fixture(scope="session")
def gpu_model(weights):
    from laya_zig_b200 import gpu
    m = gpu.LayaGPU.from_bf16(weights, device=0)
    yield m
    m.close()


@pytest.fixture(scope="session")
def c3_oracle(oracle_model):
    """The oracle's outputs (with final hidden states) for the 64-decision
    Snake-style batch, computed once per session."""
    from laya_zig_b200 import synth
    return [oracle_model.forward(d.ids, d.markers, d.qtype, want_hidden=True) for d in synth.snake_batch(64)]


def golden_cases():
    import json
    out = {}
    for f in sorted(os.listdir(GOLDEN)):
        if f.endswith(".json"):
            with open(os.path.join(GOLDEN, f)) as fh:
                g = json.load(fh)
            if "case" in g:  # refcheck forward fixtures (make_golden.py), not separated.json
                out[f[:-5]] = g
    return out


def row_rel(got: np.ndarray, ref: np.ndarray) -> float:
    """max over rows of max_j |g - r| / max_j |r| (the hidden-state metric)."""
    got = np.atleast_2d(got).astype(np.float64)
    ref = np.atleast_2d(ref).astype(np.float64)
    return float((np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)).max())
