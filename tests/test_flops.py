"""The algorithmic work the roofline and the LPT sharding use, checked
against a brute-force count: attention FLOPs per decision are 4 * 768 per
visible (query, key) pair summed over the layers, with encoder layer l
global when l % 3 == 0 (src/main.zig:2366), the two head layers global, and
sliding layers seeing |i - j| <= 64 (attWorker, 2440-2444); GEMM FLOPs are
2 per weight per token over the 124,452,864 projection weights."""
import os
import sys

import numpy as np

from conftest import ROOT


def _pairs(L, window):
    i = np.arange(L)[:, None]
    j = np.arange(L)[None, :]
    if window < 0:
        return L * L
    return int(((j >= np.maximum(0, i - window)) & (j < np.minimum(L, i + window + 1))).sum())


def brute_attention_flops(L):
    layers = [(-1 if l % 3 == 0 else 64) for l in range(22)] + [-1, -1]
    return 4.0 * 768 * sum(_pairs(L, w) for w in layers)


def test_attention_flops_match_brute_force():
    sys.path.insert(0, ROOT)
    import bench
    from laya_zig_b200 import shard
    for L in (1, 2, 63, 64, 65, 128, 129, 130, 175, 180, 257, 512, 1000):
        want = brute_attention_flops(L)
        assert shard.attention_flops(L) == want, L
        assert bench.attn_flops(L) == want, L


def test_per_decision_work_at_the_configs():
    """44.80 GFLOP of projections and 1.82 GFLOP of attention per 180-token
    decision; 2.039 TFLOP and 2.11 TFLOP at 8,192 tokens."""
    from laya_zig_b200 import shard
    assert shard.GEMM_FLOPS_PER_TOKEN == 2 * 124_452_864
    assert abs(shard.GEMM_FLOPS_PER_TOKEN * 180 / 1e9 - 44.80) < 0.01
    assert abs(shard.attention_flops(180) / 1e9 - 1.82) < 0.01
    assert abs(shard.GEMM_FLOPS_PER_TOKEN * 8192 / 1e12 - 2.039) < 0.001
    assert abs(shard.attention_flops(8192) / 1e12 - 2.11) < 0.01


def test_projection_weight_count():
    """124,452,864 = 22 encoder layers x (Wqkv 2304x768 + Wo 768x768 + Wi
    2304x768 + Wo2 768x1152) + 2 head layers x (in_proj 2304x768 + out_proj
    768x768 + linear1 3072x768 + linear2 768x3072): the count behind the
    GEMM roofline's FLOPs per step."""
    sys.path.insert(0, ROOT)
    import bench
    enc = 2304 * 768 + 768 * 768 + 2304 * 768 + 768 * 1152
    head = 2304 * 768 + 768 * 768 + 3072 * 768 + 768 * 3072
    assert 22 * enc + 2 * head == 124_452_864 == bench.GEMM_PARAMS
