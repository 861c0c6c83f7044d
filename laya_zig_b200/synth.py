"""Seeded synthetic weights and decision batches for the Laya mmBERT encoder.

No checkpoint ships with this repository (the reference keeps
`model.safetensors` out of git, README.md:214-227), so every parity test and
every benchmark runs on weights produced here from a seed.

Weights
-------
Every tensor the reference loads (src/main.zig:2344-2397) is produced under
its own safetensors name. Values come from a counter-based hash, so any
element can be produced independently and the result does not depend on the
platform, the numpy build or the chunking:

* ``h = splitmix64(seed_of(name) + index)``; its four 16-bit fields are summed
  (an Irwin-Hall(4) variate: mean 2*65535, variance 4/12 * 65536^2).
* ``z = (sum - 131070) * sqrt(3)/65536`` is then ~N(0, 1), bounded at
  +-3.46.  Only one IEEE multiply touches the value, so it is bit-identical
  everywhere (no transcendental functions, whose last bit varies between
  SIMD libraries).
* Matrices, biases and embeddings are ``0.02 * z``; LayerNorm gains are
  ``1 + 0.02 * z`` (pure N(0, 0.02) gains would collapse every activation).
* Each value is rounded to bf16 (round-to-nearest-even) and magnitudes below
  2^-14 are flushed to zero, so every value is exact in bf16 *and* in f16:
  the F16 checkpoint the reference reads and the bf16 image uploaded to the
  GPU hold bit-identical weights.

Batches
-------
Token ids are drawn with numpy's PCG64 from the workload's seed. Each
sequence starts with [CLS] (id 2), ends with [SEP] (id 1) and carries [MASK]
(id 4) at its option markers, the shape `buildSequence`
(src/main.zig:2842-2911) gives real prompts.

With random weights the hidden states of identical [MASK] tokens differ
only through their weakly mixed context, so the option logits of such a
decision lie within about 1e-2 of each other and their order is a near-tie
that 16-bit tensor-core operands cannot reproduce. `option_tokens=True`
puts a random token at each marker instead, as the distinct option text
after each <mask> does for a trained model: the logits then spread about
15x wider (median top-two margin 6e-2 against 5e-3 on the 64 x 180 batch).
"""
from __future__ import annotations

import dataclasses
import zlib
from typing import Dict, List, Sequence, Tuple

import numpy as np

# Architecture (src/main.zig:39-57).
D = 768
H = 12
HD = 64
NL = 22
INTER = 1152
HEAD_LAYERS = 2
HEAD_FF = 4 * D
VOCAB = 256000
CLS_ID = 2
SEP_ID = 1
MASK_ID = 4

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
_GOLD = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)
_SCALE = np.float32(0.02 * np.sqrt(3.0) / 65536.0)
_CHUNK = 1 << 20


def tensor_specs() -> List[Tuple[str, Tuple[int, ...], str]]:
    """(name, shape, kind) for every tensor `loadModel` reads.

    kind is "mat" (F16 matrix in the reference), "vec" (small tensor the
    reference copies to f32) or "gain" (a LayerNorm weight).
    Order and names follow src/main.zig:2344-2397.
    """
    specs: List[Tuple[str, Tuple[int, ...], str]] = [
        ("encoder.embeddings.tok_embeddings.weight", (VOCAB, D), "mat"),
        ("encoder.embeddings.norm.weight", (D,), "gain"),
        ("encoder.final_norm.weight", (D,), "gain"),
        ("type_emb.weight", (3, D), "vec"),
    ]
    for l in range(NL):
        p = "encoder.layers.%d." % l
        if l > 0:
            specs.append((p + "attn_norm.weight", (D,), "gain"))
        specs += [
            (p + "attn.Wqkv.weight", (3 * D, D), "mat"),
            (p + "attn.Wo.weight", (D, D), "mat"),
            (p + "mlp.Wi.weight", (2 * INTER, D), "mat"),
            (p + "mlp.Wo.weight", (D, INTER), "mat"),
            (p + "mlp_norm.weight", (D,), "gain"),
        ]
    for l in range(HEAD_LAYERS):
        p = "head.layers.%d." % l
        specs += [
            (p + "norm1.weight", (D,), "gain"),
            (p + "norm1.bias", (D,), "vec"),
            (p + "norm2.weight", (D,), "gain"),
            (p + "norm2.bias", (D,), "vec"),
            (p + "self_attn.in_proj_weight", (3 * D, D), "mat"),
            (p + "self_attn.in_proj_bias", (3 * D,), "vec"),
            (p + "self_attn.out_proj.weight", (D, D), "mat"),
            (p + "self_attn.out_proj.bias", (D,), "vec"),
            (p + "linear1.weight", (HEAD_FF, D), "mat"),
            (p + "linear1.bias", (HEAD_FF,), "vec"),
            (p + "linear2.weight", (D, HEAD_FF), "mat"),
            (p + "linear2.bias", (D,), "vec"),
        ]
    specs += [
        ("scorer.0.weight", (D,), "gain"),
        ("scorer.0.bias", (D,), "vec"),
        ("scorer.1.weight", (D, D), "vec"),
        ("scorer.1.bias", (D,), "vec"),
        ("scorer.3.weight", (1, D), "vec"),
        ("scorer.3.bias", (1,), "vec"),
        ("act_head.0.weight", (256, D + 4), "vec"),
        ("act_head.0.bias", (256,), "vec"),
        ("act_head.2.weight", (2, 256), "vec"),
        ("act_head.2.bias", (2,), "vec"),
    ]
    return specs


def _splitmix64(z: np.ndarray) -> np.ndarray:
    z = z ^ (z >> np.uint64(30))
    z = z * _C1
    z = z ^ (z >> np.uint64(27))
    z = z * _C2
    return z ^ (z >> np.uint64(31))


def _name_seed(seed: int, name: str) -> np.uint64:
    key = (int(seed) * 0x100000001B3 + zlib.crc32(name.encode())) & 0xFFFFFFFFFFFFFFFF
    return np.uint64(key)


def f32_to_bf16_bits(v: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, as raw uint16 bits (finite inputs)."""
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def _fill_range(base: np.uint64, kind: str, lo: int, hi: int, out_bits: np.ndarray) -> None:
    with np.errstate(over="ignore"):
        idx = np.arange(lo, hi, dtype=np.uint64)
        h = _splitmix64((base + idx) * _GOLD)
        s = (h & np.uint64(0xFFFF)) + ((h >> np.uint64(16)) & np.uint64(0xFFFF)) \
            + ((h >> np.uint64(32)) & np.uint64(0xFFFF)) + (h >> np.uint64(48))
        z = (s.astype(np.int64) - 131070).astype(np.float32) * _SCALE
        if kind == "gain":
            z = z + np.float32(1.0)
        bits = f32_to_bf16_bits(z)
        mag = bits & np.uint16(0x7FFF)
        bits[mag < np.uint16(0x3880)] = 0  # |v| < 2^-14 -> 0 (exact in f16 too)
        out_bits[lo:hi] = bits


def _fill(seed: int, name: str, kind: str, n: int, out_bits: np.ndarray, pool=None) -> None:
    base = _name_seed(seed, name)
    ranges = [(lo, min(n, lo + _CHUNK)) for lo in range(0, n, _CHUNK)]
    if pool is None or len(ranges) == 1:
        for lo, hi in ranges:
            _fill_range(base, kind, lo, hi, out_bits)
    else:
        list(pool.map(lambda r: _fill_range(base, kind, r[0], r[1], out_bits), ranges))


def make_weights(seed: int = 0) -> Dict[str, np.ndarray]:
    """All model tensors as bf16 bit patterns (numpy uint16), keyed by name."""
    import concurrent.futures
    import os
    out: Dict[str, np.ndarray] = {}
    workers = max(1, min(16, os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(workers) as pool:
        for name, shape, kind in tensor_specs():
            n = int(np.prod(shape))
            bits = np.empty(n, dtype=np.uint16)
            _fill(seed, name, kind, n, bits, pool)
            out[name] = bits.reshape(shape)
    return out


def bf16_to_f16_bits(b: np.ndarray) -> np.ndarray:
    """Exact for the values `make_weights` produces (|v| >= 2^-14 or 0)."""
    return bf16_bits_to_f32(b).astype(np.float16).view(np.uint16)


# --------------------------------------------------------------------------- batches
@dataclasses.dataclass
class Decision:
    """One sequence as `forward` sees it (src/main.zig:2529-2541)."""
    ids: np.ndarray       # uint32 [L]
    markers: np.ndarray   # uint32 [K], positions of the option [MASK] tokens
    qtype: int            # 0 choice, 1 score, 2 noul


def _decision(rng: np.random.Generator, L: int, markers: Sequence[int], qtype: int,
              option_tokens: bool = False) -> Decision:
    """Token ids uniform in [0, VOCAB) with [CLS] first and [SEP] last; the
    marker positions hold [MASK], or, with option_tokens, ids drawn at random
    (one per marker, after the sequence's ids)."""
    ids = rng.integers(0, VOCAB, size=L, dtype=np.int64).astype(np.uint32)
    ids[0] = CLS_ID
    if L > 1:
        ids[L - 1] = SEP_ID
    mk = np.asarray(markers, dtype=np.uint32)
    if option_tokens:
        ids[mk] = rng.integers(5, VOCAB, size=len(mk), dtype=np.int64).astype(np.uint32)
    else:
        ids[mk] = MASK_ID
    return Decision(ids=ids, markers=mk, qtype=int(qtype))


def parity_decision(seed: int = 1, option_tokens: bool = False) -> Decision:
    """Batch 1 x seq 64, four markers at fixed offsets, qtype 0."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return _decision(rng, 64, [8, 16, 24, 32], 0, option_tokens)


SNAKE_MARKERS = [20 + 18 * r for r in range(8)]


def snake_batch(batch: int = 64, seed: int = 2, lo: int = 175, hi: int = 180,
                option_tokens: bool = False) -> List[Decision]:
    """Snake-style decisions: lengths uniform in [lo, hi], 8 option markers
    at fixed offsets inside the head segment, qtype cycling 0/1/2."""
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = rng.integers(lo, hi + 1, size=batch)
    mk = [m for m in SNAKE_MARKERS if m < lo - 1]
    return [_decision(rng, int(L), mk, b % 3, option_tokens) for b, L in enumerate(lens)]


def long_decision(L: int = 8192, K: int = 16, seed: int = 3, option_tokens: bool = False) -> Decision:
    """One long sequence with K markers at random distinct positions."""
    rng = np.random.Generator(np.random.PCG64(seed))
    mk = np.sort(rng.choice(np.arange(1, L - 1), size=K, replace=False))
    return _decision(rng, L, mk.tolist(), 0, option_tokens)


def sweep_decisions(n: int = 65536, seed: int = 4, lo: int = 128, hi: int = 512) -> List[Decision]:
    """Throughput sweep: n decisions with lengths uniform in [lo, hi]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = rng.integers(lo, hi + 1, size=n)
    out = []
    for b, L in enumerate(lens):
        K = 4 + (b % 5)
        mk = [8 + 12 * r for r in range(K)]
        out.append(_decision(rng, int(L), mk, b % 3))
    return out


def bucket(decisions: Sequence[Decision], max_tokens: int = 32768) -> List[List[int]]:
    """Greedy length-sorted packing into batches of <= max_tokens tokens."""
    order = sorted(range(len(decisions)), key=lambda i: len(decisions[i].ids))
    buckets: List[List[int]] = []
    cur: List[int] = []
    tok = 0
    for i in order:
        L = len(decisions[i].ids)
        if cur and tok + L > max_tokens:
            buckets.append(cur)
            cur, tok = [], 0
        cur.append(i)
        tok += L
    if cur:
        buckets.append(cur)
    return buckets
