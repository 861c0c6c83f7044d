"""Host-side logic that needs no GPU: the C ABI library, synthetic inputs,
packing, sharding, safetensors and the caller-side probabilities."""
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared_symbols():
    syms = set()
    inc = os.path.join(ROOT, "include")
    for name in sorted(os.listdir(inc)):
        if name.endswith(".h"):
            with open(os.path.join(inc, name)) as f:
                syms |= set(re.findall(r"LAYA_(?:TOK_)?API\s+[\w\s\*]*?\b(laya_\w+)\s*\(", f.read()))
    return sorted(syms)


def test_library_loads_and_exports_every_declared_symbol():
    """Every entry point of include/*.h (laya_gpu.h and laya_tok.h)."""
    from laya_zig_b200 import gpu
    syms = _declared_symbols()
    assert len(syms) >= 19, syms
    assert any(s.startswith("laya_tok_") for s in syms)
    for s in syms:
        assert hasattr(gpu.lib, s), "liblaya_gpu.so does not export %s" % s
    assert gpu.lib.laya_gpu_version() == 1


def test_create_without_device_fails_cleanly(weights):
    """On a host with no usable GPU, create reports it instead of crashing."""
    import torch
    from laya_zig_b200 import gpu
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert gpu.lib.laya_gpu_device_count() == 0
    with pytest.raises(gpu.LayaError) as e:
        gpu.LayaGPU.from_bf16({k: v for k, v in list(weights.items())[:3]})
    assert e.value.code == gpu.ERR_NODEV


def test_synth_weights_are_exact_in_f16_and_deterministic(weights):
    from laya_zig_b200 import synth
    names = [n for n, _, _ in synth.tensor_specs()]
    assert len(names) == len(set(names)) == len(weights)
    assert sum(v.size for v in weights.values()) == 321_908_995
    for n in ["encoder.layers.7.mlp.Wi.weight", "scorer.1.weight", "encoder.embeddings.norm.weight"]:
        b = weights[n]
        f = synth.bf16_bits_to_f32(b)
        assert np.array_equal(synth.bf16_to_f16_bits(b).view(np.float16).astype(np.float32), f)
    again = synth.make_weights(0)
    for n in ["encoder.layers.21.attn.Wo.weight", "act_head.0.weight"]:
        assert np.array_equal(again[n], weights[n])
    w = synth.bf16_bits_to_f32(weights["encoder.layers.3.attn.Wqkv.weight"])
    assert abs(w.std() - 0.02) < 1e-3 and abs(w.mean()) < 1e-3


def test_workloads_shapes():
    from laya_zig_b200 import synth
    c1 = synth.parity_decision(1)
    assert len(c1.ids) == 64 and list(c1.markers) == [8, 16, 24, 32] and c1.qtype == 0
    b = synth.snake_batch(64)
    assert len(b) == 64 and all(175 <= len(d.ids) <= 180 and len(d.markers) == 8 for d in b)
    assert all(d.ids[0] == synth.CLS_ID and (d.ids[d.markers] == synth.MASK_ID).all() for d in b)
    lc = synth.long_decision()
    assert len(lc.ids) == 8192 and len(set(lc.markers.tolist())) == 16
    sw = synth.sweep_decisions(2000)
    assert all(128 <= len(d.ids) <= 512 for d in sw)
    for bk in synth.bucket(sw):
        assert sum(len(sw[i].ids) for i in bk) <= 32768


def test_pack():
    from laya_zig_b200 import gpu, synth
    b = synth.snake_batch(7, seed=3)
    p = gpu.pack(b)
    assert p["cu_seqlens"][-1] == len(p["ids"]) == sum(len(d.ids) for d in b)
    assert p["cu_markers"][-1] == len(p["markers"]) == 7 * 8
    assert p["max_len"] == max(len(d.ids) for d in b)
    for s, d in enumerate(b):
        assert np.array_equal(p["ids"][p["cu_seqlens"][s]:p["cu_seqlens"][s + 1]], d.ids)


def test_option_probs_matches_reference_formula():
    from laya_zig_b200 import gpu
    lg = np.array([0.3, -1.0, 2.0, 0.5], np.float32)
    for t in [1.0, 0.5, 0.0]:  # temperature clamps at 1e-3 (src/main.zig:3800)
        p = gpu.option_probs(lg, 1, (1.0, t, 1.0))
        z = lg / max(1e-3, t)
        e = np.exp(z - z.max())
        assert np.allclose(p, e / e.sum(), atol=1e-7)


def test_safetensors_roundtrip_and_errors(tmp_path):
    from laya_zig_b200 import safetensors
    t = {"a": ("F16", np.arange(6, dtype=np.float16).reshape(2, 3).view(np.uint16)),
         "b": ("F32", np.linspace(0, 1, 5, dtype=np.float32))}
    p = str(tmp_path / "m.safetensors")
    safetensors.write(p, t)
    r = safetensors.read(p)
    assert r["a"][0] == "F16" and np.array_equal(r["a"][1], t["a"][1])
    assert np.array_equal(r["b"][1], t["b"][1])
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\x00\x01")
    with pytest.raises(safetensors.SafetensorsError):
        safetensors.read(str(bad))


def test_lpt_assignment_balances():
    from laya_zig_b200 import shard, synth
    sw = synth.sweep_decisions(4096, seed=4)
    for world in [1, 2, 4, 8]:
        mine = [shard.shard(sw, world, r)[0] for r in range(world)]
        loads = shard.shard(sw, world, 0)[1]
        flat = sorted(i for r in mine for b in r for i in b)
        assert flat == list(range(len(sw)))  # every decision exactly once
        assert max(loads) / (sum(loads) / world) < 1.15


def test_prepared_batch_marshals_every_sequence():
    """PreparedBatch points each laya_seq at the caller's arrays, in order."""
    import ctypes
    from laya_zig_b200 import gpu, synth
    batch = synth.snake_batch(5, seed=3)
    pb = gpu.PreparedBatch(batch)
    assert pb.n == 5 and pb.act.shape == (5, 2)
    assert len(pb.logits) == sum(len(d.markers) for d in batch)
    for i, d in enumerate(batch):
        sq = pb.seqs[i]
        assert sq.len == len(d.ids) and sq.n_markers == len(d.markers) and sq.qtype == int(d.qtype)
        ids = np.ctypeslib.as_array(ctypes.cast(sq.ids, ctypes.POINTER(ctypes.c_uint32)), shape=(sq.len,))
        np.testing.assert_array_equal(ids, np.asarray(d.ids, np.uint32))

