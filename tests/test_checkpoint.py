"""The F16 checkpoint path: the reference ships its matrices as F16
safetensors (tensorF16 accepts nothing else, src/main.zig:1344-1362), and
loadModel (main.zig:2311-2404) maps the file and hands the views on.

* `LayaGPU.from_safetensors` reads an F16 model.safetensors written from the
  seeded weights (every value exact in f16 and bf16) and uploads it with
  LAYA_DT_F16 tags: the device converts F16 -> bf16 (or keeps f16).
* `laya_zig_b200/laya_forward` is a plain C program doing what the Zig glue
  does (mmap, parse the header, laya_gpu_create on views of the mapping,
  laya_gpu_forward / laya_gpu_forward_dumpstats); the tests run it.

The weights uploaded from F16 are bit-identical to the bf16 upload the other
GPU tests use, so the forward's outputs must be bit-identical too; they are
also checked against the oracle at the C1 and C3 bars.
"""
import json
import os
import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT, row_rel

EXE = os.path.join(ROOT, "laya_zig_b200", "laya_forward")


def _write_f16(path, weights, drop=None):
    from laya_zig_b200 import safetensors, synth
    safetensors.write(path, {k: ("F16", synth.bf16_to_f16_bits(v)) for k, v in weights.items() if k != drop})


def _run(*args):
    return subprocess.run([EXE] + [str(a) for a in args], capture_output=True, text=True, timeout=600)


def _csv(a):
    return ",".join(str(int(v)) for v in a) if len(a) else "-"


# ---------------------------------------------------------------- CPU: the loader's refusals
def test_host_program_rejects_bad_files(tmp_path):
    """BadSafetensors cases of loadModel (main.zig:2321-2323) and a header that
    is not a JSON object: exit status 2 before any device work."""
    short = tmp_path / "short.safetensors"
    short.write_bytes(b"\x01\x02\x03")
    r = _run(short, 0, "2,5,1", "-")
    assert r.returncode == 2 and "BadSafetensors" in r.stderr
    long_hdr = tmp_path / "long.safetensors"
    long_hdr.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    r = _run(long_hdr, 0, "2,5,1", "-")
    assert r.returncode == 2 and "header length" in r.stderr
    junk = tmp_path / "junk.safetensors"
    junk.write_bytes(struct.pack("<Q", 6) + b"[1, 2]")
    r = _run(junk, 0, "2,5,1", "-")
    assert r.returncode == 2 and "JSON" in r.stderr
    past = tmp_path / "past.safetensors"
    hdr = json.dumps({"a": {"dtype": "F16", "shape": [4], "data_offsets": [0, 64]}}).encode()
    past.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 8)
    r = _run(past, 0, "2,5,1", "-")
    assert r.returncode == 2 and "past the end" in r.stderr


def test_host_program_parses_a_written_checkpoint(tmp_path):
    """A well-formed file passes the loader; on a host without a GPU the
    create call is what fails (status 3, no device)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from laya_zig_b200 import safetensors
    p = tmp_path / "m.safetensors"
    safetensors.write(str(p), {"x.weight": ("F16", np.arange(6, dtype=np.uint16).reshape(2, 3)),
                               "y.bias": ("F32", np.ones(3, np.float32))})
    r = _run(p, 0, "2,5,1", "1")
    assert r.returncode == 3 and "laya_gpu_create" in r.stderr, r.stderr


# ---------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def f16_file(tmp_path_factory, weights):
    p = str(tmp_path_factory.mktemp("ckpt") / "model.safetensors")
    _write_f16(p, weights)
    return p


@pytest.mark.gpu
def test_f16_checkpoint_upload_parity(f16_file, gpu_model, oracle_model, c3_oracle):
    from laya_zig_b200 import gpu, synth
    from test_gpu_forward import _compare
    m = gpu.LayaGPU.from_safetensors(f16_file)
    try:
        d = synth.parity_decision(1)
        g = m.forward(d.ids, d.qtype, d.markers, want_hidden=True)
        b = gpu_model.forward(d.ids, d.qtype, d.markers, want_hidden=True)
        np.testing.assert_array_equal(g.hidden, b.hidden)
        np.testing.assert_array_equal(g.logits, b.logits)
        _compare(g, oracle_model.forward(d.ids, d.markers, d.qtype, want_hidden=True), "c1 from F16")
        batch = synth.snake_batch(64)
        outs = m.forward_batch(batch, want_pooled=True)
        ref = gpu_model.forward_batch(batch, want_pooled=True)
        for i, (o, r_gpu, r) in enumerate(zip(outs, ref, c3_oracle)):
            np.testing.assert_array_equal(o.logits, r_gpu.logits)
            np.testing.assert_array_equal(o.act, r_gpu.act)
            np.testing.assert_array_equal(o.pooled, r_gpu.pooled)
            assert np.abs(gpu.option_probs(o.logits, 0) - gpu.option_probs(r["logits"], 0)).max() <= 1e-3
            assert np.abs(o.act - r["act"]).max() <= 1e-3
            assert row_rel(o.pooled, r["pooled"]) <= 2e-2
    finally:
        m.close()


@pytest.mark.gpu
def test_f16_checkpoint_missing_tensor(tmp_path, weights):
    from laya_zig_b200 import gpu
    p = str(tmp_path / "model.safetensors")
    _write_f16(p, weights, drop="encoder.layers.5.mlp.Wo.weight")
    with pytest.raises(gpu.MissingTensor, match="missing tensor: encoder.layers.5.mlp.Wo.weight"):
        gpu.LayaGPU.from_safetensors(p)
    r = _run(p, 0, "2,5,1", "-")
    assert r.returncode == 3 and "missing tensor: encoder.layers.5.mlp.Wo.weight" in r.stderr


@pytest.mark.gpu
def test_host_program_forward(f16_file, gpu_model, oracle_model):
    """The C host's forward on the mapped F16 file equals the library's
    forward from bf16 arrays bit for bit, and meets the C1 bars."""
    from laya_zig_b200 import gpu, synth
    for d in (synth.parity_decision(1), synth.parity_decision(104, option_tokens=True)):
        r = _run(f16_file, d.qtype, _csv(d.ids), _csv(d.markers))
        assert r.returncode == 0, r.stderr
        out = json.loads(r.stdout)
        b = gpu_model.forward(d.ids, d.qtype, d.markers)
        np.testing.assert_array_equal(np.array(out["logits"], np.float32), b.logits)
        np.testing.assert_array_equal(np.array(out["act"], np.float32), b.act)
        np.testing.assert_array_equal(np.array(out["pooled"], np.float32), b.pooled)
        ref = oracle_model.forward(d.ids, d.markers, d.qtype)
        assert np.abs(gpu.option_probs(np.array(out["logits"]), 0) - gpu.option_probs(ref["logits"], 0)).max() <= 1e-3
        assert np.abs(np.array(out["act"]) - ref["act"]).max() <= 1e-3


@pytest.mark.gpu
def test_host_program_dumpstats(f16_file, gpu_model):
    """--dumpstats through the C host prints what laya_gpu_forward_dumpstats
    gives the Python host, byte for byte."""
    from laya_zig_b200 import synth
    d = synth.parity_decision(1)
    r = _run(f16_file, d.qtype, _csv(d.ids), _csv(d.markers), "--dumpstats")
    assert r.returncode == 0, r.stderr
    _, _, text = gpu_model.forward_dumpstats(d.ids, d.qtype, d.markers)
    assert r.stdout == text
