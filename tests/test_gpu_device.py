"""The device-resident entry point (laya_gpu_forward_device) and f16 mode."""
import numpy as np
import pytest

from conftest import row_rel

pytestmark = pytest.mark.gpu


def _device_batch(decisions):
    import torch
    from laya_zig_b200 import gpu
    p = gpu.pack(decisions)
    t = {k: torch.from_numpy(v.view(np.int32)).cuda() for k, v in p.items() if k != "max_len"}
    b = gpu.DeviceBatch(t["ids"].data_ptr(), t["cu_seqlens"].data_ptr(), t["markers"].data_ptr(),
                        t["cu_markers"].data_ptr(), t["qtypes"].data_ptr(), len(decisions), len(p["ids"]),
                        int(p["cu_markers"][-1]), p["max_len"])
    return b, t


def test_device_path_equals_host_path(gpu_model):
    import torch
    from laya_zig_b200 import synth
    batch = synth.snake_batch(16, seed=5)
    b, keep = _device_batch(batch)
    G = sum(len(d.markers) for d in batch)
    logits = torch.zeros(G, dtype=torch.float32, device="cuda")
    act = torch.zeros((len(batch), 2), dtype=torch.float32, device="cuda")
    pooled = torch.zeros((len(batch), 768), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(2):  # the second call replays the captured graph
        gpu_model.forward_device(b, logits.data_ptr(), act.data_ptr(), pooled.data_ptr(), 0, stream.cuda_stream)
    gpu_model.sync()
    host = gpu_model.forward_batch(batch, want_pooled=True)
    np.testing.assert_array_equal(np.concatenate([h.logits for h in host]), logits.cpu().numpy())
    np.testing.assert_array_equal(np.stack([h.act for h in host]), act.cpu().numpy())
    np.testing.assert_array_equal(np.stack([h.pooled for h in host]), pooled.cpu().numpy())


def test_f16_precision_parity(weights, oracle_model):
    """f16 operands (the checkpoint's own storage type) meet the same bar, tighter."""
    from laya_zig_b200 import gpu, synth
    m = gpu.LayaGPU.from_bf16(weights, precision="f16")
    try:
        d = synth.parity_decision(1)
        g = m.forward(d.ids, d.qtype, d.markers, want_hidden=True)
        r = oracle_model.forward(d.ids, d.markers, d.qtype, want_hidden=True)
        err = row_rel(g.hidden, r["hidden"])
        print("f16 hidden max-rel %.3e" % err)
        assert err <= 2e-2
        assert int(np.argmax(g.logits)) == int(np.argmax(r["logits"]))
    finally:
        m.close()


def test_prepared_batch_equals_forward_batch(gpu_model):
    """The prepared host-buffer call (used for the end-to-end timing) returns
    what forward_batch returns, call after call."""
    from laya_zig_b200 import gpu, synth
    batch = synth.snake_batch(12, seed=9)
    pb = gpu.PreparedBatch(batch)
    ref = gpu_model.forward_batch(batch)
    for _ in range(2):
        logits, act = gpu_model.forward_prepared(pb)
        np.testing.assert_array_equal(np.concatenate([h.logits for h in ref]), logits)
        np.testing.assert_array_equal(np.stack([h.act for h in ref]), act)
