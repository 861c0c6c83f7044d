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


def _bad_table_cases(batch):
    """(label, edit) pairs; each edit takes the packed host arrays of `batch`
    (4 sequences) and breaks one device-resident table in a way the kernels'
    own checks catch without touching memory outside the buffers."""
    def cu_short(p):      # the last 5 tokens belong to no sequence
        p["cu_seqlens"][-1] -= 5

    def cu_long(p):       # the last sequence runs 100 rows past the batch
        p["cu_seqlens"][-1] += 100

    def qtype(p):
        p["qtypes"][2] = 7

    def marker(p):        # a marker past its sequence's end
        L1 = int(p["cu_seqlens"][2] - p["cu_seqlens"][1])
        p["markers"][int(p["cu_markers"][1]) + 3] = L1 + 4

    def cum_end(p):       # cu_markers[n] != n_markers: the last two markers are in no run
        p["cu_markers"][-1] -= 2

    def maxlen(p):        # a sequence longer than the attention grid covers
        p["max_len"] = int(np.diff(p["cu_seqlens"]).max()) - 70

    return [("cu_seqlens[n] < n_tokens", cu_short), ("cu_seqlens[n] > n_tokens", cu_long),
            ("qtype 7", qtype), ("marker past its sequence", marker), ("cu_markers[n] != n_markers", cum_end),
            ("max_len too small", maxlen)]


def test_device_tables_checked_on_the_device(gpu_model):
    """laya_gpu_forward_device does not validate on the host; each kernel
    checks the tables it reads. A broken table makes laya_gpu_sync report
    LAYA_ERR_ARG, and the next good call on the same context is exact."""
    import torch
    from laya_zig_b200 import gpu, synth
    batch = synth.snake_batch(4, seed=17)
    good = gpu.pack(batch)
    S, M, G = len(batch), len(good["ids"]), int(good["cu_markers"][-1])
    logits = torch.zeros(G, dtype=torch.float32, device="cuda")
    act = torch.zeros((S, 2), dtype=torch.float32, device="cuda")

    def run(p):
        t = {k: torch.from_numpy(v.view(np.int32).copy()).cuda() for k, v in p.items() if k != "max_len"}
        b = gpu.DeviceBatch(t["ids"].data_ptr(), t["cu_seqlens"].data_ptr(), t["markers"].data_ptr(),
                            t["cu_markers"].data_ptr(), t["qtypes"].data_ptr(), S, M, G, p["max_len"])
        gpu_model.forward_device(b, logits.data_ptr(), act.data_ptr())
        return t

    keep = run(good)
    gpu_model.sync()
    ref_logits, ref_act = logits.cpu().numpy().copy(), act.cpu().numpy().copy()
    for label, edit in _bad_table_cases(batch):
        p = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in good.items()}
        edit(p)
        keep = run(p)
        with pytest.raises(gpu.LayaError, match="rejected an index"):
            gpu_model.sync()
        keep = run(good)  # the context is usable and exact again
        gpu_model.sync()
        np.testing.assert_array_equal(logits.cpu().numpy(), ref_logits, err_msg=label)
        np.testing.assert_array_equal(act.cpu().numpy(), ref_act, err_msg=label)


def test_device_path_rejects_1025_markers_in_one_sequence(gpu_model):
    """LAYA_MAX_MARKERS (1024) per sequence holds on the device path too: the
    act head flags the run instead of scoring only its first 1024 markers."""
    import torch
    from laya_zig_b200 import gpu, synth
    rng = np.random.Generator(np.random.PCG64(23))
    batch = [synth._decision(rng, 150, [], 0), synth._decision(rng, 40, [3, 9, 27], 1)]
    batch[0].markers = (np.arange(1025) % 150).astype(np.uint32)
    b, keep = _device_batch(batch)
    logits = torch.zeros(1028, dtype=torch.float32, device="cuda")
    act = torch.zeros((2, 2), dtype=torch.float32, device="cuda")
    gpu_model.forward_device(b, logits.data_ptr(), act.data_ptr())
    with pytest.raises(gpu.LayaError, match="rejected an index"):
        gpu_model.sync()
