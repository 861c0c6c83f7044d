"""The decision tail that allocates nothing (laya_gpu_decision_tail_noalloc).

It serves callers that cannot let the library call cudaMalloc while deciding
(a process whose caching allocator owns the device's memory, or a serving
loop with a fixed memory budget): they hold final hidden states on the
device and want the option logits, act pair and pooled state for them. The
entry point keeps its scratch in a static device array instead of the
context's growable workspace. Checked here, through the C ABI, against the
regular forward's own tail outputs on the same hidden states, on two calls in
a row (the second one runs over the scratch the first left behind).

This file is collected last on purpose.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-6  # same kernels, same inputs: only scheduling could differ


def test_noalloc_tail_matches_forward(gpu_model):
    import torch
    from laya_zig_b200 import gpu, synth
    from test_gpu_device import _device_batch
    batch = synth.snake_batch(24, seed=11)
    b, keep = _device_batch(batch)
    M, S, G = b.c.n_tokens, b.c.n_seqs, b.c.n_markers
    logits = torch.zeros(G, dtype=torch.float32, device="cuda")
    act = torch.zeros((S, 2), dtype=torch.float32, device="cuda")
    pooled = torch.zeros((S, 768), dtype=torch.float32, device="cuda")
    hidden = torch.zeros((M, 768), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    gpu_model.forward_device(b, logits.data_ptr(), act.data_ptr(), pooled.data_ptr(), hidden.data_ptr(),
                             stream.cuda_stream)
    gpu_model.sync()
    for call in range(2):
        lg2 = torch.full((G,), float("nan"), dtype=torch.float32, device="cuda")
        act2 = torch.full((S, 2), float("nan"), dtype=torch.float32, device="cuda")
        pooled2 = torch.full((S, 768), float("nan"), dtype=torch.float32, device="cuda")
        gpu_model.decision_tail_noalloc(hidden.data_ptr(), b, lg2.data_ptr(), act2.data_ptr(), pooled2.data_ptr(),
                                        stream.cuda_stream)
        gpu_model.sync()
        np.testing.assert_allclose(lg2.cpu().numpy(), logits.cpu().numpy(), atol=TOL, rtol=0)
        np.testing.assert_allclose(act2.cpu().numpy(), act.cpu().numpy(), atol=TOL, rtol=0)
        np.testing.assert_allclose(pooled2.cpu().numpy(), pooled.cpu().numpy(), atol=TOL, rtol=0)


def test_noalloc_tail_rejects_too_many_markers(gpu_model):
    import torch
    from laya_zig_b200 import gpu
    n_seqs, per = 3, 1000  # 3000 markers > 2048
    cu = torch.tensor([0, 1000, 2000, 3000], dtype=torch.int32, device="cuda")
    cum = torch.tensor([0, per, 2 * per, 3 * per], dtype=torch.int32, device="cuda")
    mk = torch.zeros(3 * per, dtype=torch.int32, device="cuda")
    hid = torch.zeros((3000, 768), dtype=torch.float32, device="cuda")
    out = torch.zeros(3 * per, dtype=torch.float32, device="cuda")
    act = torch.zeros((n_seqs, 2), dtype=torch.float32, device="cuda")
    pooled = torch.zeros((n_seqs, 768), dtype=torch.float32, device="cuda")
    b = gpu.DeviceBatch(0, cu.data_ptr(), mk.data_ptr(), cum.data_ptr(), 0, n_seqs, 3000, 3 * per, 1000)
    with pytest.raises(gpu.LayaError, match="no-allocation limit of 2048"):
        gpu_model.decision_tail_noalloc(hid.data_ptr(), b, out.data_ptr(), act.data_ptr(), pooled.data_ptr())


def _tail_setup(gpu_model, batch):
    """Device batch, the regular forward's outputs for it and its final hidden state."""
    import torch
    from test_gpu_device import _device_batch
    b, keep = _device_batch(batch)
    M, S, G = b.c.n_tokens, b.c.n_seqs, b.c.n_markers
    ref = {"logits": torch.zeros(max(G, 1), dtype=torch.float32, device="cuda"),
           "act": torch.zeros((S, 2), dtype=torch.float32, device="cuda"),
           "pooled": torch.zeros((S, 768), dtype=torch.float32, device="cuda"),
           "hidden": torch.zeros((M, 768), dtype=torch.float32, device="cuda")}
    gpu_model.forward_device(b, ref["logits"].data_ptr(), ref["act"].data_ptr(), ref["pooled"].data_ptr(),
                             ref["hidden"].data_ptr())
    gpu_model.sync()
    return b, keep, ref


def _tail(gpu_model, b, hidden, G, S):
    import torch
    out = {"logits": torch.full((max(G, 1),), float("nan"), dtype=torch.float32, device="cuda"),
           "act": torch.full((S, 2), float("nan"), dtype=torch.float32, device="cuda"),
           "pooled": torch.full((S, 768), float("nan"), dtype=torch.float32, device="cuda")}
    gpu_model.decision_tail_noalloc(hidden.data_ptr(), b, out["logits"].data_ptr(), out["act"].data_ptr(),
                                    out["pooled"].data_ptr())
    return out


def test_noalloc_tail_sequence_without_markers(gpu_model):
    """A batch in which one sequence has no option markers (K = 0 in the act
    head) gives what the regular forward gives."""
    from laya_zig_b200 import synth
    rng = np.random.Generator(np.random.PCG64(29))
    batch = [synth._decision(rng, 60, [5, 17], 0), synth._decision(rng, 33, [], 1),
             synth._decision(rng, 90, [2, 44, 61, 80], 2)]
    b, keep, ref = _tail_setup(gpu_model, batch)
    out = _tail(gpu_model, b, ref["hidden"], 6, 3)
    gpu_model.sync()
    for k in ("act", "pooled"):
        np.testing.assert_allclose(out[k].cpu().numpy(), ref[k].cpu().numpy(), atol=TOL, rtol=0)
    np.testing.assert_allclose(out["logits"].cpu().numpy()[:6], ref["logits"].cpu().numpy()[:6], atol=TOL, rtol=0)


def test_noalloc_tail_device_errors(gpu_model):
    """Inputs only the device sees: a marker past its sequence's end, a
    sequence of 1025 markers (the per-sequence limit is 1024; the call's
    total, 1028, is under the 2048 of the static array) and a marker table
    whose end is not n_markers. The call returns LAYA_OK, laya_gpu_sync
    reports the error, and the next good call on the context is exact."""
    import torch
    from laya_zig_b200 import gpu, synth
    batch = synth.snake_batch(6, seed=31)
    b, keep, ref = _tail_setup(gpu_model, batch)
    S, G = b.c.n_seqs, b.c.n_markers
    good_markers = keep["markers"].clone()

    def good_call():
        keep["markers"].copy_(good_markers)
        out = _tail(gpu_model, b, ref["hidden"], G, S)
        gpu_model.sync()
        for k in ("logits", "act", "pooled"):
            np.testing.assert_allclose(out[k].cpu().numpy(), ref[k].cpu().numpy(), atol=TOL, rtol=0)

    # a marker past the end of its sequence
    keep["markers"][int(keep["cu_markers"][2].item()) + 1] = 500
    _tail(gpu_model, b, ref["hidden"], G, S)
    with pytest.raises(gpu.LayaError, match="rejected an index"):
        gpu_model.sync()
    good_call()

    # cu_markers[n_seqs] != n_markers
    cum = keep["cu_markers"]
    cum[-1] -= 1
    _tail(gpu_model, b, ref["hidden"], G, S)
    with pytest.raises(gpu.LayaError, match="rejected an index"):
        gpu_model.sync()
    cum[-1] += 1
    good_call()

    # 1025 markers in one sequence
    rng = np.random.Generator(np.random.PCG64(37))
    big = [synth._decision(rng, 150, [], 0), synth._decision(rng, 40, [3, 9, 27], 1)]
    big[0].markers = (np.arange(1025) % 150).astype(np.uint32)
    from test_gpu_device import _device_batch
    b2, keep2 = _device_batch(big)
    hid = torch.zeros((190, 768), dtype=torch.float32, device="cuda")
    _tail(gpu_model, b2, hid, 1028, 2)
    with pytest.raises(gpu.LayaError, match="rejected an index"):
        gpu_model.sync()
    good_call()
