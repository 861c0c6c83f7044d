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
