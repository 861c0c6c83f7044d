"""tcgen05 projection GEMM through the C ABI (laya_gpu_linear).

The reference's --selftest (src/main.zig:420-536) checks its GEMM against
f64 on the model's shapes, every 29th column, with the metric
|got - ref| / max(1, |ref|) < 1e-4. The same check runs here on the GPU
kernel, with f64 computed from the same 16-bit-rounded operands, on the
isolated projection shapes: QKV 768->2304, attn-out 768->768, GLU Wi
768->2304, FFN-out 1152->768 at M = 180 and M = 11520 (64 x 180), plus the
selftest's odd row counts and the head's 3072-wide shapes.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(n, k) for n, k in [(2304, 768), (768, 768), (2304, 768), (768, 1152)]]


def _rand_bits(rng, shape, scale, f16=False):
    from laya_zig_b200.synth import f32_to_bf16_bits
    v = (rng.standard_normal(shape) * scale).astype(np.float32)
    if f16:
        return v.astype(np.float16).view(np.uint16)
    return f32_to_bf16_bits(v)


def _to_f64(bits, f16=False):
    from laya_zig_b200.synth import bf16_bits_to_f32
    if f16:
        return bits.view(np.float16).astype(np.float64)
    return bf16_bits_to_f32(bits).astype(np.float64)


def _gpu_linear(xb, wb, bias=None, f16=False):
    import torch
    from laya_zig_b200 import gpu
    dt = torch.float16 if f16 else torch.bfloat16
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(dt)
    w = torch.from_numpy(wb.view(np.int16)).cuda().view(dt)
    M, K = xb.shape
    N = wb.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b = None if bias is None else torch.from_numpy(bias).cuda()
    gpu.linear(x.data_ptr(), w.data_ptr(), 0 if b is None else b.data_ptr(), out.data_ptr(), M, N, K,
               "F16" if f16 else "BF16", torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _check(out, x64, w64, bias=None, every=29):
    cols = np.arange(0, w64.shape[0], every)
    ref = x64 @ w64[cols].T
    if bias is not None:
        ref = ref + bias[cols]
    rel = np.abs(out[:, cols] - ref) / np.maximum(1.0, np.abs(ref))
    return rel.max()


@pytest.mark.parametrize("M", [180, 11520])
@pytest.mark.parametrize("n,k", SHAPES)
def test_projection_gemm_bf16(M, n, k):
    rng = np.random.default_rng(M * 7 + n + k)
    xb = _rand_bits(rng, (M, k), 1.0)       # activations N(0, 1)
    wb = _rand_bits(rng, (n, k), 0.02)      # weights N(0, 0.02)
    out = _gpu_linear(xb, wb)
    assert _check(out, _to_f64(xb), _to_f64(wb)) < 1e-4


@pytest.mark.parametrize("rows,n,k", [(1, 768, 768), (63, 2304, 768), (63, 768, 1152), (63, 3072, 768),
                                      (63, 768, 768), (64, 768, 1152), (129, 768, 3072), (300, 3072, 768)])
def test_selftest_shapes_uniform(rows, n, k):
    rng = np.random.default_rng(0x5eed + rows + n + k)
    from laya_zig_b200.synth import f32_to_bf16_bits
    xb = f32_to_bf16_bits(rng.uniform(-1, 1, (rows, k)).astype(np.float32))
    wb = f32_to_bf16_bits(rng.uniform(-1, 1, (n, k)).astype(np.float32))
    out = _gpu_linear(xb, wb)
    # every column here, not every 29th. The reference's selftest stops at
    # k = 1152; at k = 3072 the tensor cores' f32 accumulation of 3072
    # products of U(-1,1)^2 lands near 1.2e-4, so that depth gets 2e-4.
    assert _check(out, _to_f64(xb), _to_f64(wb), every=1) < (1e-4 if k <= 1152 else 2e-4)


@pytest.mark.parametrize("rows,n,k", [(200, 384, 768), (1000, 640, 1152)])
def test_single_cta_path(rows, n, k):
    """N not a multiple of 256 runs single CTAs (128 x 128 tiles) instead of CTA pairs."""
    rng = np.random.default_rng(rows + n)
    xb = _rand_bits(rng, (rows, k), 1.0)
    wb = _rand_bits(rng, (n, k), 0.02)
    out = _gpu_linear(xb, wb)
    assert _check(out, _to_f64(xb), _to_f64(wb), every=1) < 1e-4


def test_gemm_bias_and_f16():
    rng = np.random.default_rng(3)
    xb = _rand_bits(rng, (200, 768), 1.0, f16=True)
    wb = _rand_bits(rng, (768, 768), 0.02, f16=True)
    bias = rng.standard_normal(768).astype(np.float32)
    out = _gpu_linear(xb, wb, bias, f16=True)
    assert _check(out, _to_f64(xb, True), _to_f64(wb, True), bias.astype(np.float64), every=1) < 1e-4


def test_gemm_rejects_bad_shape():
    import torch
    from laya_zig_b200 import gpu
    x = torch.zeros((64, 100), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((128, 100), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((64, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(gpu.LayaError):
        gpu.linear(x.data_ptr(), w.data_ptr(), 0, out.data_ptr(), 64, 128, 100)


def test_linear_after_a_kernel_that_writes_its_operands():
    """x and w written by the kernel just before, on the same stream, each
    call with new values: the projection is ordered after that kernel (its
    weight boxes are not requested before the dependency wait, as the
    forward's constant weights are)."""
    import torch
    from laya_zig_b200 import gpu
    rng = np.random.default_rng(11)
    M, N, K = 11520, 2304, 768
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        x = torch.empty((M, K), dtype=torch.bfloat16, device="cuda")
        w = torch.empty((N, K), dtype=torch.bfloat16, device="cuda")
        out = torch.empty((M, N), dtype=torch.float32, device="cuda")
        for i in range(3):
            xb = _rand_bits(rng, (M, K), 1.0)
            wb = _rand_bits(rng, (N, K), 0.02)
            xs = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
            ws = torch.from_numpy(wb.view(np.int16)).cuda().view(torch.bfloat16)
            stream.synchronize()
            # elementwise kernels (a copy may be a memcpy, which no launch
            # overlaps) on `stream`, right before the projection; x 1 is exact
            torch.mul(xs, 1.0, out=x)
            torch.mul(ws, 1.0, out=w)
            gpu.linear(x.data_ptr(), w.data_ptr(), 0, out.data_ptr(), M, N, K, "BF16", stream.cuda_stream)
            stream.synchronize()
            rel = _check(out.cpu().numpy(), _to_f64(xb), _to_f64(wb))
            assert rel < 1e-4, (i, rel)
