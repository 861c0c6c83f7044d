"""Every stage of an encoder layer on its own (laya_gpu_forward_dump).

For one sequence, laya_gpu_forward_dump returns what the GPU holds after each
stage of encoder layer l: xn_attn, qkv (RoPE applied), ctx (attention),
x_mid (after the attention residual), xn_mlp and glu. Each stage is
recomputed here in f64 numpy from the GPU's own input to that stage, so a
mismatch points at one kernel:

    xn_attn = LN(x_in; attn_norm)              (src/main.zig:83-95, 2660-2665)
    qkv     = rope(xn_attn Wqkv^T)             (2666-2671, 2496-2521)
    ctx     = softmax(q k^T / 8 | window) v    (2431-2489)
    x_mid   = x_in + ctx Wo^T                  (2686-2688)
    xn_mlp  = LN(x_mid; mlp_norm)              (2691)
    glu     = gelu(xn_mlp Wi_gate^T) * (xn_mlp Wi_up^T)   (2557-2569)

x_in is the trace point before the layer (laya_gpu_forward_trace). 16-bit
outputs are compared as max |d| / max |ref| per row within 1e-2 (their
rounding is 2^-9 relative in bf16); x_mid (f32) within 1e-3. Sequences of
150 tokens (windows cut on sliding layers) and 2,100 tokens (global layers
take the tcgen05 kernel from 2,048 tokens on, with a partial last key tile)
cover both attention kernels.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

D, HD, H = 768, 64, 12


def _f32(w):
    from laya_zig_b200.synth import bf16_bits_to_f32
    return bf16_bits_to_f32(w).astype(np.float64)


def _ln(x, w):
    m = x.mean(1, keepdims=True)
    v = ((x - m) ** 2).mean(1, keepdims=True)
    return (x - m) / np.sqrt(v + 1e-5) * w


def _rope_tables(L):
    inv = np.array([np.float32(1.0) / np.float32(np.power(np.float32(160000.0), np.float32(j / 32.0)))
                    for j in range(32)], np.float32)
    ang = (inv[None, :] * np.arange(L, dtype=np.float32)[:, None]).astype(np.float32)
    return np.cos(ang).astype(np.float64), np.sin(ang).astype(np.float64)


def _rope(x, cos, sin):
    x = x.reshape(len(x), H, HD).copy()
    a, b = x[:, :, :32].copy(), x[:, :, 32:].copy()
    x[:, :, :32] = a * cos[:, None, :] - b * sin[:, None, :]
    x[:, :, 32:] = b * cos[:, None, :] + a * sin[:, None, :]
    return x.reshape(len(x), D)


def _attention(qkv, window):
    L = len(qkv)
    q, k, v = (qkv[:, i * D:(i + 1) * D].reshape(L, H, HD) for i in range(3))
    out = np.zeros((L, H, HD))
    for h in range(H):
        s = q[:, h] @ k[:, h].T / 8.0
        if window is not None:
            i = np.arange(L)
            s[np.abs(i[:, None] - i[None, :]) > window] = -np.inf
        s -= s.max(1, keepdims=True)
        p = np.exp(s)
        out[:, h] = (p @ v[:, h]) / p.sum(1, keepdims=True)
    return out.reshape(L, D)


def _gelu(x):
    erf = np.vectorize(math.erf)
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def _rel(got, ref):
    return float((np.abs(got - ref).max(1) / np.maximum(np.abs(ref).max(1), 1e-30)).max())


@pytest.mark.parametrize("L,layer", [(150, 3), (150, 4), (2100, 3), (2100, 0)])
def test_layer_stages(gpu_model, weights, L, layer):
    from laya_zig_b200 import synth
    rng = np.random.Generator(np.random.PCG64(1000 + L))
    d = synth._decision(rng, L, [5, L // 2], 1)
    dump = gpu_model.forward_dump(d.ids, d.qtype, d.markers, layer)
    _, _, trace = gpu_model.forward_trace(d.ids, d.qtype, d.markers)
    x_in = trace[layer].astype(np.float64)  # tag `layer` is the state before encoder layer `layer`
    p = "encoder.layers.%d." % layer
    W = {n: _f32(weights[p + n]) for n in ("attn.Wqkv.weight", "attn.Wo.weight", "mlp.Wi.weight")}
    err = {}
    if layer > 0:
        err["xn_attn"] = _rel(dump["xn_attn"], _ln(x_in, _f32(weights[p + "attn_norm.weight"])))
    else:
        err["xn_attn"] = _rel(dump["xn_attn"], x_in)  # layer 0: attn_norm is the identity
    cos, sin = _rope_tables(L)
    qkv = dump["xn_attn"].astype(np.float64) @ W["attn.Wqkv.weight"].T
    qkv[:, :D] = _rope(qkv[:, :D], cos, sin)
    qkv[:, D:2 * D] = _rope(qkv[:, D:2 * D], cos, sin)
    err["qkv"] = _rel(dump["qkv"], qkv)
    ctx = _attention(dump["qkv"].astype(np.float64), None if layer % 3 == 0 else 64)
    err["ctx"] = _rel(dump["ctx"], ctx)
    x_mid = x_in + dump["ctx"].astype(np.float64) @ W["attn.Wo.weight"].T
    err["x_mid"] = _rel(dump["x_mid"], x_mid)
    xn_mlp = _ln(dump["x_mid"].astype(np.float64), _f32(weights[p + "mlp_norm.weight"]))
    err["xn_mlp"] = _rel(dump["xn_mlp"], xn_mlp)
    g = dump["xn_mlp"].astype(np.float64) @ W["mlp.Wi.weight"].T
    err["glu"] = _rel(dump["glu"], _gelu(g[:, :1152]) * g[:, 1152:])
    print("L=%d layer %d stage errors %s" % (L, layer, {k: "%.2e" % v for k, v in err.items()}))
    for k, v in err.items():
        assert v <= (1e-3 if k == "x_mid" else 1e-2), (k, v, err)
