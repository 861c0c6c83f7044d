"""Python host side of the Laya B200 forward pass: ctypes over liblaya_gpu.so.

Mirrors the reference's host interface for this path:

* ``LayaGPU(tensors, device)`` / ``LayaGPU.from_safetensors(path)`` is
  ``loadModel`` (src/main.zig:2311-2404): every tensor by its safetensors
  name; a missing one raises ``MissingTensor``, a wrong dtype
  ``UnsupportedDtype`` (the reference's error.MissingTensor /
  error.UnsupportedDtype, main.zig:1332, 1354).
* ``LayaGPU.forward(ids, qtype, markers)`` is ``forward(alloc, *FwdCtx)``
  (main.zig:2641-2817): it returns the option logits, the act/escalate pair
  and the pooled [CLS] state, and optionally the final hidden state that the
  reference leaves in ``f.s.x``.
* ``option_probs(logits, qtype, temperature)`` is the caller-side tempered
  softmax of main.zig:3799-3813.

There is no CPU fallback: if the CUDA library is missing this module raises
on import.
"""
from __future__ import annotations

import ctypes
import dataclasses
import os
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblaya_gpu.so")

D = 768
LAYA_OK, ERR_ARG, ERR_MISSING, ERR_DTYPE, ERR_SHAPE, ERR_OOM, ERR_CUDA, ERR_TIMEOUT, ERR_NODEV = 0, -1, -2, -3, -4, -5, -6, -7, -8
DT = {"F32": 0, "F16": 1, "BF16": 2}
PREC = {"bf16": 0, "f16": 1}
TRACE_TAGS = ["emb"] + ["l%d" % i for i in range(22)] + ["final", "temb", "h0", "h1"]


class LayaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__("%s (status %d)" % (msg, code))
        self.code = code


class MissingTensor(LayaError):
    pass


class UnsupportedDtype(LayaError):
    pass


def _error(code: int, msg: str) -> LayaError:
    if code == ERR_MISSING:
        return MissingTensor(code, msg)
    if code == ERR_DTYPE:
        return UnsupportedDtype(code, msg)
    return LayaError(code, msg)


class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("data", ctypes.c_void_p),
                ("numel", ctypes.c_uint64)]


class _Seq(ctypes.Structure):
    _fields_ = [("ids", ctypes.c_void_p), ("len", ctypes.c_uint32), ("markers", ctypes.c_void_p),
                ("n_markers", ctypes.c_uint32), ("qtype", ctypes.c_uint32)]


class _Batch(ctypes.Structure):
    _fields_ = [("ids", ctypes.c_void_p), ("cu_seqlens", ctypes.c_void_p), ("markers", ctypes.c_void_p),
                ("cu_markers", ctypes.c_void_p), ("qtypes", ctypes.c_void_p), ("n_seqs", ctypes.c_uint32),
                ("n_tokens", ctypes.c_uint32), ("n_markers", ctypes.c_uint32), ("max_len", ctypes.c_uint32)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError("liblaya_gpu.so is not built (%s); run `python -m laya_zig_b200.build`" % LIB_PATH)
    L = ctypes.CDLL(LIB_PATH)
    P, I, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32
    L.laya_gpu_version.restype = I
    L.laya_gpu_device_count.restype = I
    L.laya_gpu_create.argtypes = [I, ctypes.POINTER(_Tensor), I, I, ctypes.POINTER(P)]
    L.laya_gpu_create.restype = I
    L.laya_gpu_destroy.argtypes = [P]
    L.laya_gpu_last_error.argtypes = [P]
    L.laya_gpu_last_error.restype = ctypes.c_char_p
    L.laya_gpu_forward.argtypes = [P, P, U, U, P, U, P, P, P, P]
    L.laya_gpu_forward.restype = I
    L.laya_gpu_forward_batch.argtypes = [P, ctypes.POINTER(_Seq), U, P, P, P, P]
    L.laya_gpu_forward_batch.restype = I
    L.laya_gpu_forward_device.argtypes = [P, ctypes.POINTER(_Batch), P, P, P, P, P]
    L.laya_gpu_forward_device.restype = I
    L.laya_gpu_sync.argtypes = [P]
    L.laya_gpu_sync.restype = I
    L.laya_gpu_forward_trace.argtypes = [P, P, U, U, P, U, P, P, P]
    L.laya_gpu_forward_trace.restype = I
    L.laya_gpu_linear.argtypes = [P, P, P, P, I, I, I, I, P]
    L.laya_gpu_linear.restype = I
    L.laya_gpu_forward_profile.argtypes = [P, ctypes.POINTER(_Batch), P, P, I, P, P, P]
    L.laya_gpu_forward_profile.restype = I
    L.laya_gpu_forward_profile_launches.argtypes = [P, ctypes.POINTER(_Batch), P, P, I, P, P, P, I, P]
    L.laya_gpu_forward_profile_launches.restype = I
    L.laya_gpu_forward_dump.argtypes = [P, P, U, U, P, U, I, P, P, P, P, P, P]
    L.laya_gpu_forward_dump.restype = I
    L.laya_gpu_forward_dumpstats.argtypes = [P, P, U, U, P, U, P, P, ctypes.c_char_p, ctypes.c_uint64,
                                             ctypes.POINTER(ctypes.c_uint64)]
    L.laya_gpu_forward_dumpstats.restype = I
    L.laya_gpu_format_dump.argtypes = [P, U, U, P, U, P, P, ctypes.c_char_p, ctypes.c_uint64,
                                       ctypes.POINTER(ctypes.c_uint64)]
    L.laya_gpu_format_dump.restype = I
    L.laya_gpu_decision_tail_noalloc.argtypes = [P, P, P, P, P, U, U, P, P, P, P]
    L.laya_gpu_decision_tail_noalloc.restype = I
    return L


lib = _load()

STAGES = ["embed", "norm", "gemm_qkv", "attention", "gemm_out", "gemm_up", "gemm_down", "final", "tail"]


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a), dtype=np.uint32)


@dataclasses.dataclass
class Forward:
    """What `forward` leaves in its FwdCtx (src/main.zig:2529-2541)."""
    logits: np.ndarray            # [K] option logits
    act: np.ndarray               # [2] (act, escalate) probabilities
    pooled: np.ndarray            # [768] final hidden state of token 0
    hidden: Optional[np.ndarray] = None  # [L][768] final hidden state


def option_probs(logits: np.ndarray, qtype: int, temperature: Sequence[float] = (1.0, 1.0, 1.0)) -> np.ndarray:
    """softmax(logits / max(1e-3, temperature[qtype])) in f32 (src/main.zig:3799-3813)."""
    t = np.float32(max(1e-3, float(temperature[qtype])))
    p = np.asarray(logits, dtype=np.float32) / t
    p = np.exp(p - p.max())
    return (p / p.sum()).astype(np.float32)


class PreparedBatch:
    """Decisions marshalled once into the C call's laya_seq array, with
    output arrays, for callers that run the same host-buffer batch shape
    again and again (LayaGPU.forward_prepared). The token ids stay in the
    caller's host arrays: every call still copies them to the device and
    the results back."""

    def __init__(self, decisions):
        self.n = len(decisions)
        self.seqs = (_Seq * self.n)()
        self._keep = []
        G = 0
        for i, d in enumerate(decisions):
            ids, mk = _u32(d.ids), _u32(d.markers)
            self._keep += [ids, mk]
            self.seqs[i] = _Seq(ids.ctypes.data, len(ids), mk.ctypes.data if len(mk) else None, len(mk),
                                int(d.qtype))
            G += len(mk)
        self.logits = np.zeros(max(G, 1), np.float32)
        self.act = np.zeros((self.n, 2), np.float32)


class LayaGPU:
    """One model replica on one GPU (one context per device)."""

    def __init__(self, tensors: Dict[str, Tuple[str, np.ndarray]], device: int = 0, precision: str = "bf16"):
        arr = (_Tensor * len(tensors))()
        keep = []
        for i, (name, (dt, a)) in enumerate(tensors.items()):
            if dt not in DT:
                raise UnsupportedDtype(ERR_DTYPE, "tensor %s has dtype %s" % (name, dt))
            a = np.ascontiguousarray(a)
            nb = name.encode()
            keep += [a, nb]
            arr[i] = _Tensor(nb, DT[dt], a.ctypes.data, a.size)
        h = ctypes.c_void_p()
        rc = lib.laya_gpu_create(int(device), arr, len(tensors), PREC[precision], ctypes.byref(h))
        if rc != LAYA_OK:
            raise _error(rc, lib.laya_gpu_last_error(None).decode())
        self._h = h
        # kept on the instance: at interpreter exit the module's `lib` may be
        # cleared before a context that is still alive is collected
        self._destroy = lib.laya_gpu_destroy
        self.device = device
        self.precision = precision

    @classmethod
    def from_safetensors(cls, path: str, device: int = 0, precision: str = "bf16") -> "LayaGPU":
        from . import safetensors
        return cls(safetensors.read(path), device, precision)

    @classmethod
    def from_bf16(cls, weights: Dict[str, np.ndarray], device: int = 0, precision: str = "bf16") -> "LayaGPU":
        """Weights as bf16 bit patterns (what synth.make_weights returns)."""
        return cls({k: ("BF16", v) for k, v in weights.items()}, device, precision)

    def close(self):
        if getattr(self, "_h", None):
            self._destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def _check(self, rc: int):
        if rc != LAYA_OK:
            raise _error(rc, lib.laya_gpu_last_error(self._h).decode())

    def forward(self, ids, qtype: int, markers, want_hidden: bool = False) -> Forward:
        ids, markers = _u32(ids), _u32(markers)
        K, L = len(markers), len(ids)
        out = Forward(np.zeros(K, np.float32), np.zeros(2, np.float32), np.zeros(D, np.float32),
                      np.zeros((L, D), np.float32) if want_hidden else None)
        self._check(lib.laya_gpu_forward(self._h, _p(ids), L, int(qtype), _p(markers), K, _p(out.logits),
                                         _p(out.act), _p(out.pooled), _p(out.hidden)))
        return out

    def forward_batch(self, decisions, want_pooled: bool = False, want_hidden: bool = False) -> List[Forward]:
        """Independent sequences in one packed pass; `decisions` are objects
        with .ids, .markers, .qtype (e.g. synth.Decision)."""
        n = len(decisions)
        seqs = (_Seq * n)()
        keep = []
        G = T = 0
        for i, d in enumerate(decisions):
            ids, mk = _u32(d.ids), _u32(d.markers)
            keep += [ids, mk]
            seqs[i] = _Seq(ids.ctypes.data, len(ids), mk.ctypes.data if len(mk) else None, len(mk), int(d.qtype))
            G += len(mk)
            T += len(ids)
        logits = np.zeros(max(G, 1), np.float32)
        act = np.zeros((n, 2), np.float32)
        pooled = np.zeros((n, D), np.float32) if want_pooled else None
        hidden = np.zeros((T, D), np.float32) if want_hidden else None
        self._check(lib.laya_gpu_forward_batch(self._h, seqs, n, _p(logits), _p(act), _p(pooled), _p(hidden)))
        out, g, t = [], 0, 0
        for i, d in enumerate(decisions):
            K, L = len(d.markers), len(d.ids)
            out.append(Forward(logits[g:g + K].copy(), act[i].copy(), None if pooled is None else pooled[i],
                               None if hidden is None else hidden[t:t + L]))
            g += K
            t += L
        return out

    def forward_prepared(self, pb: PreparedBatch):
        """laya_gpu_forward_batch on a PreparedBatch: returns (logits of all
        markers in order, act[n][2]), the batch's own arrays, overwritten by
        the next call."""
        self._check(lib.laya_gpu_forward_batch(self._h, pb.seqs, pb.n, _p(pb.logits), _p(pb.act), None, None))
        return pb.logits, pb.act

    def forward_trace(self, ids, qtype: int, markers):
        """(logits, act, trace[27][L][768]) -- the hidden state after every
        --dumpstats stage (src/main.zig:2651-2753)."""
        ids, markers = _u32(ids), _u32(markers)
        K, L = len(markers), len(ids)
        logits, act = np.zeros(max(K, 1), np.float32), np.zeros(2, np.float32)
        trace = np.zeros((len(TRACE_TAGS), L, D), np.float32)
        self._check(lib.laya_gpu_forward_trace(self._h, _p(ids), L, int(qtype), _p(markers), K, _p(logits),
                                               _p(act), _p(trace)))
        return logits[:K], act, trace

    def forward_dumpstats(self, ids, qtype: int, markers):
        """(logits, act, text): forward() plus the `[dump]` lines the
        reference prints with --dumpstats (src/main.zig:113-130, 2651-2777),
        fingerprints computed on the device."""
        ids, markers = _u32(ids), _u32(markers)
        K, L = len(markers), len(ids)
        logits, act = np.zeros(max(K, 1), np.float32), np.zeros(2, np.float32)
        cap = 256 + 80 * (L // 8 + 1) + 96 * 27 + 24 * K
        need = ctypes.c_uint64(0)
        buf = ctypes.create_string_buffer(cap)
        self._check(lib.laya_gpu_forward_dumpstats(self._h, _p(ids), L, int(qtype), _p(markers), K, _p(logits),
                                                   _p(act), buf, cap, ctypes.byref(need)))
        return logits[:K], act, buf.value.decode()

    def forward_dump(self, ids, qtype: int, markers, layer: int):
        """Every intermediate of encoder layer `layer` as f32 arrays: xn_attn,
        qkv, ctx, x_mid, xn_mlp, glu (see laya_gpu_forward_dump)."""
        ids, markers = _u32(ids), _u32(markers)
        L, K = len(ids), len(markers)
        b16 = {"xn_attn": (L, D), "qkv": (L, 3 * D), "ctx": (L, D), "xn_mlp": (L, D), "glu": (L, 1152)}
        raw = {k: np.zeros(s, np.uint16) for k, s in b16.items()}
        x_mid = np.zeros((L, D), np.float32)
        self._check(lib.laya_gpu_forward_dump(self._h, _p(ids), L, int(qtype), _p(markers), K, int(layer),
                                              _p(raw["xn_attn"]), _p(raw["qkv"]), _p(raw["ctx"]), _p(x_mid),
                                              _p(raw["xn_mlp"]), _p(raw["glu"])))
        if self.precision == "f16":
            out = {k: v.view(np.float16).astype(np.float32) for k, v in raw.items()}
        else:
            out = {k: (v.astype(np.uint32) << np.uint32(16)).view(np.float32) for k, v in raw.items()}
        out["x_mid"] = x_mid
        return out

    def forward_device(self, batch: "DeviceBatch", logits_ptr: int, act_ptr: int, pooled_ptr: int = 0,
                       hidden_ptr: int = 0, stream: int = 0) -> None:
        """Asynchronous pass over a batch already in device memory (raw
        device pointers, e.g. torch tensors' data_ptr())."""
        self._check(lib.laya_gpu_forward_device(self._h, ctypes.byref(batch.c), logits_ptr or None, act_ptr or None,
                                                pooled_ptr or None, hidden_ptr or None, stream or None))

    def sync(self) -> None:
        self._check(lib.laya_gpu_sync(self._h))

    def decision_tail_noalloc(self, hidden_ptr: int, batch: "DeviceBatch", logits_ptr: int, act_ptr: int,
                              pooled_ptr: int, stream: int = 0) -> None:
        """Scorer + act head over device-resident final hidden states, for
        callers that cannot have the library allocate device memory: the
        scratch is a static device array (at most 2048 markers per call).
        Asynchronous on `stream`; calls that overlap on the GPU race."""
        b = batch.c
        self._check(lib.laya_gpu_decision_tail_noalloc(self._h, hidden_ptr, b.cu_seqlens, b.markers, b.cu_markers,
                                                       b.n_seqs, b.n_markers, logits_ptr or None, act_ptr,
                                                       pooled_ptr, stream or None))

    def profile(self, batch: "DeviceBatch", logits_ptr: int, act_ptr: int, iters: int = 1, stream: int = 0):
        """--profile (src/main.zig:132-198): ({stage: summed kernel ms}, {stage: launches per forward})
        over `iters` replays of a CUDA graph of one forward with an event pair
        around every kernel (the events stop neighbouring kernels from
        overlapping, so the times are upper bounds)."""
        ms = np.zeros(len(STAGES), np.float32)
        n = np.zeros(len(STAGES), np.int32)
        self._check(lib.laya_gpu_forward_profile(self._h, ctypes.byref(batch.c), logits_ptr or None, act_ptr or None,
                                                 int(iters), stream or None, _p(ms), _p(n)))
        return dict(zip(STAGES, ms.tolist())), dict(zip(STAGES, n.tolist()))


    def profile_launches(self, batch: "DeviceBatch", logits_ptr: int, act_ptr: int, iters: int = 1,
                         stream: int = 0):
        """[(stage, summed ms over `iters`)] for every launch of one forward,
        in launch order (the same event-pair capture as `profile`)."""
        cap = 512
        ms = np.zeros(cap, np.float32)
        st = np.zeros(cap, np.int32)
        n = ctypes.c_int(0)
        self._check(lib.laya_gpu_forward_profile_launches(self._h, ctypes.byref(batch.c), logits_ptr or None,
                                                          act_ptr or None, int(iters), stream or None, _p(ms), _p(st),
                                                          cap, ctypes.byref(n)))
        return [(STAGES[int(st[i])], float(ms[i])) for i in range(min(n.value, cap))]


class DeviceBatch:
    """Shape + device pointers of a packed batch for LayaGPU.forward_device."""

    def __init__(self, ids_ptr, cu_seqlens_ptr, markers_ptr, cu_markers_ptr, qtypes_ptr, n_seqs, n_tokens,
                 n_markers, max_len):
        self.c = _Batch(ids_ptr, cu_seqlens_ptr, markers_ptr, cu_markers_ptr, qtypes_ptr, n_seqs, n_tokens,
                        n_markers, max_len)


def pack(decisions) -> Dict[str, np.ndarray]:
    """Host arrays of a packed batch: ids, cu_seqlens, markers, cu_markers, qtypes."""
    lens = np.array([len(d.ids) for d in decisions], dtype=np.int32)
    ks = np.array([len(d.markers) for d in decisions], dtype=np.int32)
    return {
        "ids": np.concatenate([_u32(d.ids) for d in decisions]),
        "cu_seqlens": np.concatenate([[0], np.cumsum(lens)]).astype(np.int32),
        "markers": np.concatenate([_u32(d.markers) for d in decisions]) if ks.sum() else np.zeros(1, np.uint32),
        "cu_markers": np.concatenate([[0], np.cumsum(ks)]).astype(np.int32),
        "qtypes": np.array([d.qtype for d in decisions], dtype=np.uint32),
        "max_len": int(lens.max()),
    }


def format_dump(ids, qtype: int, markers, logits, stats) -> str:
    """The reference's `[dump]` text (src/main.zig:113-130) for given
    fingerprints stats[27][5] (x0, x1, x2, sum, abs-sum per tag), host only."""
    ids, markers = _u32(ids), _u32(markers)
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    st = np.ascontiguousarray(stats, dtype=np.float64)
    assert st.shape == (len(TRACE_TAGS), 5)
    cap = 256 + 80 * (len(ids) // 8 + 1) + 96 * 27 + 24 * len(markers)
    buf = ctypes.create_string_buffer(cap)
    rc = lib.laya_gpu_format_dump(_p(ids), len(ids), int(qtype), _p(markers), len(markers), _p(logits), _p(st), buf,
                                  cap, None)
    if rc != LAYA_OK:
        raise _error(rc, lib.laya_gpu_last_error(None).decode())
    return buf.value.decode()


def linear(x_ptr: int, w_ptr: int, bias_ptr: int, out_ptr: int, M: int, N: int, K: int, dtype: str = "BF16",
           stream: int = 0) -> None:
    """out[M][N] f32 = x[M][K] . w[N][K]^T (+ bias) on the current device; device pointers."""
    rc = lib.laya_gpu_linear(x_ptr, w_ptr, bias_ptr or None, out_ptr, M, N, K, DT[dtype], stream or None)
    if rc != LAYA_OK:
        raise _error(rc, lib.laya_gpu_last_error(None).decode())
