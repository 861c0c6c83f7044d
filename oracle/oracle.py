"""ctypes wrapper for the CPU oracle (liblaya_oracle.so).

TEST INFRASTRUCTURE ONLY: tests/, the smoke check and bench.py's CPU
baseline leg use this module as the checker. The product path (the CUDA
library and laya_zig_b200) never imports it.

The oracle restates the reference forward, src/main.zig:2641-2817; see
laya_oracle.c for the per-function citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, Optional, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblaya_oracle.so")

F32, F16, BF16 = 0, 1, 2
_DT = {"F32": F32, "F16": F16, "BF16": BF16}
TAGS = ["emb"] + ["l%d" % i for i in range(22)] + ["final", "temb", "h0", "h1"]


class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int),
                ("data", ctypes.c_void_p), ("numel", ctypes.c_uint64)]


def build() -> None:
    """Compile liblaya_oracle.so with its Makefile (gcc, a second or two)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.lo_create.restype = ctypes.c_void_p
        L.lo_create.argtypes = [ctypes.POINTER(_Tensor), ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
        L.lo_destroy.argtypes = [ctypes.c_void_p]
        P = ctypes.c_void_p
        L.lo_forward.restype = ctypes.c_int
        L.lo_forward.argtypes = [P, P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P, P, P, P, P, P, ctypes.c_int]
        L.lo_linear16.argtypes = [P, P, P, ctypes.c_int, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        for f in ("lo_expv", "lo_geluv", "lo_gelu_n"):
            getattr(L, f).argtypes = [P, P, ctypes.c_int]
        L.lo_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


class OracleModel:
    """The reference model on the CPU. `tensors` maps name -> (dtype tag, array);
    arrays are kept alive for the life of the model (matrices are borrowed)."""

    def __init__(self, tensors: Dict[str, Tuple[str, np.ndarray]]):
        self._keep = []
        arr = (_Tensor * len(tensors))()
        for i, (name, (dt, a)) in enumerate(tensors.items()):
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            nb = name.encode()
            self._keep.append(nb)
            arr[i] = _Tensor(nb, _DT[dt], a.ctypes.data, a.size)
        err = ctypes.create_string_buffer(256)
        self._h = lib().lo_create(arr, len(tensors), err, 256)
        if not self._h:
            raise ValueError(err.value.decode())

    def close(self):
        if getattr(self, "_h", None):
            lib().lo_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward(self, ids, markers, qtype: int, threads: int = 0, want_hidden=False, want_stats=False,
                want_trace=False):
        """Returns dict(logits, act, pooled[, hidden][, stats][, trace])."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        markers = np.ascontiguousarray(markers, dtype=np.uint32)
        L, K = len(ids), len(markers)
        out = {"logits": np.zeros(K, np.float32), "act": np.zeros(2, np.float32), "pooled": np.zeros(768, np.float32)}
        hidden = np.zeros((L, 768), np.float32) if want_hidden else None
        st = np.zeros((len(TAGS), 5), np.float64) if want_stats else None
        tr = np.zeros((len(TAGS), L, 768), np.float32) if want_trace else None
        nt = threads or lib().lo_max_threads()
        rc = lib().lo_forward(self._h, _ptr(ids), L, int(qtype), _ptr(markers), K, _ptr(out["logits"]),
                              _ptr(out["act"]), _ptr(out["pooled"]), _ptr(hidden), _ptr(st), _ptr(tr), nt)
        if rc != 0:
            raise ValueError("oracle forward rejected its input (code %d)" % rc)
        if want_hidden:
            out["hidden"] = hidden
        if want_stats:
            out["stats"] = {t: st[i] for i, t in enumerate(TAGS)}
        if want_trace:
            out["trace"] = tr
        return out


def linear16(x: np.ndarray, w_bits: np.ndarray, wdtype: str = "BF16", bias=None, threads: int = 0) -> np.ndarray:
    """The reference's packed GEMM: out = x @ w.T, x f32 [rows,k], w 16-bit [n,k]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    rows, k = x.shape
    n = w.shape[0]
    out = np.zeros((rows, n), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().lo_linear16(_ptr(out), _ptr(x), _ptr(w), _DT[wdtype], _ptr(b), rows, n, k,
                      threads or lib().lo_max_threads())
    return out


def _vec(fn, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    getattr(lib(), fn)(_ptr(x), _ptr(out), x.size)
    return out


def expv(x):
    return _vec("lo_expv", x)


def geluv(x):
    return _vec("lo_geluv", x)


def gelu(x):
    return _vec("lo_gelu_n", x)


def model_from_bf16(weights: Dict[str, np.ndarray]) -> OracleModel:
    """OracleModel over synth.make_weights() output (bf16 bit patterns)."""
    return OracleModel({k: ("BF16", v) for k, v in weights.items()})
