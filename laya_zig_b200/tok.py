"""Python host side of the tokenizer and sequence builder: ctypes over the
laya_tok_* entry points of liblaya_gpu.so (include/laya_tok.h).

Mirrors the reference's host interface (src/main.zig of laya-zig):

* ``Tokenizer(path)`` is ``loadTokenizer`` (2045-2109) on a tokenizer.json.
* ``Tokenizer.encode(text)`` is ``encodeAll`` (2197-2217).
* ``Tokenizer.build(state, qtype_name, ins, opts)`` is ``buildSequence``
  (2842-2911) and returns a ``Decision``-like object (.ids, .markers,
  .qtype) that ``LayaGPU.forward_batch`` / ``pack`` accept.
* ``Tokenizer.build_batch(decisions, threads)`` builds many decisions on
  host threads straight into the packed layout of ``LayaGPU.forward_device``
  (ids, cu_seqlens, markers, cu_markers, qtypes).

Errors raise ``TokError`` with the library's message (``BadQuestionType`` for
an unknown question type, as the reference's error.BadQuestionType).
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Dict, List, Optional, Sequence

import numpy as np

from .gpu import lib

MAX_LEN, HEAD_MAX_LEN = 1024, 256
OK, ERR_ARG, ERR_IO, ERR_PARSE, ERR_QTYPE, ERR_CAPACITY = 0, -1, -2, -3, -4, -5


class TokError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__("%s (status %d)" % (msg, code))
        self.code = code


class BadQuestionType(TokError):
    pass


class _Decision(ctypes.Structure):
    _fields_ = [("state", ctypes.c_char_p), ("qtype_name", ctypes.c_char_p), ("ins", ctypes.c_char_p),
                ("opts", ctypes.POINTER(ctypes.c_char_p)), ("n_opts", ctypes.c_uint32)]


def _bind():
    P, I, U, Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t
    lib.laya_tok_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(P)]
    lib.laya_tok_load.restype = I
    lib.laya_tok_destroy.argtypes = [P]
    lib.laya_tok_last_error.restype = ctypes.c_char_p
    lib.laya_tok_sizes.argtypes = [P, P, P, P]
    lib.laya_tok_sizes.restype = I
    lib.laya_tok_encode.argtypes = [P, ctypes.c_char_p, Z, P, Z, ctypes.POINTER(Z)]
    lib.laya_tok_encode.restype = I
    lib.laya_tok_build.argtypes = [P, ctypes.POINTER(_Decision), U, U, P, P, P, P, P]
    lib.laya_tok_build.restype = I
    lib.laya_tok_build_batch.argtypes = [P, ctypes.POINTER(_Decision), U, U, U, I, P, Z, P, P, Z, P, P,
                                         ctypes.POINTER(Z), ctypes.POINTER(Z)]
    lib.laya_tok_build_batch.restype = I


_bind()


def _check(rc: int):
    if rc != OK:
        msg = lib.laya_tok_last_error().decode(errors="replace")
        raise (BadQuestionType if rc == ERR_QTYPE else TokError)(rc, msg)


def _b(s) -> bytes:
    return s.encode() if isinstance(s, str) else bytes(s)


@dataclasses.dataclass
class Built:
    """One built sequence: what buildSequence returns, plus its qtype id."""
    ids: np.ndarray
    markers: np.ndarray
    qtype: int


class _Marshalled:
    """ctypes laya_decision array with the byte strings it points at."""

    def __init__(self, decisions: Sequence):
        self.n = len(decisions)
        self.arr = (_Decision * self.n)()
        self._keep: List = []
        for i, d in enumerate(decisions):
            state, qn, ins, opts = d
            ob = [_b(o) for o in opts]
            oarr = (ctypes.c_char_p * max(1, len(ob)))(*ob) if ob else None
            self._keep += [_b(state), _b(qn), _b(ins), ob, oarr]
            self.arr[i] = _Decision(self._keep[-5], self._keep[-4], self._keep[-3],
                                    ctypes.cast(oarr, ctypes.POINTER(ctypes.c_char_p)) if oarr else None, len(ob))


class _Packed:
    """The laya_decision array for many decisions, built with a few C-level
    operations instead of one ctypes object per string: every string
    NUL-terminated in one buffer, the pointers computed from its NUL
    positions into a numpy array laid out as the C struct. A string that
    holds a NUL itself (which the C side would cut there anyway) makes
    `ok` false; the caller then uses _Marshalled."""

    _dtype = np.dtype({"names": ["state", "qtype_name", "ins", "opts", "n_opts"],
                       "formats": [np.uint64, np.uint64, np.uint64, np.uint64, np.uint32],
                       "offsets": [_Decision.state.offset, _Decision.qtype_name.offset, _Decision.ins.offset,
                                   _Decision.opts.offset, _Decision.n_opts.offset],
                       "itemsize": ctypes.sizeof(_Decision)})

    def __init__(self, decisions: Sequence):
        self.n = n = len(decisions)
        self.ok = False
        strs: List = []
        n_opts = np.empty(n, np.int64)
        for i, (state, qn, ins, opts) in enumerate(decisions):
            strs += (state, qn, ins)
            strs += opts
            n_opts[i] = len(opts)
        if all(isinstance(x, str) for x in strs):
            buf = ("\0".join(strs) + "\0").encode()
        else:
            buf = b"\0".join(_b(x) for x in strs) + b"\0"
        self._buf = np.frombuffer(buf, dtype=np.uint8).copy()
        ends = np.flatnonzero(self._buf == 0)
        if len(ends) != len(strs):
            return
        base = np.uint64(self._buf.ctypes.data)
        starts = np.concatenate([[0], ends[:-1] + 1]).astype(np.uint64) + base
        first = np.concatenate([[0], np.cumsum(3 + n_opts)[:-1]]).astype(np.int64)
        is_opt = np.ones(len(strs), dtype=bool)
        is_opt[first] = is_opt[first + 1] = is_opt[first + 2] = False
        self._opt_ptrs = np.ascontiguousarray(starts[is_opt], dtype=np.uint64)
        opt_first = np.concatenate([[0], np.cumsum(n_opts)[:-1]]).astype(np.uint64)
        self.arr = np.zeros(max(1, n), dtype=self._dtype)
        self.arr["state"][:n] = starts[first]
        self.arr["qtype_name"][:n] = starts[first + 1]
        self.arr["ins"][:n] = starts[first + 2]
        opts_ptr = np.uint64(self._opt_ptrs.ctypes.data) + opt_first * np.uint64(8)
        self.arr["opts"][:n] = np.where(n_opts > 0, opts_ptr, np.uint64(0))
        self.arr["n_opts"][:n] = n_opts
        self.ok = True

    def ptr(self):
        return self.arr.ctypes.data_as(ctypes.POINTER(_Decision))


class Tokenizer:
    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _check(lib.laya_tok_load(_b(path), ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib.laya_tok_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sizes(self) -> Dict[str, int]:
        v, m, a = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        _check(lib.laya_tok_sizes(self._h, ctypes.byref(v), ctypes.byref(m), ctypes.byref(a)))
        return {"vocab": v.value, "merges": m.value, "added": a.value}

    def encode(self, text) -> List[int]:
        t = _b(text)
        n = ctypes.c_size_t()
        cap = len(t) + 16
        out = np.zeros(cap, np.uint32)
        rc = lib.laya_tok_encode(self._h, t, len(t), out.ctypes.data, cap, ctypes.byref(n))
        if rc == ERR_CAPACITY:  # the library reports the count it needs
            cap = n.value
            out = np.zeros(cap, np.uint32)
            rc = lib.laya_tok_encode(self._h, t, len(t), out.ctypes.data, cap, ctypes.byref(n))
        _check(rc)
        return out[:n.value].tolist()

    def build(self, state, qtype_name, ins, opts: Sequence, max_len: int = MAX_LEN,
              head_max_len: int = HEAD_MAX_LEN) -> Built:
        m = _Marshalled([(state, qtype_name, ins, opts)])
        ids = np.zeros(max_len, np.uint32)
        mk = np.zeros(max(1, len(opts)), np.uint32)
        L, K, q = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        _check(lib.laya_tok_build(self._h, m.arr, max_len, head_max_len, ids.ctypes.data, ctypes.byref(L),
                                  mk.ctypes.data, ctypes.byref(K), ctypes.byref(q)))
        return Built(ids[:L.value].copy(), mk[:K.value].copy(), q.value)

    def build_batch(self, decisions: Sequence, threads: int = 0, max_len: int = MAX_LEN,
                    head_max_len: int = HEAD_MAX_LEN) -> Dict[str, np.ndarray]:
        """decisions: (state, qtype_name, ins, opts) tuples. Returns the packed
        arrays ids, cu_seqlens, markers, cu_markers, qtypes."""
        m = _Packed(decisions)
        if not m.ok:
            m = _Marshalled(decisions)
        arr = m.ptr() if isinstance(m, _Packed) else m.arr
        n = m.n
        ids_cap = n * max_len
        mk_cap = sum(len(d[3]) for d in decisions)
        ids = np.zeros(max(1, ids_cap), np.uint32)
        markers = np.zeros(max(1, mk_cap), np.uint32)
        cu = np.zeros(n + 1, np.int32)
        cum = np.zeros(n + 1, np.int32)
        qt = np.zeros(max(1, n), np.uint32)
        nt, nm = ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib.laya_tok_build_batch(self._h, arr, n, max_len, head_max_len, threads, ids.ctypes.data, ids_cap,
                                        cu.ctypes.data, markers.ctypes.data, mk_cap, cum.ctypes.data, qt.ctypes.data,
                                        ctypes.byref(nt), ctypes.byref(nm)))
        return {"ids": ids[:nt.value].copy(), "cu_seqlens": cu, "markers": markers[:nm.value].copy(),
                "cu_markers": cum, "qtypes": qt[:n].copy()}
