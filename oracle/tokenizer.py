"""CPU restatement of the reference tokenizer and sequence builder.

Test infrastructure only: tests use it as the checker for the C++ tokenizer
in laya_zig_b200/csrc/tokenizer.cpp; nothing in the product calls it.

Follows src/main.zig of li-ming1/laya-zig:
  - loadTokenizer / walkValue / parseVocab / parseMerges / parseAdded
    (2045-2109, 1717-1873): the "vocab", "merges" and "added_tokens" keys
    wherever they appear in tokenizer.json; merges are [a, b] pairs ranked
    by position; the first occurrence of a key wins.
  - finishTokenizer (2000-2043): added-token lengths longest first, the
    bytes that can start one, and the byte-fallback ids "<0xHH>" (3 when
    absent).
  - bpePiece (2111-2156), encodeSegment (2162-2195), encodeAll (2197-2217).
  - replaceMask / buildSequence (2820-2911) and qtypeId (2914-2919).
Pinned against the reference's own tools/tokcheck.jsonl (44 texts), kept as
tests/golden/tokcheck.jsonl.
"""
from __future__ import annotations

import json
from typing import Dict, List, Optional, Sequence, Tuple

SEP_CHAR = "▁".encode()  # main.zig:57
MASK_TOKEN = b"<mask>"        # main.zig:56
CLS_ID, SEP_ID, MASK_ID = 2, 1, 4  # main.zig:53-55
MAX_LEN, HEAD_MAX_LEN = 1024, 256  # main.zig:50-51
QTYPES = {b"choice": 0, b"score": 1, b"noul": 2}  # main.zig:2914-2919


def _utf8_len(b: int) -> int:
    """std.unicode.utf8ByteSequenceLength, 1 for an invalid lead byte."""
    if b < 0x80:
        return 1
    if 0xC0 <= b < 0xE0:
        return 2
    if 0xE0 <= b < 0xF0:
        return 3
    if 0xF0 <= b < 0xF8:
        return 4
    return 1


class _Scan:
    """JScan (main.zig:1383-1535) over the raw bytes of tokenizer.json."""

    def __init__(self, s: bytes):
        self.s, self.i = s, 0

    def ws(self):
        while self.i < len(self.s) and self.s[self.i] in b" \n\r\t":
            self.i += 1

    def peek(self) -> int:
        if self.i >= len(self.s):
            raise ValueError("truncated json")
        return self.s[self.i]

    def byte(self) -> int:
        c = self.peek()
        self.i += 1
        return c

    def expect(self, c: bytes):
        self.ws()
        if self.byte() != c[0]:
            raise ValueError("bad json at %d" % self.i)

    def skip_lit(self):
        self.ws()
        while self.i < len(self.s) and self.s[self.i] not in b",}] \n\r\t":
            self.i += 1

    def raw_len(self) -> int:
        i, n = self.i + 1, 0
        while i < len(self.s):
            c = self.s[i]
            if c == 0x22:
                return n
            if c == 0x5C:
                i += 2
                n += 2
                continue
            i += 1
            n += 1
        raise ValueError("truncated json")

    def hex4(self) -> int:
        v = 0
        for _ in range(4):
            v = (v << 4) | int(chr(self.byte()), 16)
        return v

    def string(self) -> bytes:
        self.expect(b'"')
        out = bytearray()
        while True:
            c = self.byte()
            if c == 0x22:
                return bytes(out)
            if c != 0x5C:
                out.append(c)
                continue
            e = chr(self.byte())
            if e in "ntrbf":
                out.append({"n": 10, "t": 9, "r": 13, "b": 8, "f": 12}[e])
            elif e in '/"\\':
                out.append(ord(e))
            elif e == "u":
                cp = self.hex4()
                if 0xD800 <= cp < 0xDC00:
                    self.expect(b"\\")
                    if self.byte() != ord("u"):
                        raise ValueError("bad json")
                    lo = self.hex4()
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00)
                out += _enc_utf8(cp)
            else:
                raise ValueError("bad json escape")

    def uint(self) -> int:
        self.ws()
        v, any_ = 0, False
        while self.i < len(self.s) and 0x30 <= self.s[self.i] <= 0x39:
            v = (v * 10 + self.s[self.i] - 0x30) & 0xFFFFFFFF
            any_ = True
            self.i += 1
        if not any_:
            raise ValueError("bad json number")
        return v


def _enc_utf8(cp: int) -> bytes:
    """encodeUtf8 (main.zig:1537-1562), surrogates included as 3 bytes."""
    if cp < 0x80:
        return bytes([cp])
    if cp < 0x800:
        return bytes([0xC0 | (cp >> 6), 0x80 | (cp & 0x3F)])
    if cp < 0x10000:
        return bytes([0xE0 | (cp >> 12), 0x80 | ((cp >> 6) & 0x3F), 0x80 | (cp & 0x3F)])
    return bytes([0xF0 | (cp >> 18), 0x80 | ((cp >> 12) & 0x3F), 0x80 | ((cp >> 6) & 0x3F), 0x80 | (cp & 0x3F)])


class Tokenizer:
    def __init__(self, path: Optional[str] = None, data: Optional[bytes] = None):
        if data is None:
            with open(path, "rb") as f:
                data = f.read()
        self.vocab: Dict[bytes, int] = {}
        self.merges: Dict[bytes, int] = {}  # key a + NUL + b, as BytePool.addPair
        self.added: Dict[bytes, int] = {}
        sc = _Scan(data)
        self._walk(sc)
        lens = []
        self.start_byte = [False] * 256
        for k in self.added:
            if not k:
                continue
            if len(k) not in lens:
                lens.append(len(k))
            self.start_byte[k[0]] = True
        self.added_lens = sorted(lens, reverse=True)
        self.byte_ids = [self.vocab.get(("<0x%02X>" % b).encode(), 3) for b in range(256)]

    # walkValue (main.zig:1717-1771)
    def _walk(self, sc: _Scan):
        sc.ws()
        c = sc.peek()
        if c == ord("{"):
            sc.byte()
            while True:
                sc.ws()
                if sc.peek() == ord("}"):
                    sc.byte()
                    return
                if sc.peek() == ord(","):
                    sc.byte()
                    continue
                if sc.raw_len() > 128:
                    sc.string()
                    sc.expect(b":")
                    self._walk(sc)
                    continue
                key = sc.string()
                sc.expect(b":")
                if key == b"vocab":
                    self._vocab(sc)
                elif key == b"merges":
                    self._merges(sc)
                elif key == b"added_tokens":
                    self._added(sc)
                else:
                    self._walk(sc)
        elif c == ord("["):
            sc.byte()
            while True:
                sc.ws()
                if sc.peek() == ord("]"):
                    sc.byte()
                    return
                if sc.peek() == ord(","):
                    sc.byte()
                    continue
                self._walk(sc)
        elif c == ord('"'):
            sc.string()
        else:
            sc.skip_lit()

    def _vocab(self, sc: _Scan):  # parseVocab (main.zig:1773-1795)
        sc.expect(b"{")
        while True:
            sc.ws()
            if sc.peek() == ord("}"):
                sc.byte()
                return
            if sc.peek() == ord(","):
                sc.byte()
                continue
            s = sc.string()
            sc.expect(b":")
            self.vocab.setdefault(s, sc.uint())

    def _merges(self, sc: _Scan):  # parseMerges (main.zig:1797-1824)
        sc.expect(b"[")
        rank = 0
        while True:
            sc.ws()
            if sc.peek() == ord("]"):
                sc.byte()
                return
            if sc.peek() == ord(","):
                sc.byte()
                continue
            sc.expect(b"[")
            a = sc.string()
            sc.ws()
            sc.byte()
            b = sc.string()
            sc.expect(b"]")
            self.merges.setdefault(a + b"\0" + b, rank)
            rank += 1

    def _added(self, sc: _Scan):  # parseAdded (main.zig:1826-1873)
        sc.expect(b"[")
        while True:
            sc.ws()
            if sc.peek() == ord("]"):
                sc.byte()
                return
            if sc.peek() == ord(","):
                sc.byte()
                continue
            sc.expect(b"{")
            ident, content = 0, None
            while True:
                sc.ws()
                if sc.peek() == ord("}"):
                    sc.byte()
                    break
                if sc.peek() == ord(","):
                    sc.byte()
                    continue
                key = sc.string()
                sc.expect(b":")
                if key == b"id":
                    ident = sc.uint()
                elif key == b"content":
                    content = sc.string()
                elif sc.peek() == ord('"'):
                    sc.string()
                else:
                    sc.skip_lit()
            if content is not None:
                self.added.setdefault(content, ident)

    # ---------------------------------------------------------------- encode
    def bpe_piece(self, piece: bytes, out: List[int]):  # main.zig:2111-2156
        if not piece:
            return
        syms, i = [], 0
        while i < len(piece):
            n = min(_utf8_len(piece[i]), len(piece) - i)
            syms.append(piece[i:i + n])
            i += n
        while len(syms) > 1:
            best, bi = None, 0
            for s in range(len(syms) - 1):
                a, b = syms[s], syms[s + 1]
                if len(a) + len(b) + 1 > 1024:
                    continue
                r = self.merges.get(a + b"\0" + b)
                if r is not None and (best is None or r < best):
                    best, bi = r, s
            if best is None:
                break
            syms[bi:bi + 2] = [syms[bi] + syms[bi + 1]]
        for s in syms:
            v = self.vocab.get(s)
            if v is not None:
                out.append(v)
            else:
                out.extend(self.byte_ids[c] for c in s)

    def encode_segment(self, s: bytes, out: List[int]):  # main.zig:2162-2195
        t = s.replace(b" ", SEP_CHAR)
        if not t:
            return
        j = 0
        if not t.startswith(SEP_CHAR):
            while j < len(t) and not t.startswith(SEP_CHAR, j):
                j += 1
            self.bpe_piece(SEP_CHAR + t[:j], out)
        while j < len(t):
            e = j + 3
            while e < len(t) and not t.startswith(SEP_CHAR, e):
                e += 1
            self.bpe_piece(t[j:e], out)
            j = e

    def find_added(self, s: bytes):
        for n in self.added_lens:
            if n <= len(s):
                v = self.added.get(s[:n])
                if v is not None:
                    return n, v
        return None

    def encode(self, text) -> List[int]:  # encodeAll, main.zig:2197-2217
        if isinstance(text, str):
            text = text.encode()
        out: List[int] = []
        i = plain = 0
        while i < len(text):
            if self.start_byte[text[i]]:
                m = self.find_added(text[i:])
                if m is not None:
                    if i > plain:
                        self.encode_segment(text[plain:i], out)
                    out.append(m[1])
                    i += m[0]
                    plain = i
                    continue
            i += 1
        if len(text) > plain:
            self.encode_segment(text[plain:], out)
        return out


def _b(s) -> bytes:
    return s.encode() if isinstance(s, str) else bytes(s)


def replace_mask(s: bytes) -> bytes:  # main.zig:2820-2834
    return s.replace(MASK_TOKEN, b" ")


def build_sequence(tok: Tokenizer, state, qtype_name, ins, opts: Sequence, max_len: int = MAX_LEN,
                   head_max_len: int = HEAD_MAX_LEN):
    """buildSequence (main.zig:2842-2911) -> (ids, markers, qtype)."""
    state, qtype_name, ins = _b(state), _b(qtype_name), _b(ins)
    if qtype_name not in QTYPES:
        raise ValueError("BadQuestionType")
    head_ids = tok.encode(qtype_name + b" question: " + replace_mask(ins))
    opt_ids = []
    for o in opts:
        e = tok.encode(b" " + replace_mask(_b(o)))[:48]
        opt_ids.append([MASK_ID] + e)
    total = sum(len(o) for o in opt_ids)
    budget = head_max_len - total
    if budget < 16:
        per = max(4, (head_max_len - 16) // max(1, len(opt_ids)))
        opt_ids = [o[:per] for o in opt_ids]
        total = sum(len(o) for o in opt_ids)
        budget = head_max_len - total
    head_keep = max(8, max(budget, 0))
    ids = [CLS_ID] + head_ids[:head_keep] + [SEP_ID]
    markers = []
    for o in opt_ids:
        markers.append(len(ids))
        ids += o
    ids.append(SEP_ID)
    room = max_len - len(ids) - 1
    if room > 0:
        ids += tok.encode(replace_mask(state))[:room]
    ids.append(SEP_ID)
    ids = ids[:max_len]
    return ids, [m for m in markers if m < max_len], QTYPES[qtype_name]
