"""Host tokenizer and sequence builder (csrc/tokenizer.cpp through the
laya_tok_* C ABI) against the oracle restatement (oracle/tokenizer.py) and the
reference's own golden ids (tests/golden/tokcheck.jsonl, a copy of the
reference's tools/tokcheck.jsonl).

The vocabulary tests need the model's tokenizer.json (256,000 entries,
580,604 merges), which this repository does not ship. They read it from
$LAYA_TOKENIZER_JSON, else from tokenizer/tokenizer.json of a laya-zig
checkout named by $LAYA_REFERENCE or lying beside this repository as
../reference, and are skipped where none exists. The synthetic vocabulary
tests need nothing."""
import json
import os

import numpy as np
import pytest

from conftest import ROOT

def _tokenizer_json() -> str:
    if os.environ.get("LAYA_TOKENIZER_JSON"):
        return os.environ["LAYA_TOKENIZER_JSON"]
    ref = os.environ.get("LAYA_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
    return os.path.join(ref, "tokenizer", "tokenizer.json")


REAL_JSON = _tokenizer_json()
needs_vocab = pytest.mark.skipif(not os.path.exists(REAL_JSON), reason="tokenizer.json not available")


@pytest.fixture(scope="module")
def tok():
    from laya_zig_b200 import tok as T
    t = T.Tokenizer(REAL_JSON)
    yield t
    t.close()


@pytest.fixture(scope="module")
def otok():
    from oracle.tokenizer import Tokenizer
    return Tokenizer(REAL_JSON)


def _goldens():
    with open(os.path.join(ROOT, "tests", "golden", "tokcheck.jsonl")) as f:
        return [json.loads(l) for l in f if l.strip()]


@needs_vocab
def test_tables_loaded(tok, otok):
    assert tok.sizes() == {"vocab": len(otok.vocab), "merges": len(otok.merges), "added": len(otok.added)}
    assert tok.sizes() == {"vocab": 256000, "merges": 580604, "added": 249}


@needs_vocab
def test_reference_goldens(tok, otok):
    """Every text of the reference's tokcheck.jsonl: the library and the
    oracle both give the golden ids."""
    g = _goldens()
    assert len(g) == 44
    for d in g:
        assert otok.encode(d["text"]) == d["ids"], d["text"]
        assert tok.encode(d["text"]) == d["ids"], d["text"]


def _random_texts(otok, n, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    pool = sorted(set("".join(d["text"] for d in _goldens())))
    words = [d["text"].split(" ") for d in _goldens()]
    words = [w for ws in words for w in ws if w]
    added = sorted(k.decode() for k in otok.added if k)
    out = []
    for _ in range(n):
        parts = []
        for _ in range(int(rng.integers(1, 12))):
            r = rng.random()
            if r < 0.45:
                parts.append(words[int(rng.integers(len(words)))])
            elif r < 0.7:
                parts.append("".join(pool[int(i)] for i in rng.integers(0, len(pool), int(rng.integers(1, 9)))))
            elif r < 0.8:
                parts.append(added[int(rng.integers(len(added)))])
            elif r < 0.9:
                parts.append(" " * int(rng.integers(1, 5)))
            else:
                parts.append(["\t", "\n", "\r\n", "  \n "][int(rng.integers(4))])
        sep = "" if rng.random() < 0.3 else " "
        out.append(sep.join(parts))
    return out


@needs_vocab
def test_random_texts_match_oracle(tok, otok):
    """Seeded mixes of words, characters from every script in the goldens,
    added tokens (inside and between words) and whitespace runs."""
    for t in _random_texts(otok, 400, seed=11):
        assert tok.encode(t) == otok.encode(t), repr(t)


@needs_vocab
def test_encode_edge_cases(tok, otok):
    cases = ["", " ", "  ", "▁", "▁▁ x", "<mask>", "<mask><mask>", "a<mask>b", " <mask> ",
             "\x00\x01\x7f", "\xff".encode("latin-1").decode("latin-1"), "x" * 300, "é" * 100,
             "<start_of_turn>user\nhi<end_of_turn>"]
    for t in cases:
        assert tok.encode(t) == otok.encode(t), repr(t)
    raw = b"\xff\xfe abc \xc3"  # invalid UTF-8 goes through byte fallback
    assert tok.encode(raw) == otok.encode(raw)


def _random_decisions(otok, n, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    texts = _random_texts(otok, 4 * n + 8, seed + 1)
    qn = ["choice", "score", "noul"]
    out = []
    for i in range(n):
        k = int(rng.integers(0, 12))
        long_opts = rng.random() < 0.3
        opts = [(texts[(i * 7 + j) % len(texts)] * (int(rng.integers(1, 8)) if long_opts else 1)) for j in range(k)]
        state = " ".join(texts[(i * 3 + j) % len(texts)] for j in range(int(rng.integers(0, 40))))
        ins = texts[i % len(texts)] + (" <mask> " if rng.random() < 0.5 else "")
        out.append((state, qn[i % 3], ins, opts))
    return out


@needs_vocab
@pytest.mark.parametrize("max_len,head_max_len", [(1024, 256), (96, 40), (40, 16), (1, 16)])
def test_build_matches_oracle(tok, otok, max_len, head_max_len):
    """buildSequence on seeded decisions, including the paths that cut
    options to the per-option budget, cut the head, fill the remaining room
    with state and drop markers past max_len."""
    from oracle.tokenizer import build_sequence
    for d in _random_decisions(otok, 60, seed=max_len):
        b = tok.build(*d, max_len=max_len, head_max_len=head_max_len)
        ids, mk, q = build_sequence(otok, *d, max_len=max_len, head_max_len=head_max_len)
        assert b.ids.tolist() == ids and b.markers.tolist() == mk and b.qtype == q


@needs_vocab
def test_build_batch_packs_like_single_builds(tok, otok):
    """The threaded batch builder packs exactly the single builds, for any
    thread count, in the layout LayaGPU.forward_device takes."""
    from laya_zig_b200 import gpu
    ds = _random_decisions(otok, 150, seed=5)
    singles = [tok.build(*d) for d in ds]
    ref = gpu.pack(singles)
    for threads in (1, 3, 8, 0):
        p = tok.build_batch(ds, threads=threads)
        for k in ("ids", "cu_seqlens", "cu_markers", "qtypes"):
            np.testing.assert_array_equal(p[k], ref[k], err_msg=k)
        np.testing.assert_array_equal(p["markers"], ref["markers"][:len(p["markers"])])


@needs_vocab
def test_snake_move_sequence(tok, otok):
    """The Snake move builder's call shape (main.zig:3083): 'choice', four
    moves, a board state."""
    from oracle.tokenizer import build_sequence
    board = "The board: " + " ".join(". " * 10 + "A" for _ in range(12))
    d = (board, "choice", "Which move keeps the snake alive? <mask>", ["up", "down", "left", "right"])
    b = tok.build(*d)
    ids, mk, q = build_sequence(otok, *d)
    assert b.ids.tolist() == ids and b.markers.tolist() == mk and q == 0
    assert b.ids[0] == 2 and all(b.ids[m] == 4 for m in b.markers)


@needs_vocab
def test_errors(tok, tmp_path):
    from laya_zig_b200 import tok as T
    with pytest.raises(T.BadQuestionType):
        tok.build("s", "rank", "i", ["a"])
    with pytest.raises(T.TokError) as e:
        tok.build("s", "choice", "i", ["a"], head_max_len=15)
    assert e.value.code == T.ERR_ARG
    with pytest.raises(T.TokError) as e:
        T.Tokenizer(str(tmp_path / "missing.json"))
    assert e.value.code == T.ERR_IO
    bad = tmp_path / "bad.json"
    bad.write_bytes(b'{"model": {"vocab": {"a": 1, "b": }}}')
    with pytest.raises(T.TokError) as e:
        T.Tokenizer(str(bad))
    assert e.value.code == T.ERR_PARSE
    trunc = tmp_path / "trunc.json"
    trunc.write_bytes(b'{"model": {"vocab": {"a": 1')
    with pytest.raises(T.TokError) as e:
        T.Tokenizer(str(trunc))
    assert e.value.code == T.ERR_PARSE


# ---------------------------------------------------------------- synthetic vocabulary
SYNTH = r'''{
  "version": "1.0",
  "added_tokens": [
    {"id": 900, "content": "<mask>", "single_word": false, "special": true},
    {"id": 901, "content": "<ma", "special": true},
    {"id": 902, "content": "éé", "special": false},
    {"id": 903, "content": "", "special": false},
    {"id": 904, "content": "<mask>", "special": true}
  ],
  "a_key_longer_than_one_hundred_and_twenty_eight_bytes_is_not_compared_with_vocab_merges_or_added_tokens_but_its_value_is_still_walked": {"vocab": {"zz": 50}},
  "normalizer": {"type": "Replace", "pattern": {"String": " "}, "content": "▁"},
  "model": {
    "type": "BPE", "byte_fallback": true,
    "vocab": {"▁": 10, "a": 11, "b": 12, "ab": 13, "▁a": 14, "▁ab": 15, "<0x41>": 16,
              "é": 17, "😀": 18, "c": 19, "bc": 20, "abc": 21, "\"q\"": 22, "x\ny": 23,
              "a": 99, "▁abc": 24, "\/": 25},
    "merges": [["a", "b"], ["b", "c"], ["▁", "a"], ["▁a", "b"], ["ab", "c"], ["a", "b"],
               ["▁", "ab"]]
  }
}'''


@pytest.fixture(scope="module")
def synth_paths(tmp_path_factory):
    p = tmp_path_factory.mktemp("tok") / "tokenizer.json"
    p.write_text(SYNTH)
    return str(p)


def test_synthetic_vocabulary(synth_paths):
    """Escapes and surrogate pairs, first copy of a key wins, longest added
    token wins, empty added token ignored, byte fallback present (<0x41>)
    and absent (3), merge ranks and a key nested under a long key."""
    from laya_zig_b200 import tok as T
    from oracle.tokenizer import Tokenizer
    t, o = T.Tokenizer(synth_paths), Tokenizer(synth_paths)
    assert t.sizes() == {"vocab": len(o.vocab), "merges": len(o.merges), "added": len(o.added)}
    assert o.vocab[b"a"] == 11 and o.vocab[b"zz"] == 50 and o.added[b"<mask>"] == 900
    # "ab" -> pieces [U+2581 a b]: (a,b) has rank 0 -> [U+2581, ab]; (U+2581, ab) rank 6 -> [U+2581ab]
    assert t.encode("ab") == [15]
    # "abc": (a,b) rank 0 first, then (U+2581, ab) rank 6 vs (ab, c) rank 4 -> ab+c first
    assert t.encode("abc") == o.encode("abc") == [10, 21]
    assert t.encode("A") == [10, 16]          # <0x41>
    assert t.encode("B") == [10, 3]           # no <0x42>: id 3
    assert t.encode("<mask>") == [900]        # longer of <mask> / <ma
    assert t.encode("<max") == [901, 10, 3]   # "<ma" then "x": U+2581 prefix, x unknown
    texts = ["ab", "abc", "a b c", "  ab", "ééé", "\U0001F600", "\"q\"", "x\ny", "/",
             "<mask>ab<ma", "abc abc", "B<mask>", "▁ab"]
    for s in texts:
        assert t.encode(s) == o.encode(s), repr(s)
    t.close()


def test_piece_cache_is_per_tokenizer(tmp_path):
    """The library caches BPE results per host thread; the entries belong to
    one loaded tokenizer. Two vocabularies that give the same pieces
    different ids, used in turn on the same thread, and a tokenizer loaded
    after another was destroyed (possibly at the same address), each give
    their own ids."""
    from laya_zig_b200 import tok as T
    from oracle.tokenizer import Tokenizer
    other = SYNTH.replace('"▁ab": 15', '"▁ab": 115').replace('"abc": 21', '"abc": 121').replace('"▁a": 14', '"▁a": 114')
    assert other != SYNTH
    pa, pb = tmp_path / "a.json", tmp_path / "b.json"
    pa.write_text(SYNTH)
    pb.write_text(other)
    texts = ["ab", "abc abc ab", "a b c", "ab<mask>ab", "éé ab"]
    oa, ob = Tokenizer(str(pa)), Tokenizer(str(pb))
    ta, tb = T.Tokenizer(str(pa)), T.Tokenizer(str(pb))
    for _ in range(3):
        for s in texts:
            assert ta.encode(s) == oa.encode(s), s
            assert tb.encode(s) == ob.encode(s), s
    assert ta.encode("ab") != tb.encode("ab")
    ta.close()
    tc = T.Tokenizer(str(pb))
    for s in texts:
        assert tc.encode(s) == ob.encode(s), s
    tb.close()
    ta2 = T.Tokenizer(str(pa))
    for s in texts:
        assert ta2.encode(s) == oa.encode(s), s
    tc.close()
    ta2.close()


@needs_vocab
def test_build_batch_packing_paths(tok):
    """build_batch lays the decision strings out in one buffer; bytes and
    str inputs mixed, decisions without options, and a string holding a NUL
    (the C side reads it up to the NUL, on the fallback path too) all pack
    exactly as single builds do."""
    from laya_zig_b200 import gpu
    ds = [("state one two", "choice", "pick <mask>", ["a", "b"]),
          (b"byte state", b"score", "ins <mask>", [b"x", "y", "z"]),
          ("no options here", "noul", "ins", []),
          ("tail state", "choice", "q <mask>", ["only"])]
    ref = gpu.pack([tok.build(*d) for d in ds])
    p = tok.build_batch(ds, threads=2)
    for k in ("ids", "cu_seqlens", "cu_markers", "qtypes"):
        np.testing.assert_array_equal(p[k], ref[k], err_msg=k)
    cut = [("state\x00hidden", "choice", "pick <mask>", ["a", "b\x00c"]), ds[0]]
    p = tok.build_batch(cut, threads=1)
    want = gpu.pack([tok.build("state", "choice", "pick <mask>", ["a", "b"]), tok.build(*ds[0])])
    for k in ("ids", "cu_seqlens", "cu_markers", "qtypes"):
        np.testing.assert_array_equal(p[k], want[k], err_msg=k)


@needs_vocab
def test_concurrent_callers_get_sequential_results(tok, otok):
    """A loaded tokenizer may be used from any number of threads (the BPE
    cache is per thread): four Python threads encoding and building at once
    (ctypes releases the GIL during the calls) get what one thread gets."""
    import threading
    texts = _random_texts(otok, 120, seed=23)
    decs = _random_decisions(otok, 40, seed=29)
    want_enc = [tok.encode(t) for t in texts]
    want_b = tok.build_batch(decs, threads=1)
    errors = []

    def worker(k):
        try:
            for r in range(3):
                for i in range(k, len(texts), 4):
                    assert tok.encode(texts[i]) == want_enc[i]
                got = tok.build_batch(decs, threads=1 + (k + r) % 3)
                for key in ("ids", "cu_seqlens", "markers", "cu_markers", "qtypes"):
                    np.testing.assert_array_equal(got[key], want_b[key])
        except Exception as e:  # reported on the main thread
            errors.append(repr(e))

    ths = [threading.Thread(target=worker, args=(k,)) for k in range(4)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    assert not errors, errors[:3]
