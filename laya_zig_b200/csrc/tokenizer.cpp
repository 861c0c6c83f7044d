// tokenizer.cpp -- host-side tokenizer and sequence builder (C ABI in
// include/laya_tok.h).
//
// Byte-for-byte the reference's algorithm (src/main.zig of laya-zig):
//   loading   walkValue / parseVocab / parseMerges / parseAdded (1717-1873):
//             the "vocab", "merges" and "added_tokens" keys wherever they
//             appear in tokenizer.json, object keys longer than 128 raw bytes
//             skipped, JSON escapes decoded (surrogate pairs joined), merges
//             keyed a NUL b and ranked by position, the first copy of a key
//             kept; finishTokenizer (2000-2043): added-token lengths longest
//             first, the bytes that can start one, byte-fallback ids of
//             "<0xHH>" (3 when absent).
//   encoding  encodeAll (2197-2217): longest added token wherever one
//             starts, the plain text between them through encodeSegment
//             (2162-2195): ' ' -> U+2581, a U+2581 put before the first word,
//             pieces from one U+2581 to the next; bpePiece (2111-2156): UTF-8
//             characters merged by lowest merge rank (leftmost on a tie) until
//             no pair merges, then vocab ids or the bytes' fallback ids.
//   building  replaceMask / buildSequence (2820-2911), qtypeId (2914-2919).
// The tables are open-addressing hash maps over one byte pool, as the
// reference keeps them; a batch of decisions is built on a pool of host
// threads, each decision independently, then packed in order.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <cstdlib>
#include <thread>
#include <vector>

#include "laya_tok.h"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

constexpr uint32_t CLS_ID = LAYA_TOK_CLS_ID, SEP_ID = LAYA_TOK_SEP_ID, MASK_ID = LAYA_TOK_MASK_ID;
constexpr char SEP_CHAR[] = "\xE2\x96\x81";  // U+2581
constexpr size_t SEP_LEN = 3;
constexpr char MASK_TOKEN[] = "<mask>";
constexpr size_t MASK_LEN = 6;

// Open-addressing map from byte strings (kept in one pool) to u32. The first
// put of a key wins, as a lookup in the reference's maps finds its first copy.
class StrMap {
  public:
    bool get(const char* p, size_t n, uint32_t* v) const {
        if (hash_.empty()) return false;
        const uint64_t h = hash_of(p, n);
        const size_t mask = hash_.size() - 1;
        for (size_t i = h & mask; hash_[i]; i = (i + 1) & mask)
            if (hash_[i] == h && len_[i] == n && memcmp(pool_.data() + off_[i], p, n) == 0) {
                if (v) *v = val_[i];
                return true;
            }
        return false;
    }
    void put(const char* p, size_t n, uint32_t v) {
        if (get(p, n, nullptr)) return;
        if (hash_.empty() || (uint64_t)(live_ + 1) * 10 >= (uint64_t)hash_.size() * 7) grow();
        const uint64_t h = hash_of(p, n);
        const size_t mask = hash_.size() - 1;
        size_t i = h & mask;
        while (hash_[i]) i = (i + 1) & mask;
        hash_[i] = h;
        off_[i] = (uint32_t)pool_.size();
        len_[i] = (uint32_t)n;
        val_[i] = v;
        pool_.append(p, n);
        live_++;
    }
    uint32_t size() const { return live_; }
    template <typename F>
    void each(F f) const {
        for (size_t i = 0; i < hash_.size(); i++)
            if (hash_[i]) f(pool_.data() + off_[i], (size_t)len_[i], val_[i]);
    }

  private:
    // 8 bytes at a time, multiply-xorshift, then a 64-bit finaliser; never 0.
    static uint64_t hash_of(const char* p, size_t n) {
        uint64_t h = 0x243F6A8885A308D3ull ^ (n * 0x9E3779B97F4A7C15ull);
        size_t i = 0;
        for (; i + 8 <= n; i += 8) {
            uint64_t w;
            memcpy(&w, p + i, 8);
            h = (h ^ w) * 0xBF58476D1CE4E5B9ull;
            h ^= h >> 31;
        }
        uint64_t w = 0;
        for (size_t k = 0; i + k < n; k++) w |= (uint64_t)(uint8_t)p[i + k] << (8 * k);
        h = (h ^ w) * 0x94D049BB133111EBull;
        h ^= h >> 29;
        h *= 0xBF58476D1CE4E5B9ull;
        h ^= h >> 32;
        return h | 1;
    }
    void grow() {
        const size_t n = hash_.empty() ? (size_t)1 << 12 : hash_.size() * 2;
        std::vector<uint64_t> h(n, 0);
        std::vector<uint32_t> o(n), l(n), v(n);
        for (size_t i = 0; i < hash_.size(); i++) {
            if (!hash_[i]) continue;
            size_t j = hash_[i] & (n - 1);
            while (h[j]) j = (j + 1) & (n - 1);
            h[j] = hash_[i];
            o[j] = off_[i];
            l[j] = len_[i];
            v[j] = val_[i];
        }
        hash_.swap(h);
        off_.swap(o);
        len_.swap(l);
        val_.swap(v);
    }
    std::vector<uint64_t> hash_;
    std::vector<uint32_t> off_, len_, val_;
    std::string pool_;
    uint32_t live_ = 0;
};

struct ParseError {
    const char* what;
    size_t at;
};

// JScan (main.zig:1383-1535) over the file's bytes.
class Scan {
  public:
    Scan(const char* s, size_t n) : s_(s), n_(n) {}
    size_t pos() const { return i_; }
    void ws() {
        while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) i_++;
    }
    char peek() const {
        if (i_ >= n_) throw ParseError{"truncated json", i_};
        return s_[i_];
    }
    char byte() {
        const char c = peek();
        i_++;
        return c;
    }
    void expect(char c) {
        ws();
        if (byte() != c) throw ParseError{"bad json", i_ - 1};
    }
    void skip_lit() {
        ws();
        while (i_ < n_ && !strchr(",}] \n\r\t", s_[i_])) i_++;
    }
    size_t raw_len() const {  // rawStringLen: escapes count two bytes
        size_t i = i_ + 1, n = 0;
        while (i < n_) {
            if (s_[i] == '"') return n;
            if (s_[i] == '\\') {
                i += 2;
                n += 2;
                continue;
            }
            i++;
            n++;
        }
        throw ParseError{"truncated json", i};
    }
    uint32_t uint() {
        ws();
        uint32_t v = 0;
        bool any = false;
        while (i_ < n_ && s_[i_] >= '0' && s_[i_] <= '9') {
            v = v * 10u + (uint32_t)(s_[i_] - '0');
            any = true;
            i_++;
        }
        if (!any) throw ParseError{"bad json number", i_};
        return v;
    }
    // The string at the cursor into `out` (decoded).
    void string(std::string& out) {
        expect('"');
        out.clear();
        // fast path: no escape before the closing quote
        const char* q = static_cast<const char*>(memchr(s_ + i_, '"', n_ - i_));
        if (!q) throw ParseError{"truncated json", i_};
        if (!memchr(s_ + i_, '\\', (size_t)(q - (s_ + i_)))) {
            out.assign(s_ + i_, (size_t)(q - (s_ + i_)));
            i_ = (size_t)(q - s_) + 1;
            return;
        }
        while (true) {
            const char c = byte();
            if (c == '"') return;
            if (c != '\\') {
                out.push_back(c);
                continue;
            }
            const char e = byte();
            switch (e) {
                case 'n': out.push_back('\n'); break;
                case 't': out.push_back('\t'); break;
                case 'r': out.push_back('\r'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case '/': case '"': case '\\': out.push_back(e); break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00) {
                        expect('\\');
                        if (byte() != 'u') throw ParseError{"bad json", i_ - 1};
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(cp, out);
                    break;
                }
                default: throw ParseError{"bad json escape", i_ - 1};
            }
        }
    }

  private:
    uint32_t hex4() {
        uint32_t v = 0;
        for (int k = 0; k < 4; k++) {
            const char c = byte();
            uint32_t d;
            if (c >= '0' && c <= '9') d = (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') d = (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') d = (uint32_t)(c - 'A' + 10);
            else throw ParseError{"bad json hex", i_ - 1};
            v = (v << 4) | d;
        }
        return v;
    }
    // encodeUtf8 (main.zig:1537-1562): surrogate halves come out as 3 bytes
    static void utf8(uint32_t cp, std::string& o) {
        if (cp < 0x80) {
            o.push_back((char)cp);
        } else if (cp < 0x800) {
            o.push_back((char)(0xC0 | (cp >> 6)));
            o.push_back((char)(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            o.push_back((char)(0xE0 | (cp >> 12)));
            o.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            o.push_back((char)(0x80 | (cp & 0x3F)));
        } else {
            o.push_back((char)(0xF0 | (cp >> 18)));
            o.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
            o.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            o.push_back((char)(0x80 | (cp & 0x3F)));
        }
    }
    const char* s_;
    size_t n_;
    size_t i_ = 0;
};

inline size_t utf8_len(uint8_t b) {  // utf8ByteSequenceLength, 1 for an invalid lead byte
    if (b < 0x80) return 1;
    if (b >= 0xC0 && b < 0xE0) return 2;
    if (b >= 0xE0 && b < 0xF0) return 3;
    if (b >= 0xF0 && b < 0xF8) return 4;
    return 1;
}

inline bool sep_at(const std::string& t, size_t i) {
    return i + SEP_LEN <= t.size() && memcmp(t.data() + i, SEP_CHAR, SEP_LEN) == 0;
}

}  // namespace

struct laya_tok {
    StrMap vocab, merges, added;
    uint64_t serial = 0;  // unique per loaded tokenizer: keys the per-thread piece cache
    std::vector<size_t> added_lens;  // distinct, longest first
    bool start_byte[256] = {};
    uint32_t byte_ids[256] = {};

    void walk(Scan& sc, std::string& s);
    void parse_vocab(Scan& sc, std::string& s);
    void parse_merges(Scan& sc, std::string& s);
    void parse_added(Scan& sc, std::string& s);
    void finish();

    void bpe_piece(const char* p, size_t n, std::vector<uint32_t>& out) const;
    void encode_segment(const char* s, size_t n, std::vector<uint32_t>& out) const;
    void encode(const char* text, size_t n, std::vector<uint32_t>& out) const;
};

void laya_tok::walk(Scan& sc, std::string& s) {  // walkValue (main.zig:1717-1771)
    sc.ws();
    const char c = sc.peek();
    if (c == '{') {
        sc.byte();
        while (true) {
            sc.ws();
            if (sc.peek() == '}') {
                sc.byte();
                return;
            }
            if (sc.peek() == ',') {
                sc.byte();
                continue;
            }
            if (sc.raw_len() > 128) {  // too long to be a key of interest
                sc.string(s);
                sc.expect(':');
                walk(sc, s);
                continue;
            }
            sc.string(s);
            sc.expect(':');
            if (s == "vocab") parse_vocab(sc, s);
            else if (s == "merges") parse_merges(sc, s);
            else if (s == "added_tokens") parse_added(sc, s);
            else walk(sc, s);
        }
    } else if (c == '[') {
        sc.byte();
        while (true) {
            sc.ws();
            if (sc.peek() == ']') {
                sc.byte();
                return;
            }
            if (sc.peek() == ',') {
                sc.byte();
                continue;
            }
            walk(sc, s);
        }
    } else if (c == '"') {
        sc.string(s);
    } else {
        sc.skip_lit();
    }
}

void laya_tok::parse_vocab(Scan& sc, std::string& s) {  // parseVocab (main.zig:1773-1795)
    sc.expect('{');
    while (true) {
        sc.ws();
        if (sc.peek() == '}') {
            sc.byte();
            return;
        }
        if (sc.peek() == ',') {
            sc.byte();
            continue;
        }
        sc.string(s);
        sc.expect(':');
        vocab.put(s.data(), s.size(), sc.uint());
    }
}

void laya_tok::parse_merges(Scan& sc, std::string& s) {  // parseMerges (main.zig:1797-1824)
    sc.expect('[');
    uint32_t rank = 0;
    std::string b;
    while (true) {
        sc.ws();
        if (sc.peek() == ']') {
            sc.byte();
            return;
        }
        if (sc.peek() == ',') {
            sc.byte();
            continue;
        }
        sc.expect('[');
        sc.string(s);
        sc.ws();
        sc.byte();  // ','
        sc.string(b);
        sc.expect(']');
        s.push_back('\0');
        s += b;
        merges.put(s.data(), s.size(), rank);
        rank++;
    }
}

void laya_tok::parse_added(Scan& sc, std::string& s) {  // parseAdded (main.zig:1826-1873)
    sc.expect('[');
    std::string content;
    while (true) {
        sc.ws();
        if (sc.peek() == ']') {
            sc.byte();
            return;
        }
        if (sc.peek() == ',') {
            sc.byte();
            continue;
        }
        sc.expect('{');
        uint32_t id = 0;
        bool have = false;
        while (true) {
            sc.ws();
            if (sc.peek() == '}') {
                sc.byte();
                break;
            }
            if (sc.peek() == ',') {
                sc.byte();
                continue;
            }
            sc.string(s);
            sc.expect(':');
            if (s == "id") {
                id = sc.uint();
            } else if (s == "content") {
                sc.string(content);
                have = true;
            } else if (sc.peek() == '"') {
                sc.string(s);
            } else {
                sc.skip_lit();
            }
        }
        if (have) added.put(content.data(), content.size(), id);
    }
}

void laya_tok::finish() {  // finishTokenizer (main.zig:2000-2043)
    added.each([&](const char* k, size_t n, uint32_t) {
        if (n == 0) return;
        if (std::find(added_lens.begin(), added_lens.end(), n) == added_lens.end()) added_lens.push_back(n);
        start_byte[(uint8_t)k[0]] = true;
    });
    std::sort(added_lens.begin(), added_lens.end(), [](size_t a, size_t b) { return a > b; });
    static const char hexdig[] = "0123456789ABCDEF";
    for (int b = 0; b < 256; b++) {
        const char key[6] = {'<', '0', 'x', hexdig[b >> 4], hexdig[b & 15], '>'};
        uint32_t v;
        byte_ids[b] = vocab.get(key, 6, &v) ? v : 3;
    }
}

namespace {

// Per-thread cache of BPE results, piece bytes -> ids. bpePiece is a pure
// function of the tokenizer's tables and the piece, and text repeats its
// words (a Snake board most of all), so a hit skips the merge loop; the ids
// are the same either way. Direct-mapped and allocation-free: PIECE_SLOTS
// slots (~0.9 MB per thread, allocated on the thread's first piece), each
// holding one piece of up to PIECE_BYTES bytes with its ids (at most
// PIECE_IDS), tagged with the serial of the tokenizer that produced it (not
// its address, which a later tokenizer may reuse); a colliding piece
// replaces the slot's. Thread-local, so the threads of laya_tok_build_batch
// need no lock.
constexpr size_t PIECE_BYTES = 32, PIECE_IDS = 16, PIECE_SLOTS = 1 << 13;
std::atomic<uint64_t> g_tok_serial{1};

struct PieceSlot {
    uint64_t owner;  // tokenizer serial, 0 = empty
    uint32_t len, n_ids;
    char bytes[PIECE_BYTES];
    uint32_t ids[PIECE_IDS];
};

struct PieceCache {
    PieceSlot* slots = nullptr;
    ~PieceCache() { free(slots); }
    PieceSlot* slot(const char* p, size_t n) {
        if (!slots) {
            slots = static_cast<PieceSlot*>(calloc(PIECE_SLOTS, sizeof(PieceSlot)));
            if (!slots) return nullptr;
        }
        uint64_t h = 1469598103934665603ull;  // FNV-1a
        for (size_t i = 0; i < n; i++) h = (h ^ (uint8_t)p[i]) * 1099511628211ull;
        return &slots[(h ^ (h >> 29)) & (PIECE_SLOTS - 1)];
    }
};
thread_local PieceCache t_piece_cache;

}  // namespace

void laya_tok::bpe_piece(const char* p, size_t n, std::vector<uint32_t>& out) const {  // main.zig:2111-2156
    if (n == 0) return;
    PieceSlot* slot = n <= PIECE_BYTES ? t_piece_cache.slot(p, n) : nullptr;
    if (slot && slot->owner == serial && slot->len == n && memcmp(slot->bytes, p, n) == 0) {
        out.insert(out.end(), slot->ids, slot->ids + slot->n_ids);
        return;
    }
    const size_t first_out = out.size();
    struct Sym {
        uint32_t a, b;  // [a, b) within the piece
    };
    std::vector<Sym> syms;
    syms.reserve(n);
    for (size_t i = 0; i < n;) {
        const size_t len = std::min(utf8_len((uint8_t)p[i]), n - i);
        syms.push_back({(uint32_t)i, (uint32_t)(i + len)});
        i += len;
    }
    // rank[s]: merge rank of the pair (s, s + 1), NONE if it is no merge.
    // A merge changes only the two pairs beside it, so each merge costs two
    // lookups and a scan of the ranks instead of a lookup per pair; the
    // pair merged is the same (lowest rank, leftmost on ties).
    constexpr uint32_t NONE = 0xFFFFFFFFu;
    char key[1024];
    auto pair_rank = [&](size_t s) -> uint32_t {
        const size_t la = syms[s].b - syms[s].a, lb = syms[s + 1].b - syms[s + 1].a;
        if (la + lb + 1 > sizeof key) return NONE;
        memcpy(key, p + syms[s].a, la);
        key[la] = 0;
        memcpy(key + la + 1, p + syms[s + 1].a, lb);
        uint32_t r;
        return merges.get(key, la + lb + 1, &r) ? r : NONE;
    };
    std::vector<uint32_t> rank(syms.size() - 1);
    for (size_t s = 0; s < rank.size(); s++) rank[s] = pair_rank(s);
    while (!rank.empty()) {
        size_t bi = 0;
        for (size_t s = 1; s < rank.size(); s++)
            if (rank[s] < rank[bi]) bi = s;
        if (rank[bi] == NONE) break;
        syms[bi].b = syms[bi + 1].b;
        syms.erase(syms.begin() + (long)bi + 1);
        rank.erase(rank.begin() + (long)bi);  // the old pair (bi + 1, bi + 2) is now (bi, bi + 1)
        if (bi < rank.size()) rank[bi] = pair_rank(bi);
        if (bi > 0) rank[bi - 1] = pair_rank(bi - 1);
    }
    for (const Sym& s : syms) {
        uint32_t id;
        if (vocab.get(p + s.a, s.b - s.a, &id)) {
            out.push_back(id);
        } else {
            for (uint32_t i = s.a; i < s.b; i++) out.push_back(byte_ids[(uint8_t)p[i]]);
        }
    }
    const size_t n_ids = out.size() - first_out;
    if (slot && n_ids <= PIECE_IDS) {
        slot->owner = serial;
        slot->len = (uint32_t)n;
        slot->n_ids = (uint32_t)n_ids;
        memcpy(slot->bytes, p, n);
        std::copy(out.begin() + (long)first_out, out.end(), slot->ids);
    }
}

void laya_tok::encode_segment(const char* s, size_t n, std::vector<uint32_t>& out) const {  // main.zig:2162-2195
    std::string t;
    t.reserve(n + SEP_LEN);
    for (size_t i = 0; i < n; i++) {
        if (s[i] == ' ') t.append(SEP_CHAR, SEP_LEN);
        else t.push_back(s[i]);
    }
    if (t.empty()) return;
    size_t j = 0;
    if (!sep_at(t, 0)) {
        while (j < t.size() && !sep_at(t, j)) j++;
        std::string first(SEP_CHAR, SEP_LEN);
        first.append(t, 0, j);
        bpe_piece(first.data(), first.size(), out);
    }
    while (j < t.size()) {
        size_t e = j + SEP_LEN;
        while (e < t.size() && !sep_at(t, e)) e++;
        bpe_piece(t.data() + j, e - j, out);
        j = e;
    }
}

void laya_tok::encode(const char* text, size_t n, std::vector<uint32_t>& out) const {  // main.zig:2197-2217
    size_t i = 0, plain = 0;
    while (i < n) {
        if (start_byte[(uint8_t)text[i]]) {
            bool hit = false;
            for (size_t len : added_lens) {  // findAdded: longest first
                uint32_t id;
                if (len <= n - i && added.get(text + i, len, &id)) {
                    if (i > plain) encode_segment(text + plain, i - plain, out);
                    out.push_back(id);
                    i += len;
                    plain = i;
                    hit = true;
                    break;
                }
            }
            if (hit) continue;
        }
        i++;
    }
    if (n > plain) encode_segment(text + plain, n - plain, out);
}

namespace {

std::string replace_mask(const char* s) {  // main.zig:2820-2834
    std::string out;
    const size_t n = strlen(s);
    out.reserve(n);
    for (size_t i = 0; i < n;) {
        if (i + MASK_LEN <= n && memcmp(s + i, MASK_TOKEN, MASK_LEN) == 0) {
            out.push_back(' ');
            i += MASK_LEN;
        } else {
            out.push_back(s[i++]);
        }
    }
    return out;
}

struct Built {
    std::vector<uint32_t> ids, markers;
    uint32_t qtype = 0;
    int status = LAYA_TOK_OK;
    std::string err;
};

int qtype_id(const char* name, uint32_t* q) {  // qtypeId (main.zig:2914-2919)
    if (!strcmp(name, "choice")) *q = 0;
    else if (!strcmp(name, "score")) *q = 1;
    else if (!strcmp(name, "noul")) *q = 2;
    else return LAYA_TOK_ERR_QTYPE;
    return LAYA_TOK_OK;
}

// buildSequence (main.zig:2842-2911)
void build_one(const laya_tok* tok, const laya_decision& d, uint32_t max_len, uint32_t head_max_len, Built& r) {
    if (!d.state || !d.qtype_name || !d.ins || (d.n_opts && !d.opts)) {
        r.status = LAYA_TOK_ERR_ARG;
        r.err = "decision with a NULL field";
        return;
    }
    if (qtype_id(d.qtype_name, &r.qtype)) {
        r.status = LAYA_TOK_ERR_QTYPE;
        r.err = std::string("question type \"") + d.qtype_name + "\" is not choice, score or noul";
        return;
    }
    std::vector<uint32_t> head;
    const std::string head_text = std::string(d.qtype_name) + " question: " + replace_mask(d.ins);
    tok->encode(head_text.data(), head_text.size(), head);
    std::vector<std::vector<uint32_t>> opts(d.n_opts);
    for (uint32_t k = 0; k < d.n_opts; k++) {
        if (!d.opts[k]) {
            r.status = LAYA_TOK_ERR_ARG;
            r.err = "NULL option text";
            return;
        }
        const std::string t = " " + replace_mask(d.opts[k]);
        std::vector<uint32_t> e;
        tok->encode(t.data(), t.size(), e);
        if (e.size() > LAYA_TOK_OPT_MAX) e.resize(LAYA_TOK_OPT_MAX);
        opts[k].reserve(e.size() + 1);
        opts[k].push_back(MASK_ID);
        opts[k].insert(opts[k].end(), e.begin(), e.end());
    }
    int64_t total = 0;
    for (const auto& o : opts) total += (int64_t)o.size();
    int64_t budget = (int64_t)head_max_len - total;
    if (budget < 16) {
        const size_t per = std::max<size_t>(4, (head_max_len - 16) / std::max<size_t>(1, opts.size()));
        for (auto& o : opts)
            if (o.size() > per) o.resize(per);
        total = 0;
        for (const auto& o : opts) total += (int64_t)o.size();
        budget = (int64_t)head_max_len - total;
    }
    const size_t head_keep = (size_t)std::max<int64_t>(8, std::max<int64_t>(budget, 0));
    if (head.size() > head_keep) head.resize(head_keep);

    std::vector<uint32_t>& ids = r.ids;
    ids.clear();
    ids.push_back(CLS_ID);
    ids.insert(ids.end(), head.begin(), head.end());
    ids.push_back(SEP_ID);
    std::vector<uint32_t> markers;
    for (const auto& o : opts) {
        markers.push_back((uint32_t)ids.size());
        ids.insert(ids.end(), o.begin(), o.end());
    }
    ids.push_back(SEP_ID);
    const int64_t room = (int64_t)max_len - (int64_t)ids.size() - 1;
    if (room > 0) {
        const std::string st = replace_mask(d.state);
        std::vector<uint32_t> sids;
        tok->encode(st.data(), st.size(), sids);
        if ((int64_t)sids.size() > room) sids.resize((size_t)room);
        ids.insert(ids.end(), sids.begin(), sids.end());
    }
    ids.push_back(SEP_ID);
    if (ids.size() > max_len) ids.resize(max_len);
    r.markers.clear();
    for (uint32_t m : markers)
        if (m < max_len) r.markers.push_back(m);
}

int check_lens(uint32_t max_len, uint32_t head_max_len) {
    if (max_len == 0) return fail(LAYA_TOK_ERR_ARG, "max_len is 0");
    if (head_max_len < 16) return fail(LAYA_TOK_ERR_ARG, "head_max_len %u is below 16", head_max_len);
    return LAYA_TOK_OK;
}

}  // namespace

extern "C" {

LAYA_TOK_API const char* laya_tok_last_error(void) { return g_err.c_str(); }

LAYA_TOK_API int laya_tok_load(const char* path, laya_tok** out) {
    if (!path || !out) return fail(LAYA_TOK_ERR_ARG, "NULL path or output");
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return fail(LAYA_TOK_ERR_IO, "cannot open %s", path);
    std::string data;
    if (fseek(f, 0, SEEK_END) == 0) {
        const long sz = ftell(f);
        if (sz > 0) data.resize((size_t)sz);
        rewind(f);
    }
    const size_t got = data.empty() ? 0 : fread(&data[0], 1, data.size(), f);
    fclose(f);
    if (got != data.size() || data.empty()) return fail(LAYA_TOK_ERR_IO, "cannot read %s", path);
    laya_tok* t = new laya_tok();
    try {
        Scan sc(data.data(), data.size());
        std::string scratch;
        t->walk(sc, scratch);
    } catch (const ParseError& e) {
        delete t;
        return fail(LAYA_TOK_ERR_PARSE, "%s: %s at byte %zu", path, e.what, e.at);
    } catch (const std::bad_alloc&) {
        delete t;
        return fail(LAYA_TOK_ERR_IO, "out of host memory reading %s", path);
    }
    t->finish();
    t->serial = g_tok_serial.fetch_add(1);
    *out = t;
    return LAYA_TOK_OK;
}

LAYA_TOK_API void laya_tok_destroy(laya_tok* tok) { delete tok; }

LAYA_TOK_API int laya_tok_sizes(const laya_tok* tok, uint32_t* vocab, uint32_t* merges, uint32_t* added) {
    if (!tok) return fail(LAYA_TOK_ERR_ARG, "tokenizer is NULL");
    if (vocab) *vocab = tok->vocab.size();
    if (merges) *merges = tok->merges.size();
    if (added) *added = tok->added.size();
    return LAYA_TOK_OK;
}

LAYA_TOK_API int laya_tok_encode(const laya_tok* tok, const char* text, size_t len, uint32_t* ids, size_t cap,
                                 size_t* n_out) {
    if (!tok || (!text && len) || !n_out || (cap && !ids)) return fail(LAYA_TOK_ERR_ARG, "NULL argument");
    std::vector<uint32_t> out;
    tok->encode(text, len, out);
    *n_out = out.size();
    std::copy(out.begin(), out.begin() + (long)std::min(cap, out.size()), ids);
    if (out.size() > cap) return fail(LAYA_TOK_ERR_CAPACITY, "%zu ids do not fit in %zu", out.size(), cap);
    return LAYA_TOK_OK;
}

LAYA_TOK_API int laya_tok_build(const laya_tok* tok, const laya_decision* d, uint32_t max_len, uint32_t head_max_len,
                                uint32_t* ids, uint32_t* L, uint32_t* markers, uint32_t* K, uint32_t* qtype) {
    if (!tok || !d || !ids || !L || !K || !qtype || (d->n_opts && !markers))
        return fail(LAYA_TOK_ERR_ARG, "NULL argument");
    int rc = check_lens(max_len, head_max_len);
    if (rc) return rc;
    Built b;
    build_one(tok, *d, max_len, head_max_len, b);
    if (b.status) return fail(b.status, "%s", b.err.c_str());
    std::copy(b.ids.begin(), b.ids.end(), ids);
    std::copy(b.markers.begin(), b.markers.end(), markers);
    *L = (uint32_t)b.ids.size();
    *K = (uint32_t)b.markers.size();
    *qtype = b.qtype;
    return LAYA_TOK_OK;
}

LAYA_TOK_API int laya_tok_build_batch(const laya_tok* tok, const laya_decision* d, uint32_t n, uint32_t max_len,
                                      uint32_t head_max_len, int threads, uint32_t* ids, size_t ids_cap,
                                      int32_t* cu_seqlens, uint32_t* markers, size_t markers_cap,
                                      int32_t* cu_markers, uint32_t* qtypes, size_t* n_tokens, size_t* n_markers) {
    if (!tok || (n && !d) || !cu_seqlens || !cu_markers || (n && !qtypes) || !n_tokens || !n_markers ||
        (ids_cap && !ids) || (markers_cap && !markers))
        return fail(LAYA_TOK_ERR_ARG, "NULL argument");
    int rc = check_lens(max_len, head_max_len);
    if (rc) return rc;
    std::vector<Built> out(n);
    int nt = threads > 0 ? threads : (int)std::min(8u, std::max(1u, std::thread::hardware_concurrency()));
    nt = (int)std::min<uint32_t>((uint32_t)nt, std::max(1u, n));
    std::atomic<uint32_t> next{0};
    auto work = [&]() {
        for (uint32_t i; (i = next.fetch_add(1)) < n;) {
            try {
                build_one(tok, d[i], max_len, head_max_len, out[i]);
            } catch (const std::bad_alloc&) {
                out[i].status = LAYA_TOK_ERR_CAPACITY;
                out[i].err = "out of host memory";
            }
        }
    };
    if (nt <= 1) {
        work();
    } else {
        std::vector<std::thread> pool;
        pool.reserve((size_t)nt - 1);
        for (int k = 1; k < nt; k++) pool.emplace_back(work);
        work();
        for (auto& th : pool) th.join();
    }
    size_t tokens = 0, mks = 0;
    for (uint32_t i = 0; i < n; i++) {
        if (out[i].status) return fail(out[i].status, "decision %u: %s", i, out[i].err.c_str());
        tokens += out[i].ids.size();
        mks += out[i].markers.size();
    }
    *n_tokens = tokens;
    *n_markers = mks;
    if (tokens > ids_cap || mks > markers_cap)
        return fail(LAYA_TOK_ERR_CAPACITY, "batch needs %zu ids and %zu markers (room for %zu and %zu)", tokens, mks,
                    ids_cap, markers_cap);
    size_t t = 0, g = 0;
    cu_seqlens[0] = 0;
    cu_markers[0] = 0;
    for (uint32_t i = 0; i < n; i++) {
        std::copy(out[i].ids.begin(), out[i].ids.end(), ids + t);
        std::copy(out[i].markers.begin(), out[i].markers.end(), markers + g);
        t += out[i].ids.size();
        g += out[i].markers.size();
        cu_seqlens[i + 1] = (int32_t)t;
        cu_markers[i + 1] = (int32_t)g;
        qtypes[i] = out[i].qtype;
    }
    return LAYA_TOK_OK;
}

}  // extern "C"
