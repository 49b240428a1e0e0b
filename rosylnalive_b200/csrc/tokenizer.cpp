// tokenizer.cpp -- the Qwen3 byte-level BPE tokenizer at the ends of the path (the reference's QwenTokenizer,
// src/Lrm.Tokenizer/*.fs, specified by docs/contracts/tokenizer.md) behind the lrm_tok_* entry points. Host code.
//
// Encode: the text (valid UTF-8) is cut at the added tokens (leftmost-longest over a trie, on the raw text); each
// stretch between them is normalized to the oracle's NFC (Unicode 9.0: newer-Unicode NFC between the split points
// of unicode_tables.g.h, which stay as they are), split by the Qwen Split pre-tokenizer (a state machine over scalar
// values equal to the Oniguruma regex, rules 1-7 below), and each piece's UTF-8 bytes go through byte-level BPE: one
// symbol per byte, then the adjacent pair of lowest merge rank is merged, the leftmost among equal ranks, until no
// pair has a merge. Decode concatenates the tokens' bytes (added tokens by the byte map when every character is in
// it, else as UTF-8; ids past the vocabulary and below the model's 151,936 rows add nothing) and decodes UTF-8 with
// one U+FFFD per maximal invalid subpart.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <mutex>
#include <queue>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/lrm_cuda.h"
#include "internal.h"
#include "json.h"
#include "unicode_tables.g.h"

namespace lrm {
namespace tok {

constexpr int kModelRows = 151936;  // Qwen3-0.6B's embedding and lm_head rows
constexpr const char *kSplitPattern =
    "(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|"
    "\\s+(?!\\S)|\\s+";

struct FormatError {
    std::string msg;
};
// Loader refusals carry the reference's wording (TokenizerJson.fs:23-24): "tokenizer.json: <what>".
[[noreturn]] static void fail(const std::string &m) { throw FormatError{"tokenizer.json: " + m}; }

// ---- Unicode tables ---------------------------------------------------------------------------------------------

enum Cls : uint8_t { LETTER = 0, NUMBER = 1, SPACE = 2, OTHER = 3 };

struct Tables {
    uint8_t bmp_class[0x10000];
    std::unordered_map<uint32_t, std::pair<uint32_t, uint32_t>> decomp;  // scalar -> (offset, length)
    std::unordered_map<uint64_t, uint32_t> comp;                         // (first << 32 | second) -> composite
    Tables() {
        for (int r = 0; r < kClassRunCount; ++r) {
            const uint32_t a = kClassRuns[r][0], b = r + 1 < kClassRunCount ? kClassRuns[r + 1][0] : 0x110000;
            for (uint32_t c = a; c < b && c < 0x10000; ++c) bmp_class[c] = (uint8_t)kClassRuns[r][1];
        }
        for (int i = 0; i < kDecompCount; ++i) decomp[kDecompIndex[i][0]] = {kDecompIndex[i][1], kDecompIndex[i][2]};
        for (int i = 0; i < kCompCount; ++i) comp[((uint64_t)kComp[i][0] << 32) | kComp[i][1]] = kComp[i][2];
    }
};

static const Tables &tables() {
    static const Tables t;
    return t;
}

uint8_t class_of(uint32_t v) {
    if (v < 0x10000) return tables().bmp_class[v];
    int lo = 0, hi = kClassRunCount - 1;  // the last run starting at or before v
    while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (kClassRuns[mid][0] <= v)
            lo = mid;
        else
            hi = mid - 1;
    }
    return (uint8_t)kClassRuns[lo][1];
}

static bool in_ranges(const uint32_t (*r)[2], int n, uint32_t v) {
    int lo = 0, hi = n - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) / 2;
        if (v < r[mid][0])
            hi = mid - 1;
        else if (v > r[mid][1])
            lo = mid + 1;
        else
            return true;
    }
    return false;
}

static bool is_split_point(uint32_t v) { return in_ranges(kSplitRanges, kSplitRangeCount, v); }

static uint8_t ccc_of(uint32_t v) {
    int lo = 0, hi = kCccRangeCount - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) / 2;
        if (v < kCccRanges[mid][0])
            hi = mid - 1;
        else if (v > kCccRanges[mid][1])
            lo = mid + 1;
        else
            return (uint8_t)kCccRanges[mid][2];
    }
    return 0;
}

// The letter a scalar stands for in the case-insensitive group (?i:'s|'t|'re|'ve|'m|'ll|'d): simple case folding
// restricted to the group's letters, where U+017F LATIN SMALL LETTER LONG S folds to s; 0 for anything else.
char contraction_letter(uint32_t v) {
    if (v == 0x17F) return 's';
    if (v < 128) {
        const char c = (char)(v | 0x20);  // ASCII letters: both cases
        if ((v >= 'A' && v <= 'Z') || (v >= 'a' && v <= 'z'))
            if (strchr("stmdrvel", c)) return c;
    }
    return 0;
}

// ---- NFC -------------------------------------------------------------------------------------------------------

constexpr uint32_t SBase = 0xAC00, LBase = 0x1100, VBase = 0x1161, TBase = 0x11A7;
constexpr uint32_t LCount = 19, VCount = 21, TCount = 28, NCount = VCount * TCount, SCount = LCount * NCount;

static void decompose(uint32_t c, std::u32string &out) {
    if (c >= SBase && c < SBase + SCount) {  // Hangul syllables decompose by arithmetic
        const uint32_t s = c - SBase;
        out += LBase + s / NCount;
        out += VBase + (s % NCount) / TCount;
        if (s % TCount) out += TBase + s % TCount;
        return;
    }
    const auto &d = tables().decomp;
    auto it = d.find(c);
    if (it == d.end()) {
        out += c;
        return;
    }
    for (uint32_t k = 0; k < it->second.second; ++k) out += kDecompFlat[it->second.first + k];
}

static uint32_t compose_pair(uint32_t a, uint32_t b) {
    if (a >= LBase && a < LBase + LCount && b >= VBase && b < VBase + VCount)
        return SBase + ((a - LBase) * VCount + (b - VBase)) * TCount;
    if (a >= SBase && a < SBase + SCount && (a - SBase) % TCount == 0 && b > TBase && b < TBase + TCount)
        return a + (b - TBase);
    const auto &m = tables().comp;
    auto it = m.find(((uint64_t)a << 32) | b);
    return it == m.end() ? 0 : it->second;
}

// NFC of a stretch that holds no split point: canonical decomposition, canonical ordering (a stable sort of each run
// of non-starters by combining class), canonical composition (a character composes with the last starter unless a
// character between them has class zero or a class not below its own).
static void nfc_segment(const char32_t *s, size_t n, std::u32string &out) {
    std::u32string d;
    d.reserve(n + 8);
    for (size_t i = 0; i < n; ++i) decompose(s[i], d);
    std::vector<uint8_t> cc(d.size());
    for (size_t i = 0; i < d.size(); ++i) cc[i] = ccc_of(d[i]);
    for (size_t i = 0; i < d.size();) {
        if (cc[i] == 0) {
            ++i;
            continue;
        }
        size_t j = i;
        while (j < d.size() && cc[j] != 0) ++j;
        for (size_t a = i + 1; a < j; ++a)  // insertion sort: stable
            for (size_t b = a; b > i && cc[b - 1] > cc[b]; --b) {
                std::swap(d[b - 1], d[b]);
                std::swap(cc[b - 1], cc[b]);
            }
        i = j;
    }
    if (d.empty()) return;
    const size_t base = out.size();
    size_t starter = base;
    out += d[0];
    int last = cc[0] == 0 ? 0 : 256;  // a leading non-starter composes with nothing
    for (size_t i = 1; i < d.size(); ++i) {
        const uint32_t c = d[i];
        const int k = cc[i];
        const uint32_t composite = last == 256 ? 0 : compose_pair(out[starter], c);
        if (composite && (last < k || last == 0)) {
            out[starter] = composite;
            continue;
        }
        if (k == 0) starter = out.size();
        last = k;
        out += c;
    }
}

void nfc(const std::u32string &s, std::u32string &out) {
    size_t a = 0;
    for (size_t i = 0; i <= s.size(); ++i) {
        if (i == s.size() || is_split_point(s[i])) {
            nfc_segment(s.data() + a, i - a, out);
            if (i < s.size()) out += s[i];
            a = i + 1;
        }
    }
}

// ---- UTF-8 -----------------------------------------------------------------------------------------------------

// Strict decoding; on failure `bad` is the byte offset of the first invalid sequence.
bool utf8_decode(const uint8_t *p, size_t n, std::u32string &out, size_t *bad) {
    out.clear();
    out.reserve(n);
    size_t i = 0;
    while (i < n) {
        const uint8_t c = p[i];
        uint32_t cp;
        int len;
        if (c < 0x80) {
            out += c;
            ++i;
            continue;
        } else if (c >= 0xC2 && c <= 0xDF) {
            len = 2, cp = c & 0x1F;
        } else if (c >= 0xE0 && c <= 0xEF) {
            len = 3, cp = c & 0x0F;
        } else if (c >= 0xF0 && c <= 0xF4) {
            len = 4, cp = c & 0x07;
        } else {
            if (bad) *bad = i;
            return false;
        }
        if (i + len > n) {
            if (bad) *bad = i;
            return false;
        }
        for (int k = 1; k < len; ++k) {
            if ((p[i + k] & 0xC0) != 0x80) {
                if (bad) *bad = i;
                return false;
            }
            cp = (cp << 6) | (p[i + k] & 0x3F);
        }
        if ((len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) {
            if (bad) *bad = i;
            return false;
        }
        out += cp;
        i += len;
    }
    return true;
}

// Decoding with one U+FFFD per maximal subpart of an ill-formed sequence (Unicode's recommended practice, Python's
// errors="replace"): a lead byte starts a subpart that continues while each next byte is allowed there.
void utf8_decode_replace(const uint8_t *p, size_t n, std::u32string &out) {
    out.clear();
    size_t i = 0;
    while (i < n) {
        const uint8_t c = p[i];
        if (c < 0x80) {
            out += c;
            ++i;
            continue;
        }
        int len;
        uint8_t lo = 0x80, hi = 0xBF;  // the range of the second byte
        uint32_t cp;
        if (c >= 0xC2 && c <= 0xDF) {
            len = 2, cp = c & 0x1F;
        } else if (c >= 0xE0 && c <= 0xEF) {
            len = 3, cp = c & 0x0F;
            if (c == 0xE0) lo = 0xA0;
            if (c == 0xED) hi = 0x9F;
        } else if (c >= 0xF0 && c <= 0xF4) {
            len = 4, cp = c & 0x07;
            if (c == 0xF0) lo = 0x90;
            if (c == 0xF4) hi = 0x8F;
        } else {
            out += 0xFFFD;
            ++i;
            continue;
        }
        size_t k = 1;
        for (; k < (size_t)len; ++k) {
            if (i + k >= n) break;
            const uint8_t b = p[i + k];
            const uint8_t l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
            if (b < l || b > h) break;
            cp = (cp << 6) | (b & 0x3F);
        }
        if (k == (size_t)len) {
            out += cp;
        } else {
            out += 0xFFFD;  // the maximal subpart p[i, i + k)
        }
        i += k;
    }
}

void utf8_encode(const char32_t *s, size_t n, std::string &out) {
    for (size_t i = 0; i < n; ++i) {
        const uint32_t cp = s[i];
        if (cp < 0x80) {
            out += (char)cp;
        } else if (cp < 0x800) {
            out += (char)(0xC0 | (cp >> 6));
            out += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18));
            out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        }
    }
}

// ---- the Split pre-tokenizer ------------------------------------------------------------------------------------
//
// The end of the match of (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|
// \s*[\r\n]+|\s+(?!\S)|\s+ that starts at p (first alternative that matches; every scalar is a letter, a number,
// white space or other, so the matches tile the text):
//  1. p+2 or p+3 when U+0027 is followed by s, t, m or d, or by re, ve or ll (simple case folding);
//  2. the end of the letter run when p is a letter, or when p is not \r, \n or a number and p+1 is a letter;
//  3. p+1 when p is a number;
//  4. when p is other, or U+0020 followed by other: after the run of others, then the run of \r and \n;
//  5. when p starts a white-space run [p, q) holding \r or \n: just after its last \r or \n;
//  6. otherwise q when the run ends the text, or q-1 when it has two or more scalars;
//  7. otherwise q.
static size_t match_end(const char32_t *cp, const uint8_t *cls, size_t n, size_t p) {
    const uint32_t c = cp[p];
    const uint8_t k = cls[p];
    auto run_end = [&](uint8_t want, size_t from) {
        while (from < n && cls[from] == want) ++from;
        return from;
    };
    auto crlf = [](uint32_t v) { return v == 0x0D || v == 0x0A; };
    if (c == 0x27 && p + 1 < n) {
        const char a = contraction_letter(cp[p + 1]);
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return p + 2;
        if (p + 2 < n) {
            const char b = contraction_letter(cp[p + 2]);
            if ((a == 'r' || a == 'v') && b == 'e') return p + 3;
            if (a == 'l' && b == 'l') return p + 3;
        }
    }
    if (k == LETTER) return run_end(LETTER, p + 1);
    if (k != NUMBER && !crlf(c) && p + 1 < n && cls[p + 1] == LETTER) return run_end(LETTER, p + 2);
    if (k == NUMBER) return p + 1;
    if (k == OTHER || (c == 0x20 && p + 1 < n && cls[p + 1] == OTHER)) {
        size_t e = run_end(OTHER, k == OTHER ? p + 1 : p + 2);
        while (e < n && crlf(cp[e])) ++e;
        return e;
    }
    size_t q = p;
    long last_crlf = -1;
    while (q < n && cls[q] == SPACE) {
        if (crlf(cp[q])) last_crlf = (long)q;
        ++q;
    }
    if (last_crlf >= 0) return (size_t)last_crlf + 1;
    if (q == n) return n;
    if (q - p >= 2) return q - 1;
    return q;
}

// Piece boundaries of `s`: the end index of each piece, in order.
void split(const std::u32string &s, std::vector<size_t> &ends) {
    ends.clear();
    std::vector<uint8_t> cls(s.size());
    for (size_t i = 0; i < s.size(); ++i) cls[i] = class_of(s[i]);
    for (size_t p = 0; p < s.size();) {
        const size_t e = match_end(s.data(), cls.data(), s.size(), p);
        ends.push_back(e);
        p = e;
    }
}

// ---- byte level -------------------------------------------------------------------------------------------------
//
// GPT-2's map: the 188 bytes 0x21-0x7E, 0xA1-0xAC and 0xAE-0xFF stand for themselves; the other 68, in increasing
// order, become U+0100 to U+0143.
struct ByteMap {
    uint32_t to_char[256];
    int16_t to_byte[0x144];
    ByteMap() {
        for (int i = 0; i < 0x144; ++i) to_byte[i] = -1;
        int next = 0x100;
        for (int b = 0; b < 256; ++b) {
            const bool self = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
            to_char[b] = self ? (uint32_t)b : (uint32_t)next++;
            to_byte[to_char[b]] = (int16_t)b;
        }
    }
};
static const ByteMap &byte_map() {
    static const ByteMap m;
    return m;
}

// ---- the tokenizer ----------------------------------------------------------------------------------------------

struct Added {
    int id;
    std::string content;  // UTF-8
    bool special;
};

struct TrieNode {
    std::unordered_map<uint32_t, int> next;
    int added = -1;  // index into `added` of the token ending here
};

class Tokenizer {
  public:
    std::vector<std::string> tok_bytes;  // id -> raw bytes
    std::vector<std::string> tok_text;   // id -> byte-level form (UTF-8)
    std::unordered_map<std::string, int> by_text;
    int byte_id[256];
    std::unordered_map<uint64_t, uint64_t> merges;  // (left << 32 | right) -> (rank << 32 | merged)
    int n_vocab = 0, n_merges = 0;
    std::vector<Added> added;
    std::vector<std::string> added_bytes;  // what Decode emits for each added token
    std::vector<TrieNode> trie;

    void parse(const uint8_t *json, size_t n);
    void encode(const std::u32string &text, std::vector<int32_t> &ids);
    void decode_bytes(const int32_t *ids, size_t n, std::string &out) const;

    void clear_cache() {
        std::lock_guard<std::mutex> g(cache_mu_);
        cur_.clear();
        prev_.clear();
        cur_units_ = 0;
    }
    size_t cached_pieces() {
        std::lock_guard<std::mutex> g(cache_mu_);
        return cur_.size() + prev_.size();
    }

    // The piece cache (QwenTokenizer.fs:218-231): two generations, each full at 32,768 pieces or 1 Mi UTF-16 units
    // of piece text; a full current generation becomes the previous one. Pieces of more than 65,536 units are never
    // cached. The cache never changes a result.
    static constexpr size_t kGenPieces = 1u << 15, kGenUnits = 1u << 20, kMaxCachedPiece = 1u << 16;

  private:
    std::mutex cache_mu_;
    std::unordered_map<std::string, std::vector<int32_t>> cur_, prev_;
    size_t cur_units_ = 0;

    void bpe(const std::string &bytes, std::vector<int32_t> &ids) const;
    void encode_piece(const std::string &bytes, std::vector<int32_t> &ids);
    void remember(const std::string &bytes, size_t units, std::vector<int32_t> &&ids);
    void encode_stretch(const char32_t *s, size_t n, std::vector<int32_t> &ids);
};

void Tokenizer::bpe(const std::string &bytes, std::vector<int32_t> &ids) const {
    const size_t n = bytes.size();
    std::vector<int32_t> sym(n);
    std::vector<int32_t> nxt(n), prv(n);
    for (size_t i = 0; i < n; ++i) {
        sym[i] = byte_id[(uint8_t)bytes[i]];
        nxt[i] = i + 1 < n ? (int32_t)(i + 1) : -1;
        prv[i] = (int32_t)i - 1;
    }
    struct Cand {
        uint32_t rank;
        int32_t pos, left, right;
        bool operator>(const Cand &o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
    };
    std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> q;
    auto push = [&](int32_t pos) {
        if (pos < 0 || nxt[pos] < 0) return;
        auto it = merges.find(((uint64_t)(uint32_t)sym[pos] << 32) | (uint32_t)sym[nxt[pos]]);
        if (it != merges.end()) q.push(Cand{(uint32_t)(it->second >> 32), pos, sym[pos], sym[nxt[pos]]});
    };
    for (size_t i = 0; i + 1 < n; ++i) push((int32_t)i);
    while (!q.empty()) {
        const Cand c = q.top();
        q.pop();
        const int32_t r = nxt[c.pos];
        if (sym[c.pos] != c.left || r < 0 || sym[r] != c.right) continue;  // stale: the pair changed
        auto it = merges.find(((uint64_t)(uint32_t)c.left << 32) | (uint32_t)c.right);
        sym[c.pos] = (int32_t)(uint32_t)it->second;
        sym[r] = -1;
        nxt[c.pos] = nxt[r];
        if (nxt[r] >= 0) prv[nxt[r]] = c.pos;
        push(prv[c.pos]);
        push(c.pos);
    }
    for (int32_t i = n ? 0 : -1; i >= 0; i = nxt[i]) ids.push_back(sym[i]);
}

// UTF-16 code units of UTF-8 text: one per scalar, two for those past U+FFFF.
static size_t utf16_units(const std::string &b) {
    size_t u = 0;
    for (unsigned char c : b) u += (c & 0xC0) != 0x80 ? (c >= 0xF0 ? 2 : 1) : 0;
    return u;
}

void Tokenizer::encode_piece(const std::string &bytes, std::vector<int32_t> &ids) {
    const size_t units = utf16_units(bytes);
    if (units > kMaxCachedPiece) {
        bpe(bytes, ids);
        return;
    }
    {
        std::lock_guard<std::mutex> g(cache_mu_);
        auto it = cur_.find(bytes);
        if (it != cur_.end()) {
            ids.insert(ids.end(), it->second.begin(), it->second.end());
            return;
        }
        it = prev_.find(bytes);
        if (it != prev_.end()) {
            ids.insert(ids.end(), it->second.begin(), it->second.end());
            std::vector<int32_t> hit = it->second;
            remember(bytes, units, std::move(hit));
            return;
        }
    }
    std::vector<int32_t> got;
    bpe(bytes, got);
    ids.insert(ids.end(), got.begin(), got.end());
    std::lock_guard<std::mutex> g(cache_mu_);
    remember(bytes, units, std::move(got));
}

// Adds a piece to the current generation (the cache lock is held).
void Tokenizer::remember(const std::string &bytes, size_t units, std::vector<int32_t> &&ids) {
    if (cur_.emplace(bytes, std::move(ids)).second) cur_units_ += units;
    if (cur_.size() >= kGenPieces || cur_units_ >= kGenUnits) {
        prev_.swap(cur_);
        cur_.clear();
        cur_units_ = 0;
    }
}

void Tokenizer::encode_stretch(const char32_t *s, size_t n, std::vector<int32_t> &ids) {
    if (!n) return;
    std::u32string normal;
    nfc(std::u32string(s, n), normal);
    std::vector<size_t> ends;
    split(normal, ends);
    size_t a = 0;
    std::string bytes;
    for (size_t e : ends) {
        bytes.clear();
        utf8_encode(normal.data() + a, e - a, bytes);
        encode_piece(bytes, ids);
        a = e;
    }
}

void Tokenizer::encode(const std::u32string &text, std::vector<int32_t> &ids) {
    ids.clear();
    size_t last = 0, i = 0;
    while (i < text.size()) {
        int best = -1;
        size_t best_len = 0, node = 0;
        for (size_t j = i; j < text.size(); ++j) {  // the longest added token starting at i
            auto it = trie[node].next.find(text[j]);
            if (it == trie[node].next.end()) break;
            node = (size_t)it->second;
            if (trie[node].added >= 0) {
                best = trie[node].added;
                best_len = j - i + 1;
            }
        }
        if (best < 0) {
            ++i;
            continue;
        }
        encode_stretch(text.data() + last, i - last, ids);
        ids.push_back(added[(size_t)best].id);
        i += best_len;
        last = i;
    }
    encode_stretch(text.data() + last, text.size() - last, ids);
}

void Tokenizer::decode_bytes(const int32_t *ids, size_t n, std::string &out) const {
    for (size_t i = 0; i < n; ++i) {
        const int32_t id = ids[i];
        if (id < n_vocab)
            out += tok_bytes[(size_t)id];
        else if (id < n_vocab + (int32_t)added.size())
            out += added_bytes[(size_t)(id - n_vocab)];
    }
}

// ---- tokenizer.json ---------------------------------------------------------------------------------------------

using json::JValue;

static const JValue *member(const JValue &o, const char *name) {
    if (o.kind != JValue::OBJECT) return nullptr;
    for (const auto &m : o.members)
        if (m.first == name) return &m.second;
    return nullptr;
}
static const JValue &prop(const JValue &o, const std::string &path, const char *name) {
    const JValue *v = member(o, name);
    if (!v) fail(path + " has no '" + name + "'");
    return *v;
}
static bool is_null(const JValue *v) { return v && v->kind == JValue::LITERAL && v->text == "null"; }
static void expect_str(const JValue &o, const std::string &path, const char *name, const std::string &want) {
    const JValue &v = prop(o, path, name);
    if (v.kind != JValue::STRING) fail(path + "." + name + " is not a string");
    if (v.text != want) fail(path + "." + name + " is '" + v.text + "', only '" + want + "' is supported");
}
static void expect_bool(const JValue &o, const std::string &path, const char *name, bool want) {
    const JValue &v = prop(o, path, name);
    if (v.kind != JValue::LITERAL || v.text != (want ? "true" : "false"))
        fail(path + "." + name + " must be " + (want ? "true" : "false"));
}
static void expect_absent_or_null(const JValue &o, const std::string &path, const char *name) {
    const JValue *v = member(o, name);
    if (v && !is_null(v)) fail(path + "." + name + " must be null");
}
static void expect_empty_affix(const JValue &o, const std::string &path, const char *name) {
    const JValue *v = member(o, name);
    if (v && !is_null(v) && !(v->kind == JValue::STRING && v->text.empty())) fail(path + "." + name + " must be empty");
}
static void expect_false_or_absent(const JValue &o, const std::string &path, const char *name) {
    const JValue *v = member(o, name);
    if (v && !(v->kind == JValue::LITERAL && (v->text == "false" || v->text == "null")))
        fail(path + "." + name + " must be false");
}
static void check_byte_level(const JValue &o, const std::string &path, bool pre) {
    expect_str(o, path, "type", "ByteLevel");
    expect_bool(o, path, "add_prefix_space", false);
    if (pre) expect_bool(o, path, "use_regex", false);  // absent means true in tokenizers
}
// An id: a JSON integer in int32 range (System.Text.Json's GetInt32 refuses fractions and exponents).
static int as_int(const JValue &v, const std::string &what) {
    const std::string &t = v.text;
    const size_t digits = t.size() - (!t.empty() && t[0] == '-');
    if (v.kind != JValue::NUMBER || digits == 0 || digits > 10 ||
        t.find_first_not_of("0123456789", t[0] == '-' ? 1 : 0) != std::string::npos)
        fail(what + " is not a number");
    const long long x = std::stoll(t);
    if (x < INT32_MIN || x > INT32_MAX) fail(what + " is not a number");
    return (int)x;
}

// The raw bytes of a byte-level string, or false when a character is outside the byte map.
static bool byte_level_bytes(const std::string &utf8, std::string &bytes) {
    std::u32string s;
    if (!utf8_decode((const uint8_t *)utf8.data(), utf8.size(), s, nullptr)) return false;
    bytes.clear();
    for (char32_t c : s) {
        if (c >= 0x144 || byte_map().to_byte[c] < 0) return false;
        bytes += (char)byte_map().to_byte[c];
    }
    return true;
}

void Tokenizer::parse(const uint8_t *js, size_t n) {
    if (!json::valid_utf8(js, n)) throw FormatError{"tokenizer.json is not valid JSON: the text is not UTF-8"};
    JValue root;
    try {
        root = json::Parser(js, n, 64).document();
    } catch (const json::Error &e) {
        throw FormatError{"tokenizer.json is not valid JSON: " + e.msg};
    }
    if (root.kind != JValue::OBJECT) fail("$ is not an object");
    expect_absent_or_null(root, "$", "truncation");
    expect_absent_or_null(root, "$", "padding");
    expect_str(prop(root, "$", "normalizer"), "normalizer", "type", "NFC");
    const JValue &pre = prop(root, "$", "pre_tokenizer");
    expect_str(pre, "pre_tokenizer", "type", "Sequence");
    const JValue &steps = prop(pre, "pre_tokenizer", "pretokenizers");
    if (steps.kind != JValue::ARRAY || steps.items.size() != 2) fail("pre_tokenizer.pretokenizers must be [Split, ByteLevel]");
    const JValue &sp = steps.items[0];
    expect_str(sp, "pre_tokenizer.pretokenizers[0]", "type", "Split");
    expect_str(prop(sp, "Split", "pattern"), "Split.pattern", "Regex", kSplitPattern);
    expect_str(sp, "Split", "behavior", "Isolated");
    expect_bool(sp, "Split", "invert", false);
    check_byte_level(steps.items[1], "pre_tokenizer.pretokenizers[1]", true);
    const JValue *pp = member(root, "post_processor");
    if (pp && !is_null(pp)) expect_str(*pp, "post_processor", "type", "ByteLevel");
    check_byte_level(prop(root, "$", "decoder"), "decoder", false);
    const JValue &model = prop(root, "$", "model");
    expect_str(model, "model", "type", "BPE");
    expect_absent_or_null(model, "model", "dropout");
    expect_absent_or_null(model, "model", "unk_token");
    expect_empty_affix(model, "model", "continuing_subword_prefix");
    expect_empty_affix(model, "model", "end_of_word_suffix");
    expect_false_or_absent(model, "model", "fuse_unk");
    expect_false_or_absent(model, "model", "byte_fallback");
    expect_false_or_absent(model, "model", "ignore_merges");

    const JValue &vocab = prop(model, "model", "vocab");
    if (vocab.kind != JValue::OBJECT) fail("model.vocab is not an object");
    n_vocab = (int)vocab.members.size();
    tok_bytes.assign((size_t)n_vocab, std::string());
    tok_text.assign((size_t)n_vocab, std::string());
    std::vector<char> seen((size_t)n_vocab, 0);
    by_text.reserve((size_t)n_vocab * 2);
    for (const auto &m : vocab.members) {
        const int id = as_int(m.second, "model.vocab[" + m.first + "]");
        if (!by_text.emplace(m.first, id).second) fail("model.vocab has '" + m.first + "' twice");
        if (id < 0 || id >= n_vocab || seen[(size_t)id])
            fail("model.vocab ids are not 0.." + std::to_string(n_vocab - 1) + ", each once (" + m.first + " -> " +
                 std::to_string(id) + ")");
        seen[(size_t)id] = 1;
        if (!byte_level_bytes(m.first, tok_bytes[(size_t)id]) || tok_bytes[(size_t)id].empty())
            fail("model.vocab token '" + m.first + "' is not a byte-level string");
        tok_text[(size_t)id] = m.first;
    }
    for (int b = 0; b < 256; ++b) {
        std::string one;
        const char32_t c = byte_map().to_char[b];
        utf8_encode(&c, 1, one);
        auto it = by_text.find(one);
        if (it == by_text.end()) {
            char hex[8];
            snprintf(hex, sizeof hex, "%02X", b);
            fail(std::string("model.vocab has no token for byte 0x") + hex);
        }
        byte_id[b] = it->second;
    }
    const JValue &ml = prop(model, "model", "merges");
    if (ml.kind != JValue::ARRAY) fail("model.merges is not an array");
    n_merges = (int)ml.items.size();
    merges.reserve((size_t)n_merges * 2);
    for (size_t r = 0; r < ml.items.size(); ++r) {
        const JValue &e = ml.items[r];
        std::string a, b;
        if (e.kind == JValue::ARRAY && e.items.size() == 2 && e.items[0].kind == JValue::STRING &&
            e.items[1].kind == JValue::STRING) {
            a = e.items[0].text;
            b = e.items[1].text;
        } else if (e.kind == JValue::STRING) {
            const size_t sp_at = e.text.find(' ');
            if (sp_at == std::string::npos || e.text.find(' ', sp_at + 1) != std::string::npos)
                fail("model.merges[" + std::to_string(r) + "] is not 'a b'");
            a = e.text.substr(0, sp_at);
            b = e.text.substr(sp_at + 1);
        } else {
            fail("model.merges[" + std::to_string(r) + "] is not a pair");
        }
        int ids3[3];
        const std::string names[3] = {a, b, a + b};
        for (int k = 0; k < 3; ++k) {
            auto it = by_text.find(names[k]);
            if (it == by_text.end())
                fail("model.merges[" + std::to_string(r) + "] names '" + names[k] + "', which is not in the vocabulary");
            ids3[k] = it->second;
        }
        const uint64_t key = ((uint64_t)(uint32_t)ids3[0] << 32) | (uint32_t)ids3[1];
        if (!merges.emplace(key, ((uint64_t)r << 32) | (uint32_t)ids3[2]).second)
            fail("model.merges[" + std::to_string(r) + "] repeats the pair '" + a + "' '" + b + "'");
    }
    added.clear();
    added_bytes.clear();
    trie.assign(1, TrieNode());
    const JValue *at = member(root, "added_tokens");
    if (at && !is_null(at)) {
        if (at->kind != JValue::ARRAY) fail("added_tokens is not an array");
        for (const JValue &t : at->items) {
            const int id = as_int(prop(t, "added_tokens[]", "id"), "added_tokens[].id");
            const std::string path = "added_tokens[id " + std::to_string(id) + "]";
            const JValue &content = prop(t, path, "content");
            if (content.kind != JValue::STRING) fail(path + ".content is not a string");
            expect_bool(t, path, "normalized", false);
            expect_bool(t, path, "lstrip", false);
            expect_bool(t, path, "rstrip", false);
            expect_bool(t, path, "single_word", false);
            const JValue &special = prop(t, path, "special");
            if (special.kind != JValue::LITERAL || (special.text != "true" && special.text != "false"))
                fail(path + ".special is not a boolean");
            added.push_back(Added{id, content.text, special.text == "true"});
        }
        std::stable_sort(added.begin(), added.end(), [](const Added &a, const Added &b) { return a.id < b.id; });
        for (size_t i = 0; i < added.size(); ++i)
            if (added[i].id != n_vocab + (int)i)
                fail("added token ids must follow the vocabulary (" + std::to_string(n_vocab + (int)i) + " expected, " +
                     std::to_string(added[i].id) + " found)");
        for (size_t i = 0; i < added.size(); ++i) {
            const std::string &content = added[i].content;
            if (content.empty()) fail("an added token has empty content");
            std::string bytes;
            added_bytes.push_back(byte_level_bytes(content, bytes) ? bytes : content);
            std::u32string s;
            utf8_decode((const uint8_t *)content.data(), content.size(), s, nullptr);
            size_t node = 0;
            for (char32_t c : s) {
                auto it = trie[node].next.find(c);
                if (it == trie[node].next.end()) {
                    trie.push_back(TrieNode());
                    trie[node].next.emplace(c, (int)trie.size() - 1);
                    node = trie.size() - 1;
                } else {
                    node = (size_t)it->second;
                }
            }
            if (trie[node].added >= 0) fail("the added token " + content + " appears twice");
            trie[node].added = (int)i;
        }
    }
}

}  // namespace tok
}  // namespace lrm

using namespace lrm;

struct lrm_tokenizer_s {
    tok::Tokenizer t;
};

namespace {

lrm_status tfail(lrm_status s, const std::string &m) {
    set_thread_error(m);
    return s;
}

// Copies `n` items to `out` when it has room; always reports the count.
template <typename T>
lrm_status deliver(const T *src, size_t n, T *out, uint64_t cap, uint64_t *count) {
    if (count) *count = n;
    if (!out) return LRM_OK;  // a size query
    if (cap < n) return tfail(LRM_ERR_ARGUMENT, "the output buffer holds " + std::to_string(cap) + ", " + std::to_string(n) + " are needed");
    if (n) memcpy(out, src, n * sizeof(T));
    return LRM_OK;
}

bool decode_text(const char *utf8, uint64_t n, std::u32string &s) {
    size_t bad = 0;
    if (!tok::utf8_decode((const uint8_t *)utf8, (size_t)n, s, &bad)) {
        set_thread_error("the text is not valid UTF-8 (a lone surrogate or a broken sequence at byte " +
                         std::to_string(bad) + ")");
        return false;
    }
    return true;
}

}  // namespace

extern "C" {

lrm_status lrm_tok_parse(const void *json, uint64_t n, lrm_tokenizer *out) {
    if (!json || !out) return tfail(LRM_ERR_ARGUMENT, "json or out is null");
    *out = nullptr;
    std::unique_ptr<lrm_tokenizer_s> h(new lrm_tokenizer_s);
    try {
        h->t.parse((const uint8_t *)json, (size_t)n);
    } catch (const tok::FormatError &e) {
        return tfail(LRM_ERR_FORMAT, e.msg);
    } catch (const std::bad_alloc &) {
        return tfail(LRM_ERR_OUT_OF_MEMORY, "out of host memory while reading tokenizer.json");
    }
    *out = h.release();
    return LRM_OK;
}

lrm_status lrm_tok_free(lrm_tokenizer t) {
    delete t;
    return LRM_OK;
}

lrm_status lrm_tok_info(lrm_tokenizer t, int32_t *vocab_size, int32_t *merges, int32_t *added) {
    if (!t) return tfail(LRM_ERR_ARGUMENT, "tokenizer is null");
    if (vocab_size) *vocab_size = t->t.n_vocab + (int32_t)t->t.added.size();
    if (merges) *merges = t->t.n_merges;
    if (added) *added = (int32_t)t->t.added.size();
    return LRM_OK;
}

lrm_status lrm_tok_clear_cache(lrm_tokenizer t) {
    if (!t) return tfail(LRM_ERR_ARGUMENT, "tokenizer is null");
    t->t.clear_cache();
    return LRM_OK;
}

lrm_status lrm_tok_cached_pieces(lrm_tokenizer t, int64_t *pieces) {
    if (!t || !pieces) return tfail(LRM_ERR_ARGUMENT, "null argument");
    *pieces = (int64_t)t->t.cached_pieces();
    return LRM_OK;
}

lrm_status lrm_tok_added_at(lrm_tokenizer t, int32_t i, int32_t *id, const char **content, int32_t *special) {
    if (!t || !id || !content || !special) return tfail(LRM_ERR_ARGUMENT, "null argument");
    if (i < 0 || i >= (int32_t)t->t.added.size()) return tfail(LRM_ERR_ARGUMENT, "added token index out of range");
    *id = t->t.added[(size_t)i].id;
    *content = t->t.added[(size_t)i].content.c_str();
    *special = t->t.added[(size_t)i].special ? 1 : 0;
    return LRM_OK;
}

lrm_status lrm_tok_encode(lrm_tokenizer t, const char *utf8, uint64_t n, int32_t *ids, uint64_t cap, uint64_t *count) {
    if (!t || (!utf8 && n)) return tfail(LRM_ERR_ARGUMENT, "null argument");
    std::u32string s;
    if (!decode_text(utf8, n, s)) return LRM_ERR_ARGUMENT;
    std::vector<int32_t> out;
    t->t.encode(s, out);
    return deliver(out.data(), out.size(), ids, cap, count);
}

lrm_status lrm_tok_encode_bytes(lrm_tokenizer t, const uint8_t *bytes, uint64_t n, int32_t *ids, uint64_t cap,
                                uint64_t *count) {
    if (!t || (!bytes && n)) return tfail(LRM_ERR_ARGUMENT, "null argument");
    std::u32string s;
    tok::utf8_decode_replace(bytes, (size_t)n, s);
    std::vector<int32_t> out;
    t->t.encode(s, out);
    return deliver(out.data(), out.size(), ids, cap, count);
}

lrm_status lrm_tok_decode_bytes(lrm_tokenizer t, const int32_t *ids, uint64_t n, uint8_t *out, uint64_t cap,
                                uint64_t *len) {
    if (!t || (!ids && n)) return tfail(LRM_ERR_ARGUMENT, "null argument");
    for (uint64_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= tok::kModelRows)
            return tfail(LRM_ERR_ARGUMENT, "id " + std::to_string(ids[i]) + " is outside the model's " +
                                               std::to_string(tok::kModelRows) + " rows");
    std::string b;
    t->t.decode_bytes(ids, (size_t)n, b);
    return deliver((const uint8_t *)b.data(), b.size(), out, cap, len);
}

lrm_status lrm_tok_decode(lrm_tokenizer t, const int32_t *ids, uint64_t n, char *out, uint64_t cap, uint64_t *len) {
    if (!t || (!ids && n)) return tfail(LRM_ERR_ARGUMENT, "null argument");
    for (uint64_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= tok::kModelRows)
            return tfail(LRM_ERR_ARGUMENT, "id " + std::to_string(ids[i]) + " is outside the model's " +
                                               std::to_string(tok::kModelRows) + " rows");
    std::string b, text;
    t->t.decode_bytes(ids, (size_t)n, b);
    std::u32string s;
    tok::utf8_decode_replace((const uint8_t *)b.data(), b.size(), s);
    tok::utf8_encode(s.data(), s.size(), text);
    return deliver(text.data(), text.size(), out, cap, len);
}

lrm_status lrm_tok_id_of(lrm_tokenizer t, const char *token, int32_t *id) {
    if (!t || !token || !id) return tfail(LRM_ERR_ARGUMENT, "null argument");
    *id = -1;
    for (const auto &a : t->t.added)
        if (a.content == token) {
            *id = a.id;
            return LRM_OK;
        }
    auto it = t->t.by_text.find(token);
    if (it != t->t.by_text.end()) *id = it->second;
    return LRM_OK;
}

lrm_status lrm_tok_token_of(lrm_tokenizer t, int32_t id, char *out, uint64_t cap, uint64_t *len, int32_t *found) {
    if (!t || !found) return tfail(LRM_ERR_ARGUMENT, "null argument");
    *found = 0;
    const std::string *s = nullptr;
    if (id >= 0 && id < t->t.n_vocab)
        s = &t->t.tok_text[(size_t)id];
    else if (id >= t->t.n_vocab && id < t->t.n_vocab + (int32_t)t->t.added.size())
        s = &t->t.added[(size_t)(id - t->t.n_vocab)].content;
    if (!s) {
        if (len) *len = 0;
        return LRM_OK;
    }
    *found = 1;
    return deliver(s->data(), s->size(), out, cap, len);
}

// The stages, as the reference exposes them for diagnostics and tests (ByteLevel, CharClass, Nfc, PreTokenizer).

lrm_status lrm_tok_nfc(const char *utf8, uint64_t n, char *out, uint64_t cap, uint64_t *len) {
    if (!utf8 && n) return tfail(LRM_ERR_ARGUMENT, "null argument");
    std::u32string s, r;
    if (!decode_text(utf8, n, s)) return LRM_ERR_ARGUMENT;
    tok::nfc(s, r);
    std::string b;
    tok::utf8_encode(r.data(), r.size(), b);
    return deliver(b.data(), b.size(), out, cap, len);
}

lrm_status lrm_tok_split(const char *utf8, uint64_t n, uint64_t *ends, uint64_t cap, uint64_t *count) {
    if (!utf8 && n) return tfail(LRM_ERR_ARGUMENT, "null argument");
    std::u32string s;
    if (!decode_text(utf8, n, s)) return LRM_ERR_ARGUMENT;
    std::vector<size_t> e;
    tok::split(s, e);
    // scalar indices -> byte offsets
    std::vector<uint64_t> off;
    off.reserve(e.size());
    uint64_t byte = 0;
    size_t k = 0;
    for (size_t i = 0; i < s.size() && k < e.size(); ++i) {
        const uint32_t c = s[i];
        byte += c < 0x80 ? 1 : c < 0x800 ? 2 : c < 0x10000 ? 3 : 4;
        if (i + 1 == e[k]) {
            off.push_back(byte);
            ++k;
        }
    }
    return deliver(off.data(), off.size(), ends, cap, count);
}

int32_t lrm_tok_char_class(uint32_t scalar) { return scalar > 0x10FFFF ? -1 : (int32_t)tok::class_of(scalar); }

int32_t lrm_tok_contraction_letter(uint32_t scalar) { return (int32_t)tok::contraction_letter(scalar); }

uint32_t lrm_tok_byte_char(uint8_t byte) { return tok::byte_map().to_char[byte]; }

}  // extern "C"
