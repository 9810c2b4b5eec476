// Host-side Qwen3 tokenizer and chat template (tokenizer.h / tokenizer.c,
// main.c:124-185): byte-level BPE over the QW3T vocabulary file the reference
// exports (tok.bin), so a caller can go from text to tokens and back around the
// GPU runtime. Host code only; compiled into libn550_qwen3.so.
//
// Token ids must be exactly the reference's, so three things follow its
// tokenizer.c on purpose: the QW3T layout and error codes, the pre-tokenizer
// (the reference's hand-written state machine for the GPT-style split regex,
// including its whitespace set and its handling of invalid UTF-8 as single
// bytes), and the merge order (the lowest-rank adjacent pair first, the
// leftmost on equal ranks, one merge at a time). Everything else is this
// file's own: merge ranks in a hash map built at load, tokens in a linked list
// with a min-heap of candidate pairs (O(n log n) per piece), and a batch
// encoder that spreads many prompts over host threads for the data-parallel
// serving path.
#include <string.h>

#include <algorithm>
#include <queue>
#include <thread>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace {

constexpr uint32_t kMergesMax = 200000;      // tokenizer.c TOK_MERGES_MAX
constexpr size_t kPieceMax = 2048;           // QWEN3_TOK_MAX: longest piece the reference takes

uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

}  // namespace

struct n550_tok {
    std::vector<uint8_t> blob;               // owned copy of the file
    uint32_t n_vocab = 0;
    std::vector<uint32_t> index;             // [n_vocab + 1] byte offsets into data
    const uint8_t *data = nullptr;
    std::vector<uint32_t> merged;            // [n_merges] result id of merge rank r
    std::unordered_map<uint64_t, uint32_t> rank;   // (left << 32 | right) -> lowest rank
    std::vector<uint32_t> letters, digits;   // sorted inclusive [lo, hi] code point ranges
    uint32_t byte_id[256] = {};
    struct Special { uint32_t id, len, off; };
    std::vector<Special> specials;           // file order (longest first)
    const uint8_t *sdata = nullptr;
};

namespace {

bool in_ranges(const std::vector<uint32_t> &r, uint32_t cp) {
    size_t lo = 0, hi = r.size() / 2;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp < r[2 * mid]) hi = mid;
        else if (cp > r[2 * mid + 1]) lo = mid + 1;
        else return true;
    }
    return false;
}

// White space of the pre-tokenizer: the Unicode White_Space set as the
// reference's is_space lists it (U+1680 is not in its list).
bool is_space(uint32_t c) {
    return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 ||
           (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F ||
           c == 0x205F || c == 0x3000;
}
bool is_nl(uint32_t c) { return c == '\n' || c == '\r'; }

// One code point; a malformed sequence is taken as one byte whose value is
// the code point (the byte-level fallback). Returns the bytes consumed.
int utf8_step(const uint8_t *p, size_t n, uint32_t *cp) {
    const uint8_t c = p[0];
    auto cont = [&](size_t i) { return i < n && (p[i] & 0xC0) == 0x80; };
    if (c < 0x80) { *cp = c; return 1; }
    if ((c & 0xE0) == 0xC0 && cont(1)) { *cp = ((c & 0x1Fu) << 6) | (p[1] & 0x3Fu); return 2; }
    if ((c & 0xF0) == 0xE0 && cont(1) && cont(2)) {
        *cp = ((c & 0x0Fu) << 12) | ((p[1] & 0x3Fu) << 6) | (p[2] & 0x3Fu);
        return 3;
    }
    if ((c & 0xF8) == 0xF0 && cont(1) && cont(2) && cont(3)) {
        *cp = ((c & 0x07u) << 18) | ((p[1] & 0x3Fu) << 12) | ((p[2] & 0x3Fu) << 6) | (p[3] & 0x3Fu);
        return 4;
    }
    *cp = c;
    return 1;
}

struct Cursor {            // code-point walk over [p, p + n)
    const n550_tok *t;
    const uint8_t *p;
    size_t n;
    bool letter(uint32_t c) const { return in_ranges(t->letters, c); }
    bool digit(uint32_t c) const { return in_ranges(t->digits, c); }
    // code point at byte i (and its width)
    uint32_t at(size_t i, int *w) const { uint32_t c; *w = utf8_step(p + i, n - i, &c); return c; }
    // bytes from i while pred holds
    template <class F> size_t run(size_t i, F pred) const {
        while (i < n) {
            int w;
            if (!pred(at(i, &w))) break;
            i += (size_t)w;
        }
        return i;
    }
};

// Length in bytes of the next pre-tokenizer piece at the start of [p, p + n):
// the first alternative of
//   (?i:'s|'t|'re|'ve|'m|'ll|'d) | [^\r\n\p{L}\p{N}]?\p{L}+ | \p{N}
//   | ' '?[^\s\p{L}\p{N}]+[\r\n]* | \s*[\r\n]+ | \s+(?!\S) | \s+
// that matches here, as the reference's state machine decides it.
size_t piece_len(const n550_tok *t, const uint8_t *p, size_t n) {
    const Cursor cur{t, p, n};
    int w0;
    const uint32_t c0 = cur.at(0, &w0);
    // English contractions, ASCII case folded
    if (n >= 2 && p[0] == '\'') {
        const uint8_t a = p[1] | 0x20;
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
        if (n >= 3) {
            const uint8_t b = p[2] | 0x20;
            if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
        }
    }
    auto letter = [&](uint32_t c) { return cur.letter(c); };
    // letters, optionally after one character that is none of newline, letter, digit
    if (cur.letter(c0)) return cur.run((size_t)w0, letter);
    if (!is_nl(c0) && !cur.digit(c0) && (size_t)w0 < n) {
        int w1;
        if (cur.letter(cur.at((size_t)w0, &w1))) return cur.run((size_t)w0 + w1, letter);
    }
    if (cur.digit(c0)) return (size_t)w0;                    // one digit at a time
    // symbols (optionally after one space), then trailing newlines
    auto symbol = [&](uint32_t c) { return !is_space(c) && !cur.letter(c) && !cur.digit(c); };
    size_t start = 0;
    if (c0 == ' ' && (size_t)w0 < n) {
        int w1;
        if (symbol(cur.at((size_t)w0, &w1))) start = (size_t)w0;
    }
    const size_t end = cur.run(start, symbol);
    if (end > start) return cur.run(end, is_nl);
    if (is_space(c0)) {
        size_t i = 0, after_nl = 0;
        while (i < n) {
            int w;
            const uint32_t c = cur.at(i, &w);
            if (!is_space(c)) break;
            i += (size_t)w;
            if (is_nl(c)) after_nl = i;
        }
        if (after_nl) return after_nl;          // \s*[\r\n]+
        if (i >= n) return i;                   // \s+ at the end of the text
        return i > 1 ? i - 1 : i;               // leave one space to lead the next piece
    }
    return (size_t)w0;
}

// Byte-level BPE of one piece: bytes to their tokens, then the lowest-rank
// adjacent pair merged first (leftmost among equal ranks) until none is left.
// Tokens live in a doubly linked list; candidate pairs in a min-heap keyed by
// (rank, position of the left token), stale entries skipped on pop.
int bpe_piece(const n550_tok *t, const uint8_t *p, size_t n, int32_t *out, int room) {
    if (n == 0) return 0;
    if (n > kPieceMax) return N550_TOK_ERR_OVERFLOW;
    std::vector<int32_t> id(n);
    std::vector<int> prev(n), next(n);
    std::vector<char> alive(n, 1);
    for (size_t i = 0; i < n; i++) {
        id[i] = (int32_t)t->byte_id[p[i]];
        prev[i] = (int)i - 1;
        next[i] = i + 1 < n ? (int)i + 1 : -1;
    }
    struct Cand { uint32_t rank; int left; int32_t l, r; };
    auto later = [](const Cand &a, const Cand &b) {
        return a.rank != b.rank ? a.rank > b.rank : a.left > b.left;
    };
    std::priority_queue<Cand, std::vector<Cand>, decltype(later)> heap(later);
    auto push = [&](int i) {
        if (i < 0 || next[i] < 0) return;
        const auto it = t->rank.find(((uint64_t)(uint32_t)id[i] << 32) | (uint32_t)id[next[i]]);
        if (it != t->rank.end()) heap.push({it->second, i, id[i], id[next[i]]});
    };
    for (size_t i = 0; i + 1 < n; i++) push((int)i);
    int count = (int)n;
    while (!heap.empty()) {
        const Cand c = heap.top();
        heap.pop();
        const int i = c.left, j = alive[i] ? next[i] : -1;
        if (j < 0 || id[i] != c.l || id[j] != c.r) continue;      // pair changed since
        id[i] = (int32_t)t->merged[c.rank];
        alive[j] = 0;
        next[i] = next[j];
        if (next[j] >= 0) prev[next[j]] = i;
        count--;
        push(prev[i]);
        push(i);
    }
    if (count > room) return N550_TOK_ERR_OVERFLOW;
    int k = 0;
    for (int i = 0; i >= 0; i = next[i]) out[k++] = id[i];
    return k;
}

int encode(const n550_tok *t, const uint8_t *p, size_t len, int32_t *out, int max_out) {
    int total = 0;
    size_t i = 0;
    while (i < len) {
        bool special = false;
        for (const auto &s : t->specials) {       // whole special tokens first, longest first
            if (s.len <= len - i && memcmp(p + i, t->sdata + s.off, s.len) == 0) {
                if (total >= max_out) return N550_TOK_ERR_OVERFLOW;
                out[total++] = (int32_t)s.id;
                i += s.len;
                special = true;
                break;
            }
        }
        if (special) continue;
        size_t n = piece_len(t, p + i, len - i);
        if (n == 0) n = 1;
        const int got = bpe_piece(t, p + i, n, out + total, max_out - total);
        if (got < 0) return got;
        total += got;
        i += n;
    }
    return total;
}

// Qwen3's chat template with thinking disabled (main.c:124-131).
const char kChatPrefix[] = "<|im_start|>user\n";
const char kChatSuffix[] = "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n";

}  // namespace

extern "C" {

int n550_tok_init(n550_tok_t **out, const void *blob, size_t size) {
    if (!out || (!blob && size)) return N550_ERR_ARG;
    *out = nullptr;
    const uint8_t *b = (const uint8_t *)blob;
    if (size < 64) return N550_TOK_ERR_SIZE;
    if (memcmp(b, "QW3T", 4)) return N550_TOK_ERR_MAGIC;
    if (rd32(b + 4) != 1) return N550_TOK_ERR_VERSION;
    if (rd32(b + 56) != size) return N550_TOK_ERR_SIZE;
    const uint32_t n_vocab = rd32(b + 8), n_merges = rd32(b + 12), n_lr = rd32(b + 16),
                   n_nr = rd32(b + 20);
    if (n_merges > kMergesMax) return N550_TOK_ERR_SIZE;
    const uint32_t o_index = rd32(b + 24), o_data = rd32(b + 28), o_merges = rd32(b + 32),
                   o_lr = rd32(b + 36), o_nr = rd32(b + 40), o_byte = rd32(b + 44),
                   o_spec = rd32(b + 48), o_sdata = rd32(b + 52);
    // every table inside the file (the format carries no other checks)
    auto fits = [&](uint64_t off, uint64_t bytes) { return off + bytes <= size; };
    if (!fits(o_index, 4ull * (n_vocab + 1ull)) || !fits(o_merges, 12ull * n_merges) ||
        !fits(o_lr, 8ull * n_lr) || !fits(o_nr, 8ull * n_nr) || !fits(o_byte, 4ull * 256) ||
        !fits(o_spec, 4) || o_data > size || o_sdata > size)
        return N550_TOK_ERR_SIZE;
    const uint32_t n_special = rd32(b + o_spec);
    if (!fits(o_spec + 4ull, 12ull * n_special)) return N550_TOK_ERR_SIZE;

    n550_tok *t = new n550_tok();
    t->blob.assign(b, b + size);
    const uint8_t *c = t->blob.data();
    t->n_vocab = n_vocab;
    t->index.resize(n_vocab + 1);
    for (uint32_t i = 0; i <= n_vocab; i++) t->index[i] = rd32(c + o_index + 4ull * i);
    t->data = c + o_data;
    const uint64_t data_bytes = size - o_data;
    for (uint32_t i = 0; i < n_vocab; i++)
        if (t->index[i] > t->index[i + 1] || t->index[i + 1] > data_bytes) {
            delete t;
            return N550_TOK_ERR_SIZE;
        }
    t->merged.resize(n_merges);
    t->rank.reserve(2ull * n_merges);
    for (uint32_t r = 0; r < n_merges; r++) {
        const uint8_t *m = c + o_merges + 12ull * r;
        t->merged[r] = rd32(m + 8);
        t->rank.emplace(((uint64_t)rd32(m) << 32) | rd32(m + 4), r);   // duplicates: lowest rank
    }
    for (uint32_t i = 0; i < 2 * n_lr; i++) t->letters.push_back(rd32(c + o_lr + 4ull * i));
    for (uint32_t i = 0; i < 2 * n_nr; i++) t->digits.push_back(rd32(c + o_nr + 4ull * i));
    for (int i = 0; i < 256; i++) t->byte_id[i] = rd32(c + o_byte + 4ull * i);
    t->sdata = c + o_sdata;
    for (uint32_t s = 0; s < n_special; s++) {
        const uint8_t *e = c + o_spec + 4 + 12ull * s;
        n550_tok::Special sp{rd32(e), rd32(e + 4), rd32(e + 8)};
        if (sp.len == 0 || (uint64_t)o_sdata + sp.off + sp.len > size) {
            delete t;
            return N550_TOK_ERR_SIZE;
        }
        t->specials.push_back(sp);
    }
    *out = t;
    return N550_OK;
}

void n550_tok_free(n550_tok_t *t) { delete t; }

int n550_tok_vocab_size(const n550_tok_t *t) { return t ? (int)t->n_vocab : N550_ERR_ARG; }

const uint8_t *n550_tok_piece(const n550_tok_t *t, int id, size_t *len) {
    if (!t || !len) return nullptr;
    if (id < 0 || (uint32_t)id >= t->n_vocab) { *len = 0; return t->data; }
    *len = t->index[id + 1] - t->index[id];
    return t->data + t->index[id];
}

int n550_tok_encode(const n550_tok_t *t, const char *text, size_t len, int32_t *out, int max_out) {
    if (!t || (len && !text) || max_out < 0 || (max_out && !out)) return N550_ERR_ARG;
    return encode(t, (const uint8_t *)text, len, out, max_out);
}

int n550_tok_decode(const n550_tok_t *t, const int32_t *ids, int n, char *out, size_t max_out) {
    if (!t || n < 0 || (n && !ids) || !out) return N550_ERR_ARG;
    if (max_out == 0) return N550_TOK_ERR_OVERFLOW;
    size_t w = 0;
    for (int i = 0; i < n; i++) {
        size_t l;
        const uint8_t *s = n550_tok_piece(t, ids[i], &l);
        if (w + l >= max_out) return N550_TOK_ERR_OVERFLOW;   // room for the final '\0'
        memcpy(out + w, s, l);
        w += l;
    }
    out[w] = '\0';
    return (int)w;
}

int n550_tok_encode_batch(const n550_tok_t *t, const char *const *texts, const size_t *lens,
                          int n_texts, int32_t *out, int max_out, int32_t *counts, int n_threads) {
    if (!t || n_texts < 0 || (n_texts && (!texts || !lens || !counts)) || max_out < 0 ||
        (max_out && n_texts && !out))
        return N550_ERR_ARG;
    const int hw = (int)std::max(1u, std::thread::hardware_concurrency());
    const int nt = std::max(1, std::min({n_threads > 0 ? n_threads : hw, n_texts, 64}));
    auto work = [&](int w) {
        for (int i = w; i < n_texts; i += nt)
            counts[i] = encode(t, (const uint8_t *)texts[i], lens[i], out + (size_t)i * max_out, max_out);
    };
    std::vector<std::thread> pool;
    for (int w = 1; w < nt; w++) pool.emplace_back(work, w);
    work(0);
    for (auto &th : pool) th.join();
    for (int i = 0; i < n_texts; i++)
        if (counts[i] < 0) return counts[i];
    return N550_OK;
}

int n550_chat_encode(const n550_tok_t *t, const char *prompt, size_t len, int32_t *out, int max_out) {
    if (!t || (len && !prompt) || max_out < 0 || (max_out && !out)) return N550_ERR_ARG;
    std::vector<uint8_t> s;
    s.reserve(sizeof kChatPrefix + len + sizeof kChatSuffix);
    s.insert(s.end(), kChatPrefix, kChatPrefix + sizeof kChatPrefix - 1);
    s.insert(s.end(), (const uint8_t *)prompt, (const uint8_t *)prompt + len);
    s.insert(s.end(), kChatSuffix, kChatSuffix + sizeof kChatSuffix - 1);
    return encode(t, s.data(), s.size(), out, max_out);
}

}  // extern "C"
