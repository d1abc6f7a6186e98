// llama2.c-compatible SentencePiece-style BPE tokenizer (BpeTokenizer and its Tokenizer
// impl, src/tokenizer.rs:18-178), the host tokenizer in front of the decode loop.
//
// Results are the reference's:
//  - pieces are kept as UTF-8 with every ill-formed byte sequence replaced by U+FFFD, one
//    replacement per maximal subpart (String::from_utf8_lossy), and looked up by their bytes;
//    among equal pieces the lowest id is found;
//  - encode: BOS, the " " piece as a dummy prefix when the text is not empty, one piece per
//    UTF-8 character (a lead byte and up to three continuation bytes) or, when that is not a
//    well-formed character with a piece, its bytes + 3; then, while some adjacent pair
//    concatenates to a piece of score above -1e10, the highest-scoring such pair merges (the
//    leftmost one among equal scores); EOS;
//  - decode: the piece of the id ("" outside the vocabulary), without its leading space
//    after BOS; a "<0xNN>" piece (u8::from_str_radix rules) is the character U+00NN.
// The merge runs on a doubly linked list with a max-heap of candidate pairs that are
// dropped lazily once a side has merged, and pieces are found through a hash map, so an
// encode costs O(n log n) where the reference rescans every pair after each merge.
#include <cstdio>
#include <cstring>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace {

constexpr int32_t kBos = 1;  // src/tokenizer.rs:8-9
constexpr int32_t kEos = 2;

// Length of the well-formed UTF-8 character at s[0..n) (Unicode Table 3-7), or 0 with *bad
// = the length of its maximal ill-formed subpart (at least 1).
size_t utf8_char(const unsigned char* s, size_t n, size_t* bad) {
    const unsigned char c = s[0];
    if (c < 0x80) return 1;
    size_t need;
    unsigned char lo = 0x80, hi = 0xBF;  // range of the second byte
    if (c >= 0xC2 && c <= 0xDF) {
        need = 2;
    } else if (c >= 0xE0 && c <= 0xEF) {
        need = 3;
        if (c == 0xE0) lo = 0xA0;
        if (c == 0xED) hi = 0x9F;
    } else if (c >= 0xF0 && c <= 0xF4) {
        need = 4;
        if (c == 0xF0) lo = 0x90;
        if (c == 0xF4) hi = 0x8F;
    } else {
        *bad = 1;
        return 0;
    }
    size_t k = 1;
    for (; k < need; k++) {
        if (k >= n) break;
        const unsigned char b = s[k];
        const bool ok = k == 1 ? (b >= lo && b <= hi) : (b >= 0x80 && b <= 0xBF);
        if (!ok) break;
    }
    if (k == need) return need;
    *bad = k;
    return 0;
}

std::string utf8_lossy(const unsigned char* s, size_t n) {
    std::string out;
    out.reserve(n);
    size_t i = 0;
    while (i < n) {
        size_t bad = 0;
        const size_t len = utf8_char(s + i, n - i, &bad);
        if (len) {
            out.append(reinterpret_cast<const char*>(s + i), len);
            i += len;
        } else {
            out.append("\xEF\xBF\xBD");
            i += bad;
        }
    }
    return out;
}

// u8::from_str_radix(rest, 16) of a "<0x" rest ">" piece: an optional '+', then one or
// more hex digits whose value fits a byte.
bool parse_byte_token(const std::string& piece, unsigned* byte) {
    if (piece.size() < 4 || piece.compare(0, 3, "<0x") != 0 || piece.back() != '>') return false;
    size_t i = 3;
    const size_t end = piece.size() - 1;
    if (i < end && piece[i] == '+') i++;
    if (i >= end) return false;
    unsigned v = 0;
    for (; i < end; i++) {
        const char c = piece[i];
        unsigned d;
        if (c >= '0' && c <= '9') d = c - '0';
        else if (c >= 'a' && c <= 'f') d = c - 'a' + 10;
        else if (c >= 'A' && c <= 'F') d = c - 'A' + 10;
        else return false;
        v = v * 16 + d;
        if (v > 255) return false;
    }
    *byte = v;
    return true;
}

}  // namespace

// The tokenizer's state (its behaviour lives in the functions below, which stay private to
// the library).
struct ab_bpe {
    std::vector<std::string> vocab;
    std::vector<float> scores;
    uint32_t max_token_length = 0;
    std::unordered_map<std::string, int32_t> ids;
};

namespace {

void index_pieces(ab_bpe* t) {
    t->ids.reserve(t->vocab.size() * 2);
    for (size_t i = 0; i < t->vocab.size(); i++) t->ids.emplace(t->vocab[i], (int32_t)i);  // first wins
}

int32_t lookup(const ab_bpe* t, const std::string& s) {
    auto it = t->ids.find(s);
    return it == t->ids.end() ? -1 : it->second;
}

void merge_pairs(const ab_bpe* t, std::vector<int32_t>& tokens) {
    const std::vector<std::string>& vocab = t->vocab;
    const size_t n = tokens.size();
    if (n < 2) return;
    for (int32_t id : tokens)
        if (id < 0 || (size_t)id >= vocab.size())
            ab::fail(AB_ERR_ARGUMENT, "token id " + std::to_string(id) +
                                          " has no piece in a vocabulary of " +
                                          std::to_string(vocab.size()));
    // node k: the token that started at position k (merges keep the left position)
    std::vector<int32_t> tok(tokens), prev(n), next(n);
    std::vector<uint32_t> ver(n, 0);
    std::vector<char> alive(n, 1);
    for (size_t k = 0; k < n; k++) {
        prev[k] = (int32_t)k - 1;
        next[k] = k + 1 < n ? (int32_t)(k + 1) : -1;
    }
    struct Cand {
        float score;
        int32_t left, right, id;
        uint32_t vl, vr;
    };
    auto worse = [](const Cand& a, const Cand& b) {
        return a.score < b.score || (a.score == b.score && a.left > b.left);
    };
    std::priority_queue<Cand, std::vector<Cand>, decltype(worse)> heap(worse);
    auto push = [&](int32_t l) {
        if (l < 0) return;
        const int32_t r = next[l];
        if (r < 0) return;
        const int32_t id = lookup(t, vocab[tok[l]] + vocab[tok[r]]);
        if (id < 0) return;
        const float sc = t->scores[id];
        if (!(sc > -1e10f)) return;  // the reference's best_score starts at -1e10
        heap.push({sc, l, r, id, ver[l], ver[r]});
    };
    for (size_t k = 0; k + 1 < n; k++) push((int32_t)k);
    while (!heap.empty()) {
        const Cand c = heap.top();
        heap.pop();
        if (!alive[c.left] || !alive[c.right] || next[c.left] != c.right ||
            ver[c.left] != c.vl || ver[c.right] != c.vr)
            continue;
        tok[c.left] = c.id;
        ver[c.left]++;
        alive[c.right] = 0;
        next[c.left] = next[c.right];
        if (next[c.right] >= 0) prev[next[c.right]] = c.left;
        push(prev[c.left]);
        push(c.left);
    }
    tokens.clear();
    for (int32_t k = 0; k >= 0; k = next[k]) tokens.push_back(tok[k]);
}

std::vector<int32_t> encode_text(const ab_bpe* t, const unsigned char* text, size_t n, bool bos,
                                 bool eos) {
    std::vector<int32_t> tokens;
    tokens.reserve(n + 3);
    if (bos) tokens.push_back(kBos);
    if (n) {
        const int32_t dummy = lookup(t, " ");
        if (dummy >= 0) tokens.push_back(dummy);
    }
    size_t i = 0;
    while (i < n) {
        const size_t start = i++;
        while (i < n && (text[i] & 0xC0) == 0x80 && i - start < 4) i++;
        const size_t len = i - start;
        size_t bad = 0;
        if (utf8_char(text + start, len, &bad) == len) {
            const int32_t id =
                lookup(t, std::string(reinterpret_cast<const char*>(text + start), len));
            if (id >= 0) {
                tokens.push_back(id);
                continue;
            }
        }
        for (size_t k = start; k < i; k++) tokens.push_back((int32_t)text[k] + 3);
    }
    merge_pairs(t, tokens);
    if (eos) tokens.push_back(kEos);
    return tokens;
}

std::string decode_piece(const ab_bpe* t, int32_t prev_token, int32_t token) {
    std::string piece =
        token >= 0 && (size_t)token < t->vocab.size() ? t->vocab[token] : std::string();
    if (prev_token == kBos && !piece.empty() && piece[0] == ' ') piece.erase(0, 1);
    unsigned b;
    if (parse_byte_token(piece, &b)) {
        std::string out;
        if (b < 0x80) {
            out.push_back((char)b);
        } else {
            out.push_back((char)(0xC0 | (b >> 6)));
            out.push_back((char)(0x80 | (b & 0x3F)));
        }
        return out;
    }
    return piece;
}

}  // namespace

using namespace ab;

extern "C" {

int ab_bpe_from_path(const char* path, uint32_t vocab_size, ab_bpe** out) {
    return guard([&] {
        if (!path || !out) fail(AB_ERR_ARGUMENT, "null argument");
        FILE* f = std::fopen(path, "rb");
        if (!f) fail(AB_ERR_ARGUMENT, std::string("open tokenizer ") + path);
        auto* t = new ab_bpe();
        auto take = [&](void* dst, size_t n, const std::string& what) {
            if (std::fread(dst, 1, n, f) != n) fail(AB_ERR_ARGUMENT, "read tokenizer " + what);
        };
        try {
            take(&t->max_token_length, 4, "max_token_length");
            t->vocab.reserve(vocab_size);
            t->scores.reserve(vocab_size);
            std::vector<unsigned char> buf;
            for (uint32_t i = 0; i < vocab_size; i++) {
                float score;
                int32_t len;
                take(&score, 4, "score " + std::to_string(i));
                take(&len, 4, "length " + std::to_string(i));
                if (len < 0)
                    fail(AB_ERR_ARGUMENT, "tokenizer piece " + std::to_string(i) +
                                              " has negative length " + std::to_string(len));
                buf.resize((size_t)len);
                if (len) take(buf.data(), (size_t)len, "piece " + std::to_string(i));
                t->scores.push_back(score);
                t->vocab.push_back(utf8_lossy(buf.data(), buf.size()));
            }
            index_pieces(t);
        } catch (...) {
            std::fclose(f);
            delete t;
            throw;
        }
        std::fclose(f);
        *out = t;
    });
}

int ab_bpe_from_parts(const char* const* pieces, const uint32_t* lengths, const float* scores,
                      uint32_t n, uint32_t max_token_length, ab_bpe** out) {
    return guard([&] {
        if (!out || (n && (!pieces || !lengths || !scores))) fail(AB_ERR_ARGUMENT, "null argument");
        auto* t = new ab_bpe();
        try {
            t->max_token_length = max_token_length;
            t->vocab.reserve(n);
            for (uint32_t i = 0; i < n; i++) {
                if (lengths[i] && !pieces[i]) fail(AB_ERR_ARGUMENT, "null piece");
                t->vocab.push_back(
                    utf8_lossy(reinterpret_cast<const unsigned char*>(pieces[i]), lengths[i]));
            }
            t->scores.assign(scores, scores + n);
            index_pieces(t);
        } catch (...) {
            delete t;
            throw;
        }
        *out = t;
    });
}

int ab_bpe_info(const ab_bpe* t, uint32_t* vocab_size, uint32_t* max_token_length) {
    return guard([&] {
        if (!t) fail(AB_ERR_ARGUMENT, "null tokenizer");
        if (vocab_size) *vocab_size = (uint32_t)t->vocab.size();
        if (max_token_length) *max_token_length = t->max_token_length;
    });
}

int ab_bpe_encode(const ab_bpe* t, const char* text, size_t len, int32_t bos, int32_t eos,
                  int32_t* out, uint32_t cap, uint32_t* n_out) {
    return guard([&] {
        if (!t || (len && !text)) fail(AB_ERR_ARGUMENT, "null argument");
        const std::vector<int32_t> ids =
            encode_text(t, reinterpret_cast<const unsigned char*>(text), len, bos != 0, eos != 0);
        if (out) std::memcpy(out, ids.data(), std::min<size_t>(ids.size(), cap) * 4);
        if (n_out) *n_out = (uint32_t)ids.size();
    });
}

int ab_bpe_decode(const ab_bpe* t, int32_t prev_token, int32_t token, char* out, uint32_t cap,
                  uint32_t* n_out) {
    return guard([&] {
        if (!t) fail(AB_ERR_ARGUMENT, "null tokenizer");
        const std::string s = decode_piece(t, prev_token, token);
        if (out && cap) std::memcpy(out, s.data(), std::min<size_t>(s.size(), cap));
        if (n_out) *n_out = (uint32_t)s.size();
    });
}

int ab_bpe_destroy(ab_bpe* t) {
    delete t;
    return AB_OK;
}

}  // extern "C"
