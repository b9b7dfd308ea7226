// bpe.cpp -- byte-level BPE tokenizer: the GPT-4 split pattern followed by
// greedy lowest-rank merges, behind the C ABI of the reference's Rust
// tokenizer (src/rust_tokenizer/src/lib.rs:8-123, bound from Python by
// src/rust_tokenizer.py).  Host code (C++17), no GPU.
//
// The split pattern of the reference (lib.rs:8-9),
//   '(?i:[sdmt]|ll|ve|re) | [^\r\n\p{L}\p{N}]?+\p{L}+ | \p{N}{1,3}
//   | ' '?[^\s\p{L}\p{N}]+[\r\n]* | \s*[\r\n] | \s+(?!\S) | \s+
// is matched by hand below, alternative by alternative in the order a
// backtracking engine tries them (leftmost-first: the first alternative that
// matches at a position wins, not the longest); the character classes come
// from unicode_classes.h.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/mi_bpe.h"
#include "unicode_classes.h"

namespace mi_bpe {

static bool in_ranges(uint32_t cp, const uint32_t (*r)[2], int n) {
    int lo = 0, hi = n - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        if (cp < r[mid][0]) hi = mid - 1;
        else if (cp > r[mid][1]) lo = mid + 1;
        else return true;
    }
    return false;
}
static inline bool is_letter(uint32_t cp) {
    if (cp < 0x80) return (cp | 0x20) >= 'a' && (cp | 0x20) <= 'z';
    return in_ranges(cp, kLetterRanges, kLetterCount);
}
static inline bool is_number(uint32_t cp) {
    if (cp < 0x80) return cp >= '0' && cp <= '9';
    return in_ranges(cp, kNumberRanges, kNumberCount);
}
static inline bool is_space(uint32_t cp) { return in_ranges(cp, kSpaceRanges, kSpaceCount); }
static inline bool is_crlf(uint32_t cp) { return cp == '\r' || cp == '\n'; }
// [^\s\p{L}\p{N}]
static inline bool is_other(uint32_t cp) { return !is_space(cp) && !is_letter(cp) && !is_number(cp); }

// Strict UTF-8 (what a Rust &str holds): code points and the byte offset of
// each (offs has one more entry, the total length).  False on invalid input.
static bool utf8_decode(const unsigned char* s, size_t len, std::vector<uint32_t>& cps, std::vector<size_t>& offs) {
    cps.clear();
    offs.clear();
    size_t i = 0;
    while (i < len) {
        const unsigned char b0 = s[i];
        uint32_t cp;
        size_t n;
        if (b0 < 0x80) { cp = b0; n = 1; }
        else if ((b0 & 0xE0) == 0xC0) { cp = b0 & 0x1F; n = 2; }
        else if ((b0 & 0xF0) == 0xE0) { cp = b0 & 0x0F; n = 3; }
        else if ((b0 & 0xF8) == 0xF0) { cp = b0 & 0x07; n = 4; }
        else return false;
        if (i + n > len) return false;
        for (size_t k = 1; k < n; k++) {
            if ((s[i + k] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (s[i + k] & 0x3F);
        }
        static const uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
        if (cp < kMin[n] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
        cps.push_back(cp);
        offs.push_back(i);
        i += n;
    }
    offs.push_back(len);
    return true;
}

// End (code-point index) of the match that starts at i.
static size_t match_at(const std::vector<uint32_t>& c, size_t i) {
    const size_t n = c.size();
    // '(?i:[sdmt]|ll|ve|re)  -- simple case folding adds U+017F (long s) to s
    if (c[i] == '\'' && i + 1 < n) {
        const uint32_t a = c[i + 1];
        if (a == 's' || a == 'S' || a == 0x17F || a == 'd' || a == 'D' || a == 'm' || a == 'M' || a == 't' ||
            a == 'T')
            return i + 2;
        if (i + 2 < n) {
            const uint32_t b = c[i + 2];
            const bool e = b == 'e' || b == 'E';
            if ((a == 'l' || a == 'L') && (b == 'l' || b == 'L')) return i + 3;
            if ((a == 'v' || a == 'V') && e) return i + 3;
            if ((a == 'r' || a == 'R') && e) return i + 3;
        }
    }
    // [^\r\n\p{L}\p{N}]?+\p{L}+  (the optional character is possessive: taken whenever it matches)
    {
        size_t j = i;
        if (!is_crlf(c[j]) && !is_letter(c[j]) && !is_number(c[j])) j++;
        if (j < n && is_letter(c[j])) {
            while (j < n && is_letter(c[j])) j++;
            return j;
        }
    }
    // \p{N}{1,3}
    if (is_number(c[i])) {
        size_t j = i;
        while (j < n && j - i < 3 && is_number(c[j])) j++;
        return j;
    }
    // ' '?[^\s\p{L}\p{N}]+[\r\n]*  (the space is taken only if an "other" character follows)
    {
        size_t j = i;
        if (c[j] == ' ' && j + 1 < n && is_other(c[j + 1])) j++;
        if (is_other(c[j])) {
            while (j < n && is_other(c[j])) j++;
            while (j < n && is_crlf(c[j])) j++;
            return j;
        }
    }
    if (is_space(c[i])) {
        size_t k = i;
        while (k < n && is_space(c[k])) k++;  // the maximal white-space run [i, k)
        // \s*[\r\n]: the longest prefix of the run that ends in CR or LF
        for (size_t q = k; q > i; q--)
            if (is_crlf(c[q - 1])) return q;
        // \s+(?!\S): the run up to the end, or all of it but the space before the next token
        if (k == n) return k;
        if (k - i >= 2) return k - 1;
        // \s+
        return k;
    }
    return i + 1;  // not reached: every code point is a letter, a number, a space or an "other"
}

struct Tokenizer {
    std::unordered_map<uint64_t, uint32_t> merges;  // (a << 32 | b) -> merged id
};

static inline uint64_t pair_key(uint32_t a, uint32_t b) { return ((uint64_t)a << 32) | b; }

// The pieces of a text, as byte ranges.  False on invalid UTF-8.
static bool split_text(const char* text, size_t len, std::vector<std::pair<size_t, size_t>>& pieces) {
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    if (!utf8_decode(reinterpret_cast<const unsigned char*>(text), len, cps, offs)) return false;
    pieces.clear();
    size_t i = 0;
    while (i < cps.size()) {
        const size_t k = match_at(cps, i);
        pieces.emplace_back(offs[i], offs[k]);
        i = k;
    }
    return true;
}

// Greedy merging of one piece (lib.rs:84-93): repeatedly merge the leftmost
// occurrence of the pair with the lowest merged id.
static void encode_piece(const Tokenizer& t, const unsigned char* b, size_t len, std::vector<uint32_t>& out) {
    std::vector<uint32_t> ids(b, b + len);
    while (ids.size() >= 2) {
        bool found = false;
        size_t bi = 0;
        uint32_t bid = 0;
        for (size_t i = 0; i + 1 < ids.size(); i++) {
            const auto it = t.merges.find(pair_key(ids[i], ids[i + 1]));
            if (it != t.merges.end() && (!found || it->second < bid)) {
                found = true;
                bi = i;
                bid = it->second;
            }
        }
        if (!found) break;
        ids[bi] = bid;
        ids.erase(ids.begin() + (long)bi + 1);
    }
    out.insert(out.end(), ids.begin(), ids.end());
}

}  // namespace mi_bpe

using mi_bpe::Tokenizer;

extern "C" {

Tokenizer* tokenizer_new(void) { return new (std::nothrow) Tokenizer(); }

void tokenizer_free(Tokenizer* t) { delete t; }

int tokenizer_train(Tokenizer* t, const char* input_path, uint32_t vocab_size) {
    if (!t || !input_path) return -1;
    std::ifstream f(input_path, std::ios::binary);
    if (!f) return -1;
    // counts of each piece's byte sequence over the file, line by line (the line
    // terminator, "\n" or "\r\n", is not part of the line)
    std::map<std::vector<uint32_t>, long long> counts;
    std::string line;
    std::vector<std::pair<size_t, size_t>> pieces;
    while (std::getline(f, line)) {
        if (!line.empty() && line.back() == '\r') line.pop_back();
        if (!mi_bpe::split_text(line.data(), line.size(), pieces)) continue;  // invalid UTF-8: skipped
        for (const auto& p : pieces) {
            std::vector<uint32_t> ids;
            for (size_t k = p.first; k < p.second; k++) ids.push_back((unsigned char)line[k]);
            counts[ids] += 1;
        }
    }
    if (vocab_size <= 256) return 0;
    const uint32_t num_merges = vocab_size - 256;
    for (uint32_t i = 0; i < num_merges; i++) {
        std::map<std::pair<uint32_t, uint32_t>, long long> pc;
        for (const auto& kv : counts)
            for (size_t k = 0; k + 1 < kv.first.size(); k++) pc[{kv.first[k], kv.first[k + 1]}] += kv.second;
        if (pc.empty()) break;
        // the most frequent pair; ties go to the smallest pair (the reference's
        // HashMap iteration order decides them arbitrarily)
        auto best = pc.begin();
        for (auto it = pc.begin(); it != pc.end(); ++it)
            if (it->second > best->second) best = it;
        const uint32_t new_id = 256 + i;
        const auto pr = best->first;
        t->merges[mi_bpe::pair_key(pr.first, pr.second)] = new_id;
        std::map<std::vector<uint32_t>, long long> next;
        for (const auto& kv : counts) {
            std::vector<uint32_t> out;
            const auto& ids = kv.first;
            size_t j = 0;
            while (j < ids.size()) {
                if (j + 1 < ids.size() && ids[j] == pr.first && ids[j + 1] == pr.second) {
                    out.push_back(new_id);
                    j += 2;
                } else {
                    out.push_back(ids[j]);
                    j += 1;
                }
            }
            next[out] += kv.second;
        }
        counts.swap(next);
    }
    return 0;
}

uint32_t* tokenizer_encode(Tokenizer* t, const char* text, size_t* out_len) {
    if (out_len) *out_len = 0;
    if (!t || !text || !out_len) return nullptr;
    const size_t len = std::strlen(text);
    std::vector<std::pair<size_t, size_t>> pieces;
    if (!mi_bpe::split_text(text, len, pieces)) return nullptr;  // not UTF-8
    std::vector<uint32_t> all;
    for (const auto& p : pieces)
        mi_bpe::encode_piece(*t, reinterpret_cast<const unsigned char*>(text) + p.first, p.second - p.first, all);
    if (all.empty()) return nullptr;
    uint32_t* res = static_cast<uint32_t*>(std::malloc(all.size() * sizeof(uint32_t)));
    if (!res) return nullptr;
    std::memcpy(res, all.data(), all.size() * sizeof(uint32_t));
    *out_len = all.size();
    return res;
}

void tokenizer_free_ids(uint32_t* ids, size_t len) {
    (void)len;
    std::free(ids);
}

int tokenizer_save(Tokenizer* t, const char* path) {
    if (!t || !path) return -1;
    std::vector<std::pair<uint32_t, uint64_t>> rows;
    for (const auto& kv : t->merges) rows.emplace_back(kv.second, kv.first);
    std::sort(rows.begin(), rows.end());
    FILE* f = std::fopen(path, "w");
    if (!f) return -1;
    for (const auto& r : rows)
        std::fprintf(f, "%u,%u %u\n", (unsigned)(r.second >> 32), (unsigned)(r.second & 0xffffffffu), r.first);
    return std::fclose(f) == 0 ? 0 : -1;
}

int tokenizer_load(Tokenizer* t, const char* path) {
    if (!t || !path) return -1;
    std::ifstream f(path);
    if (!f) return -1;
    std::string line;
    while (std::getline(f, line)) {
        unsigned a, b, id;
        char comma;
        if (line.find_first_not_of(" \t\r") == std::string::npos) continue;
        if (std::sscanf(line.c_str(), "%u%c%u %u", &a, &comma, &b, &id) != 4 || comma != ',') return -1;
        t->merges[mi_bpe::pair_key(a, b)] = id;
    }
    return 0;
}

int mi_bpe_pretokenize(const char* text, size_t* ends, size_t cap, size_t* n_out) {
    if (!text || !n_out) return -1;
    std::vector<std::pair<size_t, size_t>> pieces;
    if (!mi_bpe::split_text(text, std::strlen(text), pieces)) return -1;
    *n_out = pieces.size();
    if (pieces.size() > cap || (!ends && !pieces.empty())) return -2;
    for (size_t i = 0; i < pieces.size(); i++) ends[i] = pieces[i].second;
    return 0;
}

}  // extern "C"
