// g2_tokenizer.cpp -- GPT-2 byte-level BPE tokenizer for the text path of the
// command-line program (the reference's tokenizer.c:442-579, same results).
//
//  * vocab.json: a JSON object of token string -> id (\uXXXX escapes and
//    surrogate pairs decoded to UTF-8); merges.txt: one "left right" pair per
//    line in rank order after an optional "#version" line (tokenizer.c:227-330).
//  * Bytes map to code points with GPT-2's bytes_to_unicode table: printable
//    Latin-1 bytes map to themselves, the other 68 to 256, 257, ... in byte
//    order (tokenizer.c:332-347).
//  * Pre-tokenization is the reference's ASCII-class scan (tokenizer.c:476-549):
//    contractions 's 't 'm 'd 're 've 'll; a space followed by a letter run,
//    digit run or punctuation run; bare letter / digit / punctuation runs; any
//    other whitespace one character at a time.
//  * Each pre-token's symbols are merged pair by pair: every pass finds the
//    lowest-ranked adjacent pair present and merges all its non-overlapping
//    occurrences left to right (tokenizer.c:360-421); symbols missing from the
//    vocabulary are dropped.
//  * Decoding maps each code point of a token string back to its byte ('?' for
//    code points outside the table) (tokenizer.c:552-579).
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "gpt2b200.h"

struct g2_tokenizer {
    std::unordered_map<std::string, int> vocab;   // byte-level string -> id
    std::unordered_map<std::string, int> ranks;   // "left right" -> merge rank
    std::vector<std::string> id_str;              // id -> byte-level string ("" if unused)
    int byte_cp[256];
    int cp_byte[512];
};

namespace {

void put_utf8(std::string &out, int cp) {
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

// One UTF-8 code point at s[i..n); returns its length, 0 if malformed.
int get_utf8(const std::string &s, size_t i, int *cp) {
    const unsigned char c = (unsigned char)s[i];
    auto cont = [&](size_t k) { return k < s.size() ? ((unsigned char)s[k] & 0x3F) : 0; };
    if (c < 0x80) {
        *cp = c;
        return 1;
    }
    if ((c & 0xE0) == 0xC0) {
        *cp = ((c & 0x1F) << 6) | cont(i + 1);
        return 2;
    }
    if ((c & 0xF0) == 0xE0) {
        *cp = ((c & 0x0F) << 12) | (cont(i + 1) << 6) | cont(i + 2);
        return 3;
    }
    if ((c & 0xF8) == 0xF0) {
        *cp = ((c & 0x07) << 18) | (cont(i + 1) << 12) | (cont(i + 2) << 6) | cont(i + 3);
        return 4;
    }
    return 0;
}

bool read_file(const std::string &path, std::string &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
    fclose(f);
    return true;
}

int hexval(char h) {
    if (h >= '0' && h <= '9') return h - '0';
    if (h >= 'a' && h <= 'f') return h - 'a' + 10;
    if (h >= 'A' && h <= 'F') return h - 'A' + 10;
    return -1;
}
bool hex4(const std::string &s, size_t at, int *v) {
    if (at + 4 > s.size()) return false;
    int x = 0;
    for (size_t k = at; k < at + 4; ++k) {
        const int h = hexval(s[k]);
        if (h < 0) return false;
        x = x * 16 + h;
    }
    *v = x;
    return true;
}

// JSON string starting at s[i] == '"'; on success i is past the closing quote.
bool json_string(const std::string &s, size_t &i, std::string &out) {
    if (i >= s.size() || s[i] != '"') return false;
    ++i;
    out.clear();
    while (i < s.size() && s[i] != '"') {
        char c = s[i];
        if (c != '\\') {
            out += c;
            ++i;
            continue;
        }
        if (++i >= s.size()) return false;
        const char e = s[i];
        switch (e) {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u': {
                int cp;
                if (!hex4(s, i + 1, &cp)) return false;
                i += 4;
                int lo;
                if (cp >= 0xD800 && cp <= 0xDBFF && i + 6 < s.size() && s[i + 1] == '\\' && s[i + 2] == 'u' &&
                    hex4(s, i + 3, &lo) && lo >= 0xDC00 && lo <= 0xDFFF) {
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    i += 6;
                }
                put_utf8(out, cp);
                break;
            }
            default: return false;
        }
        ++i;
    }
    if (i >= s.size()) return false;
    ++i;
    return true;
}

bool load_vocab(g2_tokenizer *t, const std::string &path) {
    std::string s;
    if (!read_file(path, s)) return false;
    size_t i = 0;
    auto ws = [&](bool comma) {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r' || (comma && s[i] == ',')))
            ++i;
    };
    ws(false);
    if (i >= s.size() || s[i] != '{') return false;
    ++i;
    std::string key;
    for (;;) {
        ws(true);
        if (i >= s.size() || s[i] == '}') break;
        if (!json_string(s, i, key)) return false;
        while (i < s.size() && (s[i] == ' ' || s[i] == '\t')) ++i;
        if (i >= s.size() || s[i] != ':') return false;
        ++i;
        while (i < s.size() && (s[i] == ' ' || s[i] == '\t')) ++i;
        long long id = 0;
        while (i < s.size() && s[i] >= '0' && s[i] <= '9' && id < INT_MAX) id = id * 10 + (s[i++] - '0');
        if (id >= INT_MAX / 2) return false;
        t->vocab[key] = (int)id;
        if ((size_t)id >= t->id_str.size()) t->id_str.resize((size_t)id + 1);
        t->id_str[(size_t)id] = key;
    }
    return true;
}

bool load_merges(g2_tokenizer *t, const std::string &path) {
    std::string s;
    if (!read_file(path, s)) return false;
    size_t i = 0;
    if (!s.empty() && s[0] == '#') {   // "#version: 0.2"
        while (i < s.size() && s[i] != '\n') ++i;
        if (i < s.size()) ++i;
    }
    int rank = 0;
    while (i < s.size()) {
        size_t e = s.find('\n', i);
        if (e == std::string::npos) e = s.size();
        size_t le = e;
        while (le > i && s[le - 1] == '\r') --le;
        const size_t sp = s.find(' ', i);
        if (le > i && sp != std::string::npos && sp < le) {
            // key "left right" (split at the first space); a repeated pair takes its later rank
            t->ranks[s.substr(i, le - i)] = rank++;
        }
        i = e + 1;
    }
    return true;
}

void byte_tables(g2_tokenizer *t) {
    for (int &v : t->cp_byte) v = -1;
    int extra = 0;
    for (int b = 0; b < 256; ++b) {
        const bool printable = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
        const int cp = printable ? b : 256 + extra++;
        t->byte_cp[b] = cp;
        t->cp_byte[cp] = b;
    }
}

// Merge rank of the adjacent pair (a, b), or -1.  Pairs whose key would exceed
// 512 bytes never merge (the reference's fixed key buffer, tokenizer.c:349-358).
int rank_of(const g2_tokenizer *t, const std::string &a, const std::string &b) {
    if (a.size() + 1 + b.size() > 512) return -1;
    std::string key;
    key.reserve(a.size() + 1 + b.size());
    key += a;
    key += ' ';
    key += b;
    auto it = t->ranks.find(key);
    return it == t->ranks.end() ? -1 : it->second;
}

// BPE of one pre-token (raw bytes text[0..n)), ids appended while there is room.
void bpe(const g2_tokenizer *t, const char *text, int n, std::vector<int> &ids, int max_ids) {
    std::vector<std::string> sym(n);
    for (int k = 0; k < n; ++k) put_utf8(sym[k], t->byte_cp[(unsigned char)text[k]]);
    std::vector<std::string> next;
    while (sym.size() > 1) {
        int best = INT_MAX;
        for (size_t k = 0; k + 1 < sym.size(); ++k) {
            const int r = rank_of(t, sym[k], sym[k + 1]);
            if (r >= 0 && r < best) best = r;
        }
        if (best == INT_MAX) break;
        next.clear();
        for (size_t k = 0; k < sym.size();) {
            if (k + 1 < sym.size() && rank_of(t, sym[k], sym[k + 1]) == best) {
                next.push_back(sym[k] + sym[k + 1]);
                k += 2;
            } else {
                next.push_back(sym[k]);
                k += 1;
            }
        }
        sym.swap(next);
    }
    for (const std::string &p : sym) {
        auto it = t->vocab.find(p);
        if (it != t->vocab.end() && (int)ids.size() < max_ids) ids.push_back(it->second);
    }
}

bool is_letter(char c) { return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z'); }
bool is_digit(char c) { return c >= '0' && c <= '9'; }
bool is_space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f' || c == '\v'; }
bool is_punct(char c) { return !is_space(c) && !is_letter(c) && !is_digit(c); }

// Length of the contraction at p[0..n) ('s 't 'm 'd 're 've 'll), or 0.
int contraction(const char *p, int n) {
    if (n < 2 || p[0] != '\'') return 0;
    const char a = p[1];
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
    if (n >= 3) {
        const char b = p[2];
        if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
    }
    return 0;
}

}  // namespace

extern "C" int g2_tokenizer_load(const char *dir, g2_tokenizer **out) {
    if (!dir || !out) return G2_ERR_ARG;
    *out = nullptr;
    g2_tokenizer *t = new g2_tokenizer();
    byte_tables(t);
    const std::string d(dir);
    if (!load_vocab(t, d + "/vocab.json") || !load_merges(t, d + "/merges.txt")) {
        delete t;
        return G2_ERR_IO;
    }
    *out = t;
    return G2_OK;
}

extern "C" void g2_tokenizer_free(g2_tokenizer *t) { delete t; }

extern "C" int g2_tokenizer_vocab_size(const g2_tokenizer *t) { return t ? (int)t->id_str.size() : 0; }

extern "C" int g2_tok_encode(const g2_tokenizer *t, const char *text, int *ids, int max_ids) {
    if (!t || !text || !ids || max_ids <= 0) return G2_ERR_ARG;
    const int len = (int)strlen(text);
    std::vector<int> out;
    out.reserve(max_ids);
    int i = 0;
    while (i < len && (int)out.size() < max_ids) {
        const char c = text[i];
        int j;
        const int cl = c == '\'' ? contraction(text + i, len - i) : 0;
        if (cl > 0) {
            j = i + cl;
        } else if (c == ' ' && i + 1 < len && !is_space(text[i + 1])) {
            const char c2 = text[i + 1];
            bool (*same)(char) = is_letter(c2) ? is_letter : is_digit(c2) ? is_digit : is_punct;
            j = i + 1;
            while (j < len && same(text[j])) ++j;
        } else if (!is_space(c)) {
            bool (*same)(char) = is_letter(c) ? is_letter : is_digit(c) ? is_digit : is_punct;
            j = i;
            while (j < len && same(text[j])) ++j;
        } else {
            j = i + 1;   // whitespace: one character at a time
        }
        bpe(t, text + i, j - i, out, max_ids);
        i = j;
    }
    memcpy(ids, out.data(), out.size() * sizeof(int));
    return (int)out.size();
}

extern "C" int g2_tok_decode(const g2_tokenizer *t, const int *ids, int n, char *out, int max_bytes) {
    if (!t || !ids || !out || max_bytes <= 0 || n < 0) return G2_ERR_ARG;
    int w = 0;
    for (int k = 0; k < n; ++k) {
        const int id = ids[k];
        if (id < 0 || id >= (int)t->id_str.size()) continue;
        const std::string &s = t->id_str[(size_t)id];
        for (size_t j = 0; j < s.size();) {
            int cp;
            const int used = get_utf8(s, j, &cp);
            if (used <= 0) break;
            int b = cp >= 0 && cp < 512 ? t->cp_byte[cp] : -1;
            if (b < 0) b = '?';
            if (w >= max_bytes - 1) {
                out[w] = 0;
                return w;
            }
            out[w++] = (char)b;
            j += (size_t)used;
        }
    }
    out[w] = 0;
    return w;
}
