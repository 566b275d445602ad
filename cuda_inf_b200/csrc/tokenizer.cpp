// Byte-level BPE tokenizer at the reference's tokenizer boundary
// (src/tokenizer.h of g023/cuda_inf): the files written by
// tools/export_tokenizer.py from tokenizer.json,
//   vocab.tsv   <id>\t<token in byte-level unicode>
//   merges.tsv  <rank>\t<left>\t<right>
//   special.tsv <id>\t<literal text>
// and the same text <-> ids behaviour:
//   - special tokens are cut out literally (the earliest occurrence, the
//     longest one when several start there);
//   - the rest is split into pieces by the GPT-2 pre-tokenizer rules as the
//     reference states them (tokenizer.h:104-152: contractions, letter runs
//     with one optional leading non-letter, digit runs of at most 3,
//     punctuation runs with an optional leading space and trailing newlines,
//     whitespace runs); "letter" is an ASCII letter or any non-ASCII
//     non-whitespace code point, as in the reference;
//   - each piece is mapped byte by byte to the GPT-2 byte-level alphabet and
//     BPE-merged by rank (lowest rank first, leftmost pair on ties), unless
//     the whole piece is a vocabulary entry;
//   - decode joins tokens, maps the byte-level symbols back to bytes, and
//     writes special tokens literally unless asked to skip them.
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <unordered_map>
#include <vector>

#include "cuinf.h"

int cuinf_set_arg_error(const char* what);

struct cuinf_tokenizer {
    std::unordered_map<std::string, int> tok2id;
    std::vector<std::string> id2tok;
    std::unordered_map<std::string, int> rank;  // left + '\x01' + right -> merge rank
    std::vector<std::pair<std::string, int>> specials;
    std::unordered_map<int, std::string> special_of;
    std::string sym[256];                        // byte -> byte-level symbol (UTF-8)
    std::unordered_map<std::string, int> byte_of;  // symbol -> byte
};

namespace {

void put_utf8(uint32_t cp, std::string& out) {
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

// Byte length of the UTF-8 sequence a lead byte starts (ill-formed leads
// count as 4, as the reference does).
int utf8_len(unsigned char b) { return b < 0x80 ? 1 : (b >> 5) == 0x6 ? 2 : (b >> 4) == 0xE ? 3 : 4; }

// GPT-2 byte-level alphabet: printable Latin-1 bytes map to themselves, the
// other 68 bytes to U+0100.. in byte order.
void build_alphabet(cuinf_tokenizer* t) {
    int next = 256;
    for (int b = 0; b < 256; b++) {
        const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
        std::string s;
        put_utf8(keep ? (uint32_t)b : (uint32_t)next++, s);
        t->sym[b] = s;
        t->byte_of[s] = b;
    }
}

std::vector<uint32_t> code_points(const std::string& s) {
    std::vector<uint32_t> cps;
    for (size_t i = 0; i < s.size();) {
        const unsigned char b = (unsigned char)s[i];
        const int k = utf8_len(b);
        uint32_t cp = k == 1 ? b : k == 2 ? (b & 0x1F) : k == 3 ? (b & 0x0F) : (b & 0x07);
        for (int j = 1; j < k && i + j < s.size(); j++) cp = (cp << 6) | ((unsigned char)s[i + j] & 0x3F);
        cps.push_back(cp);
        i += k;
    }
    return cps;
}

enum Cls { WS, DIGIT, LETTER, PUNCT };
Cls cls(uint32_t c) {
    if (c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == 0x0B || c == 0x0C || c == 0xA0) return WS;
    if (c >= '0' && c <= '9') return DIGIT;
    if ((c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z') || c >= 0x80) return LETTER;
    return PUNCT;
}
bool is_nl(uint32_t c) { return c == '\n' || c == '\r'; }
uint32_t fold(uint32_t c) { return (c >= 'A' && c <= 'Z') ? c + 32 : c; }

// Piece boundaries [start, end) over code points.
std::vector<std::pair<int, int>> pieces(const std::vector<uint32_t>& c) {
    const int n = (int)c.size();
    std::vector<std::pair<int, int>> out;
    auto letters_from = [&](int j) {
        while (j < n && cls(c[j]) == LETTER) j++;
        return j;
    };
    int i = 0;
    while (i < n) {
        // 's 't 'm 'd 're 've 'll (either case)
        if (c[i] == '\'' && i + 1 < n) {
            const uint32_t a = fold(c[i + 1]);
            int len = 0;
            if (a == 's' || a == 't' || a == 'm' || a == 'd') len = 2;
            else if (i + 2 < n) {
                const uint32_t b2 = fold(c[i + 2]);
                if ((a == 'r' && b2 == 'e') || (a == 'v' && b2 == 'e') || (a == 'l' && b2 == 'l')) len = 3;
            }
            if (len) {
                out.push_back({i, i + len});
                i += len;
                continue;
            }
        }
        const Cls k = cls(c[i]);
        const bool next_letter = i + 1 < n && cls(c[i + 1]) == LETTER;
        if (k == LETTER) {  // a letter run
            const int j = letters_from(i);
            out.push_back({i, j});
            i = j;
            continue;
        }
        if ((k == PUNCT || c[i] == ' ') && next_letter) {  // one leading non-letter, then letters
            const int j = letters_from(i + 1);
            out.push_back({i, j});
            i = j;
            continue;
        }
        if (k == DIGIT) {  // at most three digits
            int j = i;
            while (j < n && j - i < 3 && cls(c[j]) == DIGIT) j++;
            out.push_back({i, j});
            i = j;
            continue;
        }
        {  // optional space, punctuation run, trailing newlines
            const int p = c[i] == ' ' ? i + 1 : i;
            if (p < n && cls(c[p]) == PUNCT) {
                int q = p;
                while (q < n && cls(c[q]) == PUNCT) q++;
                while (q < n && is_nl(c[q])) q++;
                out.push_back({i, q});
                i = q;
                continue;
            }
        }
        if (k == WS) {
            int e = i;
            while (e < n && cls(c[e]) == WS) e++;
            int last_nl = -1;
            for (int j = i; j < e; j++)
                if (is_nl(c[j])) last_nl = j;
            int end;
            if (last_nl >= 0) end = last_nl + 1;          // whitespace up to the last newline
            else if (e == n) end = e;                      // trailing whitespace
            else if (e - 1 > i) end = e - 1;               // leave one space for the next piece
            else end = e;
            out.push_back({i, end});
            i = end;
            continue;
        }
        out.push_back({i, i + 1});
        i++;
    }
    return out;
}

void bpe(const cuinf_tokenizer* t, const std::string& word, std::vector<int>& out) {
    auto whole = t->tok2id.find(word);
    if (whole != t->tok2id.end()) {
        out.push_back(whole->second);
        return;
    }
    std::vector<std::string> s;
    for (size_t i = 0; i < word.size();) {
        const int k = utf8_len((unsigned char)word[i]);
        s.push_back(word.substr(i, k));
        i += k;
    }
    std::string key;
    while (s.size() > 1) {
        int best = -1, best_rank = 0;
        for (size_t j = 0; j + 1 < s.size(); j++) {
            key.assign(s[j]);
            key += '\x01';
            key += s[j + 1];
            auto r = t->rank.find(key);
            if (r != t->rank.end() && (best < 0 || r->second < best_rank)) {
                best = (int)j;
                best_rank = r->second;
            }
        }
        if (best < 0) break;
        s[best] += s[best + 1];
        s.erase(s.begin() + best + 1);
    }
    for (const std::string& x : s) {
        auto v = t->tok2id.find(x);
        if (v != t->tok2id.end()) out.push_back(v->second);
    }
}

// Lines of a tab-separated file, each split at its first `fields - 1` tabs.
bool read_tsv(const std::string& path, int fields, std::vector<std::vector<std::string>>& rows) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return false;
    std::string line;
    int ch;
    auto flush = [&]() {
        std::vector<std::string> r;
        size_t start = 0;
        for (int k = 0; k < fields - 1; k++) {
            const size_t tab = line.find('\t', start);
            if (tab == std::string::npos) return;
            r.push_back(line.substr(start, tab - start));
            start = tab + 1;
        }
        r.push_back(line.substr(start));
        rows.push_back(std::move(r));
    };
    while ((ch = fgetc(f)) != EOF) {
        if (ch == '\n') {
            flush();
            line.clear();
        } else {
            line += (char)ch;
        }
    }
    if (!line.empty()) flush();
    fclose(f);
    return true;
}

}  // namespace

extern "C" int cuinf_tokenizer_load(const char* dir, cuinf_tokenizer** out) {
    if (!dir || !out) return cuinf_set_arg_error("null pointer");
    const std::string d(dir);
    std::vector<std::vector<std::string>> voc, mer, spe;
    if (!read_tsv(d + "/vocab.tsv", 2, voc)) return cuinf_set_arg_error("cannot read vocab.tsv");
    if (!read_tsv(d + "/merges.tsv", 3, mer)) return cuinf_set_arg_error("cannot read merges.tsv");
    if (!read_tsv(d + "/special.tsv", 2, spe)) return cuinf_set_arg_error("cannot read special.tsv");
    cuinf_tokenizer* t = new cuinf_tokenizer();
    build_alphabet(t);
    int max_id = -1;
    for (auto& r : voc) {
        const int id = atoi(r[0].c_str());
        t->tok2id[r[1]] = id;
        max_id = std::max(max_id, id);
    }
    t->id2tok.assign(max_id + 1, std::string());
    for (auto& r : voc) {
        const int id = atoi(r[0].c_str());
        if (id >= 0) t->id2tok[id] = r[1];
    }
    for (auto& r : mer) t->rank[r[1] + '\x01' + r[2]] = atoi(r[0].c_str());
    for (auto& r : spe) {
        const int id = atoi(r[0].c_str());
        t->specials.push_back({r[1], id});
        t->special_of[id] = r[1];
    }
    std::stable_sort(t->specials.begin(), t->specials.end(),
                     [](const std::pair<std::string, int>& a, const std::pair<std::string, int>& b) {
                         return a.first.size() > b.first.size();
                     });
    *out = t;
    return CUINF_OK;
}

extern "C" int cuinf_tokenizer_free(cuinf_tokenizer* t) {
    delete t;
    return CUINF_OK;
}

extern "C" int cuinf_tokenizer_vocab_size(const cuinf_tokenizer* t) { return t ? (int)t->id2tok.size() : -1; }

extern "C" int cuinf_tokenizer_encode(const cuinf_tokenizer* t, const char* text, size_t len, int* ids, int cap,
                                      int* n_out) {
    if (!t || (!text && len) || !n_out || (cap > 0 && !ids)) return cuinf_set_arg_error("null pointer");
    const std::string s(text ? text : "", len);
    std::vector<int> out;
    size_t pos = 0;
    while (pos < s.size()) {
        size_t at = std::string::npos, slen = 0;
        int sid = -1;
        for (auto& sp : t->specials) {  // longest first: a longer one at the same place wins
            if (sp.first.empty()) continue;
            const size_t f = s.find(sp.first, pos);
            if (f != std::string::npos && (f < at || (f == at && sp.first.size() > slen))) {
                at = f;
                slen = sp.first.size();
                sid = sp.second;
            }
        }
        const size_t end = at == std::string::npos ? s.size() : at;
        if (end > pos) {
            const std::vector<uint32_t> cps = code_points(s.substr(pos, end - pos));
            for (auto& p : pieces(cps)) {
                std::string raw, word;
                for (int k = p.first; k < p.second; k++) put_utf8(cps[k], raw);
                for (unsigned char b : raw) word += t->sym[b];
                bpe(t, word, out);
            }
        }
        if (at == std::string::npos) break;
        out.push_back(sid);
        pos = at + slen;
    }
    const int n = (int)out.size();
    for (int i = 0; i < n && i < cap; i++) ids[i] = out[i];
    *n_out = n;
    return CUINF_OK;
}

extern "C" int cuinf_tokenizer_decode(const cuinf_tokenizer* t, const int* ids, int n, int skip_special, char* out,
                                      size_t cap, size_t* len_out) {
    if (!t || (n > 0 && !ids) || !len_out || (cap > 0 && !out)) return cuinf_set_arg_error("null pointer");
    std::string res, pend;
    auto to_bytes = [&](const std::string& bl) {
        for (size_t i = 0; i < bl.size();) {
            const int k = utf8_len((unsigned char)bl[i]);
            auto b = t->byte_of.find(bl.substr(i, k));
            if (b != t->byte_of.end()) res += (char)b->second;
            i += k;
        }
    };
    for (int i = 0; i < n; i++) {
        auto sp = t->special_of.find(ids[i]);
        if (sp != t->special_of.end()) {
            to_bytes(pend);
            pend.clear();
            if (!skip_special) res += sp->second;
            continue;
        }
        if (ids[i] >= 0 && ids[i] < (int)t->id2tok.size()) pend += t->id2tok[ids[i]];
    }
    to_bytes(pend);
    memcpy(out, res.data(), std::min(cap, res.size()));
    *len_out = res.size();
    return CUINF_OK;
}

// The reference's single-turn chat template (engine.cu:697-699).
extern "C" int cuinf_chat_prompt(const char* user, char* out, size_t cap, size_t* len_out) {
    if (!user || !len_out || (cap > 0 && !out)) return cuinf_set_arg_error("null pointer");
    const std::string s = std::string("<|startoftext|><|im_start|>user\n") + user + "<|im_end|>\n<|im_start|>assistant\n";
    memcpy(out, s.data(), std::min(cap, s.size()));
    *len_out = s.size();
    return CUINF_OK;
}
