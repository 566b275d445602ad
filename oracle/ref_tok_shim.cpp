// The reference's own tokenizer (src/tokenizer.h of g023/cuda_inf, included
// unmodified from the reference tree) behind extern "C" entry points, built by
// `make ref` into _ref/libreftok.so.  TEST INFRASTRUCTURE ONLY: tests compare
// cuinf's tokenizer with it.
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "tokenizer.h"

extern "C" void* reftok_load(const char* dir) {
    Tokenizer* t = new Tokenizer();
    if (!t->load(dir)) {
        delete t;
        return nullptr;
    }
    return t;
}
extern "C" void reftok_free(void* t) { delete (Tokenizer*)t; }
extern "C" int reftok_encode(void* t, const char* text, int len, int* ids, int cap) {
    std::vector<int> v = ((Tokenizer*)t)->encode(std::string(text, (size_t)len));
    const int n = (int)v.size();
    for (int i = 0; i < n && i < cap; i++) ids[i] = v[i];
    return n;
}
extern "C" int reftok_decode(void* t, const int* ids, int n, int skip_special, char* out, int cap) {
    std::string s = ((Tokenizer*)t)->decode(std::vector<int>(ids, ids + n), skip_special != 0);
    const int len = (int)s.size();
    memcpy(out, s.data(), (size_t)std::min(len, cap));
    return len;
}
