// ref_tok_harness.cpp — the reference's own Tokenizer (src/tokenizer/tokenizer.cpp, unmodified,
// compiled from the reference tree next to this file's object) behind C functions, so the tests can
// run the product tokenizer and the reference one on the same GGUF files and texts. Test
// infrastructure only: nothing in the product links it.
#include <cstring>
#include <string>
#include <vector>

#include "tokenizer/tokenizer.h"

namespace {
// the last id list a call produced, whole, for ref_tok_last (a caller whose buffer was too small
// fetches it there instead of calling again: the turn helpers change the tokenizer's state)
thread_local std::vector<int> g_last;
int copy_ids(const std::vector<int>& v, int* out, int cap) {
    g_last = v;
    for (int i = 0; i < (int)v.size() && i < cap; ++i) out[i] = v[i];
    return (int)v.size();
}
}  // namespace

extern "C" {
void* ref_tok_load(const char* path) {
    Tokenizer* t = new Tokenizer();
    if (!t->load_from_gguf(path)) {
        delete t;
        return nullptr;
    }
    return t;
}
void ref_tok_free(void* h) { delete static_cast<Tokenizer*>(h); }
void ref_tok_info(void* h, int* fmt, int* bos, int* eos, int* vocab) {
    const Tokenizer* t = static_cast<Tokenizer*>(h);
    *fmt = (int)t->chat_format();
    *bos = t->bos_id();
    *eos = t->eos_id();
    *vocab = t->vocab_size();
}
// Tokenizer::encode; returns the id count (ids beyond cap are not written)
int ref_tok_encode(void* h, const char* text, size_t len, int* out, int cap) {
    return copy_ids(static_cast<Tokenizer*>(h)->encode(std::string(text, len)), out, cap);
}
// Tokenizer::decode(vector); returns the byte count (bytes beyond cap are not written)
size_t ref_tok_decode(void* h, const int* ids, int n, char* out, size_t cap) {
    const std::string s = static_cast<Tokenizer*>(h)->decode(std::vector<int>(ids, ids + n));
    std::memcpy(out, s.data(), s.size() < cap ? s.size() : cap);
    return s.size();
}
int ref_tok_format_chat(void* h, const char* sys, const char* user, int* out, int cap) {
    return copy_ids(static_cast<Tokenizer*>(h)->format_chat(sys, user), out, cap);
}
// One multi-turn helper (0 begin, 1 system, 2 user, 3 assistant header, 4 turn end) on
// tokens[0..n); returns the new count
int ref_tok_append(void* h, int turn, const char* content, int* tokens, int n, int cap) {
    const Tokenizer* t = static_cast<Tokenizer*>(h);
    std::vector<int> v(tokens, tokens + n);
    switch (turn) {
        case 0: t->begin_sequence(v); break;
        case 1: t->append_system_turn(v, content); break;
        case 2: t->append_user_turn(v, content); break;
        case 3: t->append_assistant_header(v); break;
        default: t->append_turn_end(v); break;
    }
    return copy_ids(v, tokens, cap);
}
// copies the last call's ids (up to cap) and returns their count
int ref_tok_last(int* out, int cap) {
    for (int i = 0; i < (int)g_last.size() && i < cap; ++i) out[i] = g_last[i];
    return (int)g_last.size();
}
}
