// tokenizer.cpp — the reference CLI's text side (src/tokenizer/tokenizer.cpp,
// src/model/chat_template.h) behind the C-ABI: byte-level BPE over the GGUF's
// tokenizer.ggml.tokens / tokenizer.ggml.merges, decoding back to bytes, and the ChatML / LLaMA-3 /
// LLaMA-2 / Mistral / raw prompt formats with their multi-turn helpers. Host code only: a prompt is
// tokenised once per turn, so nothing here is on the device path.
//
// Kept as the reference does it (its results are the contract): merges apply to the WHOLE text
// (no pre-tokeniser split), lowest merge rank first and, between equal ranks, the leftmost pair;
// without merges, greedy longest match over at most 128 bytes of the mapped text; a merged symbol
// missing from the vocabulary falls back to its characters, and characters missing too are
// dropped; decoding maps code points back to bytes and writes '?' for unmappable or truncated
// sequences; the ChatML markers are the fixed ids 151644 / 151645, the other formats' markers are
// looked up by name. The merge loop itself is a priority queue over (rank, position) with stale
// entries skipped, which picks the same pair at every step as the reference's full rescan.
#include <cstdint>
#include <cstring>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/fence_b200.h"
#include "gguf.h"

namespace fence {
int set_error(int code, const char* fmt, ...);

namespace {

// GPT-2's byte <-> code point table: printable ASCII and most of Latin-1 keep their value, the other
// 68 bytes take 256, 257, ... in byte order.
struct ByteMap {
    int b2u[256];
    int u2b[512];
    ByteMap() {
        for (int& v : u2b) v = -1;
        int n = 0;
        for (int b = 0; b < 256; ++b) {
            const bool keep = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
            b2u[b] = keep ? b : 256 + n++;
            u2b[b2u[b]] = b;
        }
    }
};
const ByteMap& bytemap() {
    static const ByteMap m;
    return m;
}

void put_utf8(std::string& s, int cp) {  // code points below 0x10000 (the table's range)
    if (cp < 0x80) {
        s += (char)cp;
    } else if (cp < 0x800) {
        s += (char)(0xC0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3F));
    } else {
        s += (char)(0xE0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    }
}

// Length of the UTF-8 character led by byte c, as the reference's splitter counts it (a stray
// continuation byte counts as one).
int utf8_len(unsigned char c) {
    if ((c & 0xE0) == 0xC0) return 2;
    if ((c & 0xF0) == 0xE0) return 3;
    if ((c & 0xF8) == 0xF0) return 4;
    return 1;
}

constexpr int kNoMerge = 1000000000;

}  // namespace
}  // namespace fence

using namespace fence;

struct fence_tokenizer {
    std::vector<std::string> id_to_token;
    std::unordered_map<std::string, int> token_to_id;
    std::unordered_map<std::string, int> merges;  // "left right" -> rank
    int format = FENCE_CHAT_CHATML;
    int bos = 151643, eos = 151645;  // the reference's Qwen defaults, overridden by the GGUF
    int l3_begin = 0, l3_start_hdr = 0, l3_end_hdr = 0, l3_eot = 0;
    int m_bos = 0, m_eos = 0, inst_start = 0, inst_end = 0;
    // multi-turn state (LLaMA-2 / Mistral carry the system prompt into the first user turn)
    std::string pending_system;
    bool system_used = false;

    int lookup(const std::string& s) const {
        auto it = token_to_id.find(s);
        return it == token_to_id.end() ? -1 : it->second;
    }

    // ---- encode (tokenizer.cpp:251-401)
    void bpe(std::vector<std::string>& w) const {
        const int n = (int)w.size();
        if (n < 2) return;
        std::vector<int> prev(n), next(n), ver(n, 0);
        std::vector<char> alive(n, 1);
        for (int i = 0; i < n; ++i) {
            prev[i] = i - 1;
            next[i] = i + 1 < n ? i + 1 : -1;
        }
        struct E {
            int rank, i, j, vi, vj;
            bool operator>(const E& o) const { return rank != o.rank ? rank > o.rank : i > o.i; }
        };
        std::priority_queue<E, std::vector<E>, std::greater<E>> q;
        auto push = [&](int i) {
            if (i < 0 || next[i] < 0) return;
            const int j = next[i];
            auto it = merges.find(w[i] + " " + w[j]);
            if (it != merges.end() && it->second < kNoMerge) q.push({it->second, i, j, ver[i], ver[j]});
        };
        for (int i = 0; i + 1 < n; ++i) push(i);
        while (!q.empty()) {
            const E e = q.top();
            q.pop();
            if (!alive[e.i] || !alive[e.j] || next[e.i] != e.j || ver[e.i] != e.vi || ver[e.j] != e.vj) continue;
            w[e.i] += w[e.j];
            ++ver[e.i];
            alive[e.j] = 0;
            next[e.i] = next[e.j];
            if (next[e.j] >= 0) prev[next[e.j]] = e.i;
            push(prev[e.i]);
            push(e.i);
        }
        std::vector<std::string> out;
        for (int i = 0; i >= 0; i = next[i]) out.push_back(std::move(w[i]));
        w = std::move(out);
    }

    std::vector<int> encode(const std::string& text) const {
        const ByteMap& bm = bytemap();
        std::string u;
        for (unsigned char c : text) put_utf8(u, bm.b2u[c]);
        std::vector<std::string> words;
        if (!merges.empty()) {
            for (size_t i = 0; i < u.size();) {
                const int l = utf8_len((unsigned char)u[i]);
                words.push_back(u.substr(i, l));
                i += l;
            }
            bpe(words);
        } else {  // no merge table: greedy longest match, at most 128 bytes at a time
            for (size_t pos = 0; pos < u.size();) {
                size_t len = std::min<size_t>(u.size() - pos, 128);
                for (; len > 0; --len)
                    if (token_to_id.count(u.substr(pos, len))) break;
                if (len == 0) len = 1;
                words.push_back(u.substr(pos, len));
                pos += len;
            }
        }
        std::vector<int> ids;
        for (const std::string& w : words) {
            const int id = lookup(w);
            if (id >= 0) {
                ids.push_back(id);
                continue;
            }
            for (size_t i = 0; i < w.size();) {  // per-character fallback; unknown characters are dropped
                const int l = utf8_len((unsigned char)w[i]);
                const int c = lookup(w.substr(i, l));
                if (c >= 0) ids.push_back(c);
                i += l;
            }
        }
        return ids;
    }

    // ---- decode (tokenizer.cpp:71-118, 403-414)
    std::string decode(int id) const {
        if (id < 0 || id >= (int)id_to_token.size()) return "";
        const ByteMap& bm = bytemap();
        const std::string& s = id_to_token[id];
        std::string out;
        const size_t n = s.size();
        for (size_t i = 0; i < n;) {
            const unsigned char c = (unsigned char)s[i];
            int cp, l;
            if (c < 0x80) {
                cp = c;
                l = 1;
            } else if ((c & 0xE0) == 0xC0) {
                if (i + 1 >= n) { out += '?'; ++i; continue; }
                cp = ((c & 0x1F) << 6) | ((unsigned char)s[i + 1] & 0x3F);
                l = 2;
            } else if ((c & 0xF0) == 0xE0) {
                if (i + 2 >= n) { out += '?'; ++i; continue; }
                cp = ((c & 0x0F) << 12) | (((unsigned char)s[i + 1] & 0x3F) << 6) | ((unsigned char)s[i + 2] & 0x3F);
                l = 3;
            } else {
                if (i + 3 >= n) { out += '?'; ++i; continue; }
                cp = ((c & 0x07) << 18) | (((unsigned char)s[i + 1] & 0x3F) << 12) |
                     (((unsigned char)s[i + 2] & 0x3F) << 6) | ((unsigned char)s[i + 3] & 0x3F);
                l = 4;
            }
            i += l;
            out += (cp >= 0 && cp < 512 && bm.u2b[cp] >= 0) ? (char)bm.u2b[cp] : '?';
        }
        return out;
    }

    void push(std::vector<int>& t, const std::string& text) const {
        const std::vector<int> ids = encode(text);
        t.insert(t.end(), ids.begin(), ids.end());
    }

    // ---- chat formats (tokenizer.cpp:410-627, chat_template.h:36-60)
    static int detect(const std::string& arch, const std::string& tmpl) {
        if (!tmpl.empty()) {
            if (tmpl.find("im_start") != std::string::npos) return FENCE_CHAT_CHATML;
            if (tmpl.find("begin_of_text") != std::string::npos || tmpl.find("start_header_id") != std::string::npos)
                return FENCE_CHAT_LLAMA3;
            if (tmpl.find("<<SYS>>") != std::string::npos) return FENCE_CHAT_LLAMA2;
            if (tmpl.find("[INST]") != std::string::npos) return FENCE_CHAT_MISTRAL;
        }
        if (arch == "qwen2" || arch == "qwen3" || arch == "internlm2" || arch == "deepseek2") return FENCE_CHAT_CHATML;
        if (arch == "llama") return FENCE_CHAT_LLAMA3;
        if (arch == "mistral" || arch == "mixtral") return FENCE_CHAT_MISTRAL;
        return FENCE_CHAT_RAW;
    }

    void begin(std::vector<int>& t) {
        system_used = false;
        pending_system.clear();
        if (format == FENCE_CHAT_LLAMA3 && l3_begin > 0) t.push_back(l3_begin);
        if ((format == FENCE_CHAT_LLAMA2 || format == FENCE_CHAT_MISTRAL) && m_bos > 0) t.push_back(m_bos);
    }
    void llama3_turn(std::vector<int>& t, const char* role, const std::string& content) const {
        if (l3_start_hdr > 0) t.push_back(l3_start_hdr);
        push(t, role);
        if (l3_end_hdr > 0) t.push_back(l3_end_hdr);
        push(t, "\n\n" + content);
        if (l3_eot > 0) t.push_back(l3_eot);
    }
    void system_turn(std::vector<int>& t, const std::string& content) {
        switch (format) {
            case FENCE_CHAT_CHATML:
                t.push_back(kImStart);
                push(t, "system\n" + content);
                t.push_back(kImEnd);
                push(t, "\n");
                break;
            case FENCE_CHAT_LLAMA3: llama3_turn(t, "system", content); break;
            case FENCE_CHAT_LLAMA2:
            case FENCE_CHAT_MISTRAL: pending_system = content; break;  // goes into the first [INST] block
            default: push(t, content + "\n"); break;
        }
    }
    void user_turn(std::vector<int>& t, const std::string& content) {
        switch (format) {
            case FENCE_CHAT_CHATML:
                t.push_back(kImStart);
                push(t, "user\n" + content);
                t.push_back(kImEnd);
                push(t, "\n");
                break;
            case FENCE_CHAT_LLAMA3: llama3_turn(t, "user", content); break;
            case FENCE_CHAT_LLAMA2:
            case FENCE_CHAT_MISTRAL:
                if (inst_start > 0) t.push_back(inst_start);
                if (!pending_system.empty() && !system_used) {
                    push(t, format == FENCE_CHAT_LLAMA2 ? " <<SYS>>\n" + pending_system + "\n<</SYS>>\n\n"
                                                        : " " + pending_system + "\n\n");
                    system_used = true;
                } else {
                    push(t, " ");
                }
                push(t, content + " ");
                if (inst_end > 0) t.push_back(inst_end);
                break;
            default: push(t, content + "\n"); break;
        }
    }
    void assistant_header(std::vector<int>& t) const {
        switch (format) {
            case FENCE_CHAT_CHATML:
                t.push_back(kImStart);
                push(t, "assistant\n");
                break;
            case FENCE_CHAT_LLAMA3:
                if (l3_start_hdr > 0) t.push_back(l3_start_hdr);
                push(t, "assistant");
                if (l3_end_hdr > 0) t.push_back(l3_end_hdr);
                push(t, "\n\n");
                break;
            case FENCE_CHAT_LLAMA2:
            case FENCE_CHAT_MISTRAL: push(t, " "); break;
            default: break;
        }
    }
    void turn_end(std::vector<int>& t) const {
        switch (format) {
            case FENCE_CHAT_CHATML:
                t.push_back(kImEnd);
                push(t, "\n");
                break;
            case FENCE_CHAT_LLAMA3:
                if (l3_eot > 0) t.push_back(l3_eot);
                break;
            case FENCE_CHAT_LLAMA2:
            case FENCE_CHAT_MISTRAL:
                if (m_eos > 0) t.push_back(m_eos);
                break;
            default: break;
        }
    }
    static constexpr int kImStart = 151644, kImEnd = 151645;  // <|im_start|>, <|im_end|> (tokenizer.h:84-85)
};

namespace {

int meta_int(const GGUFFile& g, const char* key, int dflt) {
    const GGUFMetadataKV* kv = g.find_metadata(key);
    if (!kv) return dflt;
    if (kv->type == GGUFValueType::UINT32) return (int)std::get<uint32_t>(kv->value);
    if (kv->type == GGUFValueType::INT32) return std::get<int32_t>(kv->value);
    return dflt;  // other types are skipped, as the reference's reader does
}
std::string meta_str(const GGUFFile& g, const char* key) {
    const GGUFMetadataKV* kv = g.find_metadata(key);
    return (kv && kv->type == GGUFValueType::STRING) ? std::get<std::string>(kv->value) : std::string();
}

// Copies ids to out (capacity cap): FENCE_OK, or FENCE_E_ARG when they do not fit (*n_out = the
// count needed either way).
int emit(const std::vector<int>& ids, size_t from, int* out, int cap, int* n_out) {
    if (n_out) *n_out = (int)ids.size();
    if ((long long)ids.size() > (long long)cap)
        return set_error(FENCE_E_ARG, "tokenizer: %zu ids do not fit the buffer of %d", ids.size(), cap);
    if (ids.size() > from) std::memcpy(out + from, ids.data() + from, (ids.size() - from) * sizeof(int));
    return FENCE_OK;
}

}  // namespace

extern "C" fence_tokenizer* fence_tokenizer_load(const char* gguf_path) {
    if (!gguf_path) {
        set_error(FENCE_E_ARG, "tokenizer_load: null path");
        return nullptr;
    }
    GGUFFile g;
    if (!g.open(gguf_path)) {
        set_error(FENCE_E_FORMAT, "tokenizer_load: %s", g.last_error().c_str());
        return nullptr;
    }
    const std::vector<std::string>* toks = g.get_string_array("tokenizer.ggml.tokens");
    if (!toks || toks->empty()) {
        set_error(FENCE_E_FORMAT, "tokenizer_load: no tokenizer.ggml.tokens in %s", gguf_path);
        return nullptr;
    }
    fence_tokenizer* t = new fence_tokenizer();
    t->id_to_token = *toks;
    for (int i = 0; i < (int)toks->size(); ++i) t->token_to_id[(*toks)[i]] = i;  // a repeated string keeps its last id
    if (const std::vector<std::string>* mg = g.get_string_array("tokenizer.ggml.merges"))
        for (int r = 0; r < (int)mg->size(); ++r) t->merges[(*mg)[r]] = r;
    t->bos = meta_int(g, "tokenizer.ggml.bos_token_id", t->bos);
    t->eos = meta_int(g, "tokenizer.ggml.eos_token_id", t->eos);
    t->format = fence_tokenizer::detect(meta_str(g, "general.architecture"), meta_str(g, "tokenizer.chat_template"));
    auto id = [&](const char* s) { const int v = t->lookup(s); return v >= 0 ? v : 0; };
    t->l3_begin = id("<|begin_of_text|>");
    t->l3_start_hdr = id("<|start_header_id|>");
    t->l3_end_hdr = id("<|end_header_id|>");
    t->l3_eot = id("<|eot_id|>");
    t->m_bos = id("<s>");
    t->m_eos = id("</s>");
    t->inst_start = id("[INST]");
    t->inst_end = id("[/INST]");
    if (t->format == FENCE_CHAT_LLAMA3 && t->l3_begin > 0) t->bos = t->l3_begin;
    if (t->format == FENCE_CHAT_LLAMA3 && t->l3_eot > 0) t->eos = t->l3_eot;
    if ((t->format == FENCE_CHAT_MISTRAL || t->format == FENCE_CHAT_LLAMA2) && t->m_eos > 0) t->eos = t->m_eos;
    return t;
}

extern "C" void fence_tokenizer_free(fence_tokenizer* t) { delete t; }

extern "C" int fence_tokenizer_info(const fence_tokenizer* t, int* chat_format, int* bos_id, int* eos_id,
                                    int* vocab_size) {
    if (!t) return set_error(FENCE_E_ARG, "tokenizer_info: null tokenizer");
    if (chat_format) *chat_format = t->format;
    if (bos_id) *bos_id = t->bos;
    if (eos_id) *eos_id = t->eos;
    if (vocab_size) *vocab_size = (int)t->id_to_token.size();
    return FENCE_OK;
}

extern "C" int fence_tokenize(const fence_tokenizer* t, const char* text, size_t len, int* out, int cap, int* n_out) {
    if (!t || (!text && len) || (!out && cap > 0) || cap < 0) return set_error(FENCE_E_ARG, "tokenize: bad arguments");
    return emit(t->encode(std::string(text ? text : "", len)), 0, out, cap, n_out);
}

extern "C" int fence_detokenize(const fence_tokenizer* t, const int* ids, int n, char* out, size_t cap,
                                size_t* len_out) {
    if (!t || n < 0 || (!ids && n) || (!out && cap)) return set_error(FENCE_E_ARG, "detokenize: bad arguments");
    std::string s;
    for (int i = 0; i < n; ++i) s += t->decode(ids[i]);
    if (len_out) *len_out = s.size();
    if (s.size() + 1 > cap) return set_error(FENCE_E_ARG, "detokenize: %zu bytes do not fit the buffer of %zu", s.size() + 1, cap);
    std::memcpy(out, s.data(), s.size());
    out[s.size()] = '\0';
    return FENCE_OK;
}

extern "C" int fence_format_chat(fence_tokenizer* t, const char* system_prompt, const char* user_message, int* out,
                                 int cap, int* n_out) {
    if (!t || !user_message || (!out && cap > 0) || cap < 0) return set_error(FENCE_E_ARG, "format_chat: bad arguments");
    std::vector<int> ids;
    t->begin(ids);
    if (system_prompt && *system_prompt) t->system_turn(ids, system_prompt);
    t->user_turn(ids, user_message);
    t->assistant_header(ids);
    return emit(ids, 0, out, cap, n_out);
}

extern "C" int fence_chat_append(fence_tokenizer* t, int turn, const char* content, int* tokens, int cap,
                                 int* n_inout) {
    if (!t || !n_inout || *n_inout < 0 || *n_inout > cap || (!tokens && cap > 0))
        return set_error(FENCE_E_ARG, "chat_append: bad arguments");
    if ((turn == FENCE_TURN_SYSTEM || turn == FENCE_TURN_USER) && !content)
        return set_error(FENCE_E_ARG, "chat_append: null content");
    const size_t n0 = (size_t)*n_inout;
    std::vector<int> ids(tokens, tokens + n0);
    // the conversation state a turn may change (a LLaMA-2 / Mistral system prompt held for the first
    // user turn), restored when the ids do not fit, so the caller can retry with a larger buffer
    const std::string held = t->pending_system;
    const bool held_used = t->system_used;
    switch (turn) {
        case FENCE_TURN_BEGIN: t->begin(ids); break;
        case FENCE_TURN_SYSTEM: t->system_turn(ids, content); break;
        case FENCE_TURN_USER: t->user_turn(ids, content); break;
        case FENCE_TURN_ASSISTANT: t->assistant_header(ids); break;
        case FENCE_TURN_END: t->turn_end(ids); break;
        default: return set_error(FENCE_E_ARG, "chat_append: unknown turn %d", turn);
    }
    const int rc = emit(ids, n0, tokens, cap, n_inout);
    if (rc != FENCE_OK) {
        t->pending_system = held;
        t->system_used = held_used;
    }
    return rc;
}
