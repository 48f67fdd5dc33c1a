// fence_main.cpp — the `fence` command line with the reference's flags and defaults
// (src/main.cu:17-162): --model --prompt --system --max-tokens --max-ctx --temp --top-p --top-k
// --rep-penalty --debug --help. Sampling flags are applied to the model after load, as there.
//
// Text handling is minimal: the prompt is encoded by greedy longest match over the GGUF's
// tokenizer.ggml.tokens after GPT-2 byte-to-unicode mapping, and generated ids are decoded the same
// way; the reference's BPE merges and chat templates are not rebuilt. Harness flags on top:
//   --tokens 1,2,3   prompt given as token ids (skips text encoding)
//   --seed N         sampler seed (the reference seeds from random_device)
//   --kv f16|bf16    KV-cache element type (default f16, the reference cache type)
//   --no-graph       launch kernels one by one instead of replaying the captured step
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/fence_b200.h"
#include "gguf.h"

namespace {

void print_usage(const char* prog) {
    printf("Usage: %s --model PATH [options]\n\n", prog);
    printf("Required:\n  --model PATH       GGUF model file\n\n");
    printf("Options:\n");
    printf("  --prompt TEXT      Single prompt (non-interactive mode)\n");
    printf("  --system TEXT      System prompt (default: 'You are a helpful assistant.')\n");
    printf("  --max-tokens N     Max new tokens to generate (default: 512)\n");
    printf("  --max-ctx N        Max context length in tokens (default: 4096)\n");
    printf("  --temp F           Sampling temperature (default: 0.7)\n");
    printf("  --top-p F          Top-p nucleus cutoff (default: 0.8)\n");
    printf("  --top-k N          Top-k candidates (default: 50)\n");
    printf("  --rep-penalty F    Repetition penalty (default: 1.15)\n");
    printf("  --debug            Print per-step statistics\n");
    printf("  --help             Show this help\n\n");
    printf("Harness options:\n");
    printf("  --tokens LIST      Comma-separated prompt token ids\n");
    printf("  --seed N           Sampler seed\n");
    printf("  --kv f16|bf16      KV cache type (default f16, the reference cache type)\n");
    printf("  --no-graph         Do not replay a captured CUDA graph\n");
}

// GPT-2 byte <-> unicode code point table (printable bytes map to themselves, the rest to 256+n).
std::vector<int> byte_to_cp() {
    std::vector<int> t(256, -1);
    int n = 0;
    for (int b = 0; b < 256; ++b) {
        const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
        t[b] = keep ? b : 256 + n++;
    }
    return t;
}
void put_utf8(std::string& s, int cp) {
    if (cp < 0x80) s += (char)cp;
    else if (cp < 0x800) {
        s += (char)(0xC0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3F));
    } else {
        s += (char)(0xE0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    }
}

struct Vocab {
    std::vector<std::string> tokens;
    std::unordered_map<std::string, int> index;
    std::unordered_map<int, int> cp_to_byte;
    int eos = 151645;  // reference default (tokenizer.h, Qwen <|im_end|>)
    bool ok = false;

    void load(const fence::GGUFFile& g) {
        const auto* t = g.get_string_array("tokenizer.ggml.tokens");
        if (!t) return;
        tokens = *t;
        for (int i = 0; i < (int)tokens.size(); ++i) index.emplace(tokens[i], i);
        const auto b2c = byte_to_cp();
        for (int b = 0; b < 256; ++b) cp_to_byte[b2c[b]] = b;
        if (const auto* kv = g.find_metadata("tokenizer.ggml.eos_token_id")) {
            if (kv->type == fence::GGUFValueType::UINT32) eos = (int)std::get<uint32_t>(kv->value);
            if (kv->type == fence::GGUFValueType::INT32) eos = std::get<int32_t>(kv->value);
        }
        ok = true;
    }
    std::vector<int> encode(const std::string& text) const {
        const auto b2c = byte_to_cp();
        std::string u;
        for (unsigned char ch : text) put_utf8(u, b2c[ch]);
        std::vector<int> ids;
        size_t pos = 0;
        while (pos < u.size()) {
            int best = -1;
            size_t blen = 0;
            for (size_t len = std::min<size_t>(128, u.size() - pos); len > 0; --len) {
                auto it = index.find(u.substr(pos, len));
                if (it != index.end()) {
                    best = it->second;
                    blen = len;
                    break;
                }
            }
            if (best < 0) {
                ++pos;  // unknown byte: skip
                continue;
            }
            ids.push_back(best);
            pos += blen;
        }
        return ids;
    }
    std::string decode(int id) const {
        if (id < 0 || id >= (int)tokens.size()) return "";
        const std::string& s = tokens[id];
        std::string out;
        for (size_t i = 0; i < s.size();) {
            const unsigned char c = s[i];
            int cp, n;
            if (c < 0x80) { cp = c; n = 1; }
            else if ((c >> 5) == 6) { cp = c & 0x1F; n = 2; }
            else if ((c >> 4) == 14) { cp = c & 0x0F; n = 3; }
            else { cp = c & 0x07; n = 4; }
            for (int k = 1; k < n && i + k < s.size(); ++k) cp = (cp << 6) | (s[i + k] & 0x3F);
            auto it = cp_to_byte.find(cp);
            if (it != cp_to_byte.end()) out += (char)it->second;
            else out += s.substr(i, n);
            i += n;
        }
        return out;
    }
};

}  // namespace

int main(int argc, char** argv) {
    printf("Fence Inference Engine (B200 / sm_100a)\n\n");
    std::string model_path, prompt, system_prompt = "You are a helpful assistant.", tokens_arg, kv = "f16";
    int max_tokens = 512, max_ctx = 4096, top_k = 50;
    float temp = 0.7f, top_p = 0.8f, rep = 1.15f;
    bool debug = false, graph = true;
    unsigned long long seed = 0;
    bool have_seed = false;
    for (int i = 1; i < argc; ++i) {
        auto next = [&]() -> const char* { return (i + 1 < argc) ? argv[++i] : nullptr; };
        const char* a = argv[i];
        const char* v = nullptr;
        if (!strcmp(a, "--model") && (v = next())) model_path = v;
        else if (!strcmp(a, "--prompt") && (v = next())) prompt = v;
        else if (!strcmp(a, "--system") && (v = next())) system_prompt = v;
        else if (!strcmp(a, "--max-tokens") && (v = next())) max_tokens = atoi(v);
        else if (!strcmp(a, "--max-ctx") && (v = next())) max_ctx = atoi(v);
        else if (!strcmp(a, "--temp") && (v = next())) temp = (float)atof(v);
        else if (!strcmp(a, "--top-p") && (v = next())) top_p = (float)atof(v);
        else if (!strcmp(a, "--top-k") && (v = next())) top_k = atoi(v);
        else if (!strcmp(a, "--rep-penalty") && (v = next())) rep = (float)atof(v);
        else if (!strcmp(a, "--tokens") && (v = next())) tokens_arg = v;
        else if (!strcmp(a, "--seed") && (v = next())) { seed = strtoull(v, nullptr, 10); have_seed = true; }
        else if (!strcmp(a, "--kv") && (v = next())) kv = v;
        else if (!strcmp(a, "--no-graph")) graph = false;
        else if (!strcmp(a, "--debug")) debug = true;
        else if (!strcmp(a, "--help")) { print_usage(argv[0]); return 0; }
        else {
            fprintf(stderr, "Unknown option: %s\n", a);
            print_usage(argv[0]);
            return 1;
        }
    }
    if (model_path.empty()) {
        fprintf(stderr, "Error: --model PATH is required.\n\n");
        print_usage(argv[0]);
        return 1;
    }

    fence::GGUFFile g;
    if (!g.open(model_path)) return 1;
    Vocab vocab;
    vocab.load(g);
    g.close();

    std::vector<int> ids;
    if (!tokens_arg.empty()) {
        for (const char* p = tokens_arg.c_str(); *p;) {
            ids.push_back((int)strtol(p, const_cast<char**>(&p), 10));
            while (*p == ',' || *p == ' ') ++p;
        }
    } else if (!prompt.empty()) {
        if (!vocab.ok) {
            fprintf(stderr, "Error: the model has no tokenizer.ggml.tokens; pass --tokens\n");
            return 1;
        }
        ids = vocab.encode(prompt);
    } else {
        fprintf(stderr, "Error: interactive chat is not built; pass --prompt TEXT or --tokens LIST\n");
        return 1;
    }
    if (ids.empty()) {
        fprintf(stderr, "Error: empty prompt\n");
        return 1;
    }

    fence_load_opts o;
    fence_load_opts_default(&o);
    o.max_ctx = max_ctx;
    o.kv_dtype = (kv == "bf16") ? FENCE_KV_BF16 : FENCE_KV_F16;
    o.use_graph = graph ? 1 : 0;
    o.verbose = 1;
    fence_model* m = fence_model_load(model_path.c_str(), &o);
    if (!m) {
        fprintf(stderr, "Error: %s\n", fence_last_error());
        return 1;
    }
    fence_set_sampling(m, temp, top_p, top_k, rep);
    if (have_seed) fence_set_seed(m, seed);

    printf("Prompt tokens: %zu\n", ids.size());
    std::vector<int> out(ids.size() + (size_t)max_tokens + 1);
    int n_out = 0;
    const auto t0 = std::chrono::steady_clock::now();
    const int rc = fence_generate(m, ids.data(), (int)ids.size(), max_tokens, vocab.ok ? vocab.eos : -1, out.data(),
                                  (int)out.size(), &n_out);
    const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (rc) {
        fprintf(stderr, "Error: %s\n", fence_last_error());
        fence_model_free(m);
        return 1;
    }
    printf("Assistant: ");
    for (int i = (int)ids.size(); i < n_out; ++i) {
        if (vocab.ok) printf("%s", vocab.decode(out[i]).c_str());
        else printf("%d ", out[i]);
    }
    printf("\n");
    const int gen = n_out - (int)ids.size();
    printf("\n[%zu prompt + %d generated tokens in %.0f ms]\n", ids.size(), gen, sec * 1e3);
    if (debug) {
        printf("ids:");
        for (int i = 0; i < n_out; ++i) printf(" %d", out[i]);
        printf("\n");
    }
    (void)system_prompt;
    fence_model_free(m);
    return 0;
}
