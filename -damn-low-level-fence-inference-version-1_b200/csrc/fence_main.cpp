// fence_main.cpp — the `fence` command line with the reference's flags, defaults and flow
// (src/main.cu:17-162): --model --prompt --system --max-tokens --max-ctx --temp --top-p --top-k
// --rep-penalty --debug --help. The tokenizer and chat format come from the GGUF
// (fence_tokenizer_*, the reference's Tokenizer); --prompt formats one turn with the system
// prompt (format_chat) and streams the reply, no --prompt runs the interactive chat loop (history
// kept across turns, cleared when fewer than 256 positions of max_ctx remain). Sampling flags are
// applied to the model after load, as there. Harness flags on top:
//   --tokens 1,2,3   prompt given as token ids (skips text encoding and the chat format)
//   --seed N         sampler seed (the reference seeds from random_device)
//   --kv f16|bf16    KV-cache element type (default f16, the reference cache type)
//   --no-graph       launch kernels one by one instead of replaying the captured step
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <string>
#include <vector>

#include "../../include/fence_b200.h"

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

std::string detok(const fence_tokenizer* t, int id) {
    char buf[1024];
    size_t n = 0;
    if (fence_detokenize(t, &id, 1, buf, sizeof buf, &n) == 0) return std::string(buf, n);
    std::string big(n + 1, '\0');
    fence_detokenize(t, &id, 1, &big[0], big.size(), &n);
    big.resize(n);
    return big;
}

// Qwen3Model::generate (qwen3.cu:463-519): prefill of the whole history (fence_prefill: batched on
// the tensor cores where the model allows it, as fence_generate does; the reference runs it token
// by token), then sample (nucleus, the CLI's parameters), stop at eos or max_ctx, stream each new
// token's text. Returns the history plus the reply (without eos), or an empty vector on an engine
// error.
std::vector<int> generate(fence_model* m, const fence_tokenizer* tok, const std::vector<int>& prompt, int max_new,
                          int eos, int max_ctx, bool debug) {
    std::vector<int> out(prompt);
    const auto t0 = std::chrono::steady_clock::now();
    const float* logits = fence_prefill(m, prompt.data(), (int)prompt.size(), 0);
    if (!logits) return {};
    const auto t1 = std::chrono::steady_clock::now();
    const double pre_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    printf("[prefill %zu tokens in %.0f ms (%.1f tok/s)]\n", prompt.size(), pre_ms, prompt.size() / (pre_ms / 1e3));
    int pos = (int)prompt.size(), gen = 0;
    for (int i = 0; i < max_new && pos < max_ctx; ++i) {
        const int next = fence_sample_nucleus(m, logits, out.data(), (int)out.size());
        if (next < 0) return {};
        if (next == eos) break;
        out.push_back(next);
        ++gen;
        if (tok) printf("%s", detok(tok, next).c_str());
        else printf("%d ", next);
        fflush(stdout);
        if (debug) fprintf(stderr, "[step %d: id %d]\n", pos, next);
        if (!(logits = fence_forward(m, next, pos))) return {};
        ++pos;
    }
    const double dec_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t1).count();
    if (gen > 0) printf("\n[generated %d tokens in %.0f ms (%.1f tok/s)]\n", gen, dec_ms, gen / (dec_ms / 1e3));
    return out;
}

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

    fence_tokenizer* tok = nullptr;
    if (tokens_arg.empty()) {
        tok = fence_tokenizer_load(model_path.c_str());
        if (!tok) {
            fprintf(stderr, "Error: %s (pass --tokens to skip text)\n", fence_last_error());
            return 1;
        }
        int fmt = 0, bos = 0, eos = 0, nv = 0;
        fence_tokenizer_info(tok, &fmt, &bos, &eos, &nv);
        static const char* names[] = {"ChatML", "LLaMA-3", "LLaMA-2", "Mistral", "Raw"};
        printf("Tokenizer: %d tokens, format=%s  bos=%d  eos=%d\n", nv, names[fmt], bos, eos);
        printf("Chat format : %s\n\n", names[fmt]);
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
        fence_tokenizer_free(tok);
        return 1;
    }
    fence_set_sampling(m, temp, top_p, top_k, rep);
    if (have_seed) fence_set_seed(m, seed);
    int eos = -1;
    if (tok) fence_tokenizer_info(tok, nullptr, nullptr, &eos, nullptr);
    auto fail = [&]() {
        fprintf(stderr, "\nError: %s\n", fence_last_error());
        fence_model_free(m);
        fence_tokenizer_free(tok);
        return 1;
    };
    auto ids_of = [&](auto fn) {  // a tokenizer call into a growing buffer
        std::vector<int> v(256);
        int n = 0;
        while (fn(v, n) != 0) {
            if (n <= (int)v.size()) return std::vector<int>();
            v.resize(n);
        }
        v.resize(n);
        return v;
    };

    if (!tokens_arg.empty() || !prompt.empty()) {  // ---- single-prompt mode
        std::vector<int> ids;
        if (!tokens_arg.empty()) {
            for (const char* p = tokens_arg.c_str(); *p;) {
                ids.push_back((int)strtol(p, const_cast<char**>(&p), 10));
                while (*p == ',' || *p == ' ') ++p;
            }
        } else {
            ids = ids_of([&](std::vector<int>& v, int& n) {
                return fence_format_chat(tok, system_prompt.c_str(), prompt.c_str(), v.data(), (int)v.size(), &n);
            });
        }
        if (ids.empty()) {
            fprintf(stderr, "Error: empty prompt\n");
            fence_model_free(m);
            fence_tokenizer_free(tok);
            return 1;
        }
        printf("Prompt tokens: %zu\n", ids.size());
        printf("Assistant: ");
        fflush(stdout);
        const std::vector<int> out = generate(m, tok, ids, max_tokens, eos, max_ctx, debug);
        if (out.empty()) return fail();
        printf("\n");
        if (debug) {
            printf("ids:");
            for (int id : out) printf(" %d", id);
            printf("\n");
        }
        fence_model_free(m);
        fence_tokenizer_free(tok);
        return 0;
    }

    // ---- interactive chat loop (main.cu:116-157)
    printf("System: %s\n", system_prompt.c_str());
    printf("Type your message (empty line to quit).\n\n");
    std::vector<int> history;
    auto append = [&](int turn, const char* content) {
        const int n0 = (int)history.size();
        history.resize(history.size() + 4096 + (content ? 4 * strlen(content) : 0));
        int n = n0;
        int rc = fence_chat_append(tok, turn, content, history.data(), (int)history.size(), &n);
        if (rc != 0 && n > (int)history.size()) {  // too small (a long held system prompt): retry at the size needed
            history.resize(n);
            n = n0;
            rc = fence_chat_append(tok, turn, content, history.data(), (int)history.size(), &n);
        }
        history.resize(rc == 0 ? n : n0);
        return rc == 0;
    };
    auto start = [&]() {
        history.clear();
        append(FENCE_TURN_BEGIN, nullptr);
        if (!system_prompt.empty()) append(FENCE_TURN_SYSTEM, system_prompt.c_str());
    };
    start();
    while (true) {
        printf("You: ");
        fflush(stdout);
        std::string line;
        if (!std::getline(std::cin, line) || line.empty()) break;
        if ((int)history.size() > max_ctx - 256) {
            fprintf(stderr, "\n[Context limit approaching — clearing history]\n");
            start();
        }
        append(FENCE_TURN_USER, line.c_str());
        append(FENCE_TURN_ASSISTANT, nullptr);
        printf("  [%zu tokens in context]\n", history.size());
        printf("Assistant: ");
        fflush(stdout);
        std::vector<int> out = generate(m, tok, history, max_tokens, eos, max_ctx, debug);
        if (out.empty()) return fail();
        printf("\n\n");
        history = std::move(out);
        append(FENCE_TURN_END, nullptr);
    }
    fence_model_free(m);
    fence_tokenizer_free(tok);
    printf("Goodbye!\n");
    return 0;
}
