// ref_model_harness.cu — drives the reference's unmodified CUDA forward (Qwen3Model, compiled from
// the reference tree for sm_100a) over a prompt of token ids and records, for every decode step,
// the fp32 logits and the greedy id. Used to produce golden fixtures and the "reference on B200"
// timing. Test infrastructure only; needs a GPU.
//
//   ref_model MODEL OUT --tokens 1,2,3 --steps N [--teacher 4,5,6] [--max-ctx N] [--no-logits]
//
// OUT layout: int32 magic 0x46524546 ("FERF"), int32 vocab, int32 n_prompt, int32 n_steps, then
// per step: int32 greedy id, float32 logits[vocab] (omitted with --no-logits).
// The loop calls forward + sample_greedy directly, not generate(), because generate() stops at
// id 151645 (the default eos), a legal id in a random model (qwen3.cu:472,496).
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "src/model/qwen3.h"

static std::vector<int> parse_ids(const char* s) {
    std::vector<int> v;
    while (*s) {
        char* e;
        v.push_back((int)strtol(s, &e, 10));
        s = e;
        while (*s == ',' || *s == ' ') ++s;
    }
    return v;
}

int main(int argc, char** argv) {
    if (argc < 3) {
        fprintf(stderr, "usage: %s MODEL OUT --tokens LIST --steps N [--teacher LIST] [--max-ctx N] [--no-logits]\n", argv[0]);
        return 2;
    }
    std::vector<int> prompt, teacher;
    int steps = 0, max_ctx = 4096;
    bool logits_out = true;
    for (int i = 3; i < argc; ++i) {
        if (!strcmp(argv[i], "--tokens") && i + 1 < argc) prompt = parse_ids(argv[++i]);
        else if (!strcmp(argv[i], "--steps") && i + 1 < argc) steps = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--teacher") && i + 1 < argc) teacher = parse_ids(argv[++i]);
        else if (!strcmp(argv[i], "--max-ctx") && i + 1 < argc) max_ctx = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--no-logits")) logits_out = false;
    }
    if (prompt.empty()) return 2;
    Qwen3Model model;
    model.config.max_ctx = max_ctx;
    if (!model.load(argv[1])) return 3;
    const int V = model.config.vocab_size;
    FILE* f = fopen(argv[2], "wb");
    if (!f) return 4;
    const int hdr[4] = {0x46524546, V, (int)prompt.size(), steps};
    fwrite(hdr, 4, 4, f);
    float* logits = nullptr;
    const auto t0 = std::chrono::steady_clock::now();
    for (size_t i = 0; i < prompt.size(); ++i) logits = model.forward(prompt[i], (int)i);
    const auto t1 = std::chrono::steady_clock::now();
    std::vector<float> h(V);
    int pos = (int)prompt.size();
    double decode_s = 0.0;
    for (int s = 0; s < steps; ++s) {
        if (logits_out) cudaMemcpy(h.data(), logits, (size_t)V * 4, cudaMemcpyDeviceToHost);
        const auto a = std::chrono::steady_clock::now();
        const int next = model.sample_greedy(logits);
        fwrite(&next, 4, 1, f);
        if (logits_out) fwrite(h.data(), 4, (size_t)V, f);
        const int feed = (s < (int)teacher.size()) ? teacher[s] : next;
        if (s + 1 < steps) logits = model.forward(feed, pos++);
        decode_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - a).count();
    }
    fclose(f);
    const double prefill_s = std::chrono::duration<double>(t1 - t0).count();
    printf("{\"ref_prefill_tok_s\": %.3f, \"ref_decode_tok_s\": %.3f, \"prompt\": %zu, \"steps\": %d}\n",
           prompt.size() / prefill_s, steps > 1 ? (steps - 1) / decode_s : 0.0, prompt.size(), steps);
    model.unload();
    return 0;
}
