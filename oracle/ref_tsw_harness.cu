// ref_tsw_harness.cu — ORACLE EXTENSION (test infrastructure only; needs a GPU).
//
// The reference's forward cannot load a model whose linears are Q8_0: Qwen3Model::load casts every
// linear to block_q6_K and forward calls gemv_q6k on it (src/model/qwen3.cu:191-211,280-337). For
// the all-Q8_0 Llama-shaped model this harness restates Qwen3Model::load and
// Qwen3Model::forward / forward_attention / forward_mlp (src/model/qwen3.cu:116-228,241-341) op for
// op, with one change: a "type switch" per linear. A Q8_0 linear runs the reference's own gemv_q8_0
// (src/kernels/gemv_q8_0.cuh:99-104) on the fp32 activation, as the reference does for its Q8_0 LM
// head (qwen3.cu:261); a Q6_K linear keeps the reference's f32_to_f16 + gemv_q6k(_bias). Every op is
// the reference's own kernel from its headers (ops.cuh, gemv_q6k.cuh, gemv_q8_0.cuh), launched on
// the legacy stream in the reference's order; KV cache fp16 [max_ctx][kv_dim] per layer; tied LM head.
//
// Same command line and output file as ref_model_harness.cu:
//   ref_model_tsw MODEL OUT --tokens 1,2,3 --steps N [--teacher 4,5,6] [--max-ctx N] [--no-logits]
// This file includes the reference's kernel headers, so it is a separate program from ref_model
// (which links qwen3.cu, where the same kernels are defined).
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "src/gguf/gguf_parser.h"
#include "src/kernels/gemv_q6k.cuh"
#include "src/kernels/gemv_q8_0.cuh"
#include "src/kernels/ops.cuh"

#define CK(call)                                                                               \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess) {                                                               \
            fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            exit(5);                                                                           \
        }                                                                                      \
    } while (0)

struct Lin {
    const void* w = nullptr;
    GGMLType type = GGMLType::Q6_K;
    const float* bias = nullptr;
};

struct Layer {
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    Lin q, k, v, o, gate, up, down;
};

struct Model {
    GGUFFile gguf;
    int n_layers = 0, embed_dim = 0, ff_dim = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, vocab = 0,
        max_ctx = 4096;
    float rope_base = 10000.f, rms_eps = 1e-5f;
    const block_q8_0* embd = nullptr;
    const float* out_norm = nullptr;
    std::vector<Layer> layers;
    std::vector<__half*> kc, vc;
    float *hidden, *residual, *normed, *q, *k, *v, *attn_out, *gate, *up, *logits, *score_buf;
    __half* x_half;
    int* argmax_out;
    std::vector<void*> allocs;

    int q_dim() const { return n_heads * head_dim; }
    int kv_dim() const { return n_kv_heads * head_dim; }

    const void* upload(const GGUFTensorInfo* t) {
        if (!t) return nullptr;
        void* d = nullptr;
        CK(cudaMalloc(&d, t->data_size_bytes));
        CK(cudaMemcpy(d, t->data, t->data_size_bytes, cudaMemcpyHostToDevice));
        allocs.push_back(d);
        return d;
    }
    float* dev(size_t n) {
        void* d = nullptr;
        CK(cudaMalloc(&d, n * sizeof(float)));
        allocs.push_back(d);
        return static_cast<float*>(d);
    }

    // qwen3.cu:116-228 (config keys, fallbacks, tensor names), weights kept with their type
    bool load(const char* path) {
        if (!gguf.open(path)) return false;
        std::string arch = "qwen2";
        try {
            arch = gguf.get_string("general.architecture");
        } catch (...) {
        }
        n_layers = gguf.get_u32(arch + ".block_count");
        embed_dim = gguf.get_u32(arch + ".embedding_length");
        ff_dim = gguf.get_u32(arch + ".feed_forward_length");
        n_heads = gguf.get_u32(arch + ".attention.head_count");
        n_kv_heads = gguf.get_u32(arch + ".attention.head_count_kv");
        try {
            head_dim = gguf.get_u32(arch + ".attention.key_length");
        } catch (...) {
            head_dim = embed_dim / n_heads;
        }
        try {
            rope_base = gguf.get_f32(arch + ".rope.freq_base");
        } catch (...) {
            rope_base = 10000.0f;
        }
        try {
            rms_eps = gguf.get_f32(arch + ".attention.layer_norm_rms_epsilon");
        } catch (...) {
            rms_eps = 1e-5f;
        }
        const GGUFTensorInfo* et = gguf.find_tensor("token_embd.weight");
        if (!et) return false;
        vocab = (int)et->dims[1];
        embd = static_cast<const block_q8_0*>(upload(et));
        out_norm = static_cast<const float*>(upload(gguf.find_tensor("output_norm.weight")));
        layers.resize(n_layers);
        for (int l = 0; l < n_layers; ++l) {
            Layer& L = layers[l];
            const std::string p = "blk." + std::to_string(l) + ".";
            auto vecf = [&](const char* n) { return static_cast<const float*>(upload(gguf.find_tensor(p + n))); };
            auto lin = [&](const char* n, const char* bias) {
                Lin r;
                const GGUFTensorInfo* t = gguf.find_tensor(p + n);
                if (!t) {
                    fprintf(stderr, "missing %s%s\n", p.c_str(), n);
                    exit(3);
                }
                r.type = t->type;
                if (r.type != GGMLType::Q6_K && r.type != GGMLType::Q8_0) {
                    fprintf(stderr, "%s%s: type %d not Q6_K / Q8_0\n", p.c_str(), n, (int)r.type);
                    exit(3);
                }
                r.w = upload(t);
                if (bias) r.bias = vecf(bias);
                return r;
            };
            L.attn_norm = vecf("attn_norm.weight");
            L.q = lin("attn_q.weight", "attn_q.bias");
            L.k = lin("attn_k.weight", "attn_k.bias");
            L.v = lin("attn_v.weight", "attn_v.bias");
            L.q_norm = vecf("attn_q_norm.weight");
            L.k_norm = vecf("attn_k_norm.weight");
            L.o = lin("attn_output.weight", nullptr);
            L.ffn_norm = vecf("ffn_norm.weight");
            L.gate = lin("ffn_gate.weight", nullptr);
            L.up = lin("ffn_up.weight", nullptr);
            L.down = lin("ffn_down.weight", nullptr);
        }
        kc.resize(n_layers);
        vc.resize(n_layers);
        for (int l = 0; l < n_layers; ++l) {  // KVCache::allocate (qwen3.cu:47-56)
            const size_t n = (size_t)max_ctx * kv_dim();
            CK(cudaMalloc(&kc[l], n * sizeof(__half)));
            CK(cudaMalloc(&vc[l], n * sizeof(__half)));
            CK(cudaMemset(kc[l], 0, n * sizeof(__half)));
            CK(cudaMemset(vc[l], 0, n * sizeof(__half)));
            allocs.push_back(kc[l]);
            allocs.push_back(vc[l]);
        }
        hidden = dev(embed_dim);
        residual = dev(embed_dim);
        normed = dev(embed_dim);
        q = dev(q_dim());
        k = dev(kv_dim());
        v = dev(kv_dim());
        attn_out = dev(q_dim());
        gate = dev(ff_dim);
        up = dev(ff_dim);
        logits = dev(vocab);
        score_buf = dev((size_t)n_heads * max_ctx);
        x_half = reinterpret_cast<__half*>(dev((std::max(ff_dim, embed_dim) + 1) / 2));
        argmax_out = reinterpret_cast<int*>(dev(1));
        return true;
    }

    // One linear on an fp32 activation x[K] -> y[M]. Q8_0: gemv_q8_0 on fp32 x (gemv_q8_0.cuh:99);
    // Q6_K: f32_to_f16 then gemv_q6k / gemv_q6k_bias (the reference's path, qwen3.cu:278-289).
    void linear(const Lin& L, const float* x, float* y, int M, int K) {
        if (L.type == GGMLType::Q8_0) {
            gemv_q8_0(static_cast<const block_q8_0*>(L.w), x, y, M, K);
            if (L.bias) residual_add(y, L.bias, M);
        } else {
            f32_to_f16(x_half, x, K);
            if (L.bias) gemv_q6k_bias(static_cast<const block_q6_K*>(L.w), x_half, L.bias, y, M, K);
            else gemv_q6k(static_cast<const block_q6_K*>(L.w), x_half, y, M, K);
        }
    }

    // qwen3.cu:241-341 with the type switch above
    float* forward(int token, int pos) {
        embed_q8_0(hidden, embd, token, embed_dim);
        CK(cudaDeviceSynchronize());
        for (int l = 0; l < n_layers; ++l) {
            const Layer& L = layers[l];
            // attention block
            CK(cudaMemcpyAsync(residual, hidden, embed_dim * sizeof(float), cudaMemcpyDeviceToDevice));
            rms_norm(normed, hidden, L.attn_norm, embed_dim, rms_eps);
            linear(L.q, normed, q, q_dim(), embed_dim);
            linear(L.k, normed, k, kv_dim(), embed_dim);
            linear(L.v, normed, v, kv_dim(), embed_dim);
            if (L.q_norm && L.k_norm) {
                rms_norm_per_head(q, L.q_norm, n_heads, head_dim, rms_eps);
                rms_norm_per_head(k, L.k_norm, n_kv_heads, head_dim, rms_eps);
            }
            apply_rope(q, k, head_dim, n_heads, n_kv_heads, pos, rope_base);
            store_kv(kc[l], vc[l], k, v, pos, kv_dim(), max_ctx);
            gqa_attention(attn_out, q, kc[l], vc[l], head_dim, n_heads, n_kv_heads, pos + 1, max_ctx, score_buf);
            linear(L.o, attn_out, hidden, embed_dim, q_dim());
            residual_add(hidden, residual, embed_dim);
            // MLP block
            CK(cudaMemcpyAsync(residual, hidden, embed_dim * sizeof(float), cudaMemcpyDeviceToDevice));
            rms_norm(normed, hidden, L.ffn_norm, embed_dim, rms_eps);
            linear(L.gate, normed, gate, ff_dim, embed_dim);
            linear(L.up, normed, up, ff_dim, embed_dim);
            silu_elementwise_mul(gate, gate, up, ff_dim);
            linear(L.down, gate, hidden, embed_dim, ff_dim);
            residual_add(hidden, residual, embed_dim);
        }
        rms_norm_inplace(hidden, out_norm, embed_dim, rms_eps);
        gemv_q8_0(embd, hidden, logits, vocab, embed_dim);
        CK(cudaDeviceSynchronize());
        return logits;
    }

    int sample_greedy(const float* lg) {  // qwen3.cu:344-349
        argmax(lg, argmax_out, vocab);
        int r = 0;
        CK(cudaMemcpy(&r, argmax_out, sizeof(int), cudaMemcpyDeviceToHost));
        return r;
    }

    ~Model() {
        for (void* p : allocs) cudaFree(p);
    }
};

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
        fprintf(stderr, "usage: %s MODEL OUT --tokens LIST --steps N [--teacher LIST] [--max-ctx N] [--no-logits]\n",
                argv[0]);
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
    Model m;
    m.max_ctx = max_ctx;
    if (!m.load(argv[1])) return 3;
    const int V = m.vocab;
    FILE* f = fopen(argv[2], "wb");
    if (!f) return 4;
    const int hdr[4] = {0x46524546, V, (int)prompt.size(), steps};
    fwrite(hdr, 4, 4, f);
    float* logits = nullptr;
    const auto t0 = std::chrono::steady_clock::now();
    for (size_t i = 0; i < prompt.size(); ++i) logits = m.forward(prompt[i], (int)i);
    const auto t1 = std::chrono::steady_clock::now();
    std::vector<float> h(V);
    int pos = (int)prompt.size();
    double decode_s = 0.0;
    for (int s = 0; s < steps; ++s) {
        if (logits_out) CK(cudaMemcpy(h.data(), logits, (size_t)V * 4, cudaMemcpyDeviceToHost));
        const auto a = std::chrono::steady_clock::now();
        const int next = m.sample_greedy(logits);
        fwrite(&next, 4, 1, f);
        if (logits_out) fwrite(h.data(), 4, (size_t)V, f);
        const int feed = (s < (int)teacher.size()) ? teacher[s] : next;
        if (s + 1 < steps) logits = m.forward(feed, pos++);
        decode_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - a).count();
    }
    fclose(f);
    const double prefill_s = std::chrono::duration<double>(t1 - t0).count();
    printf("{\"ref_prefill_tok_s\": %.3f, \"ref_decode_tok_s\": %.3f, \"prompt\": %zu, \"steps\": %d}\n",
           prompt.size() / prefill_s, steps > 1 ? (steps - 1) / decode_s : 0.0, prompt.size(), steps);
    return 0;
}
