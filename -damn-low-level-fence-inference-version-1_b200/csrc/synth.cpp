// synth.cpp — seeded synthetic GGUF models with the shapes, tensor names, metadata types and
// weight distributions of the benchmark configurations (random-init; no real checkpoints exist
// offline). Generation is counter-based (SplitMix64 of seed, tensor number and word index), so a
// file is byte-reproducible and tensors are filled in parallel straight into a shared mapping.
//
// Distributions: Q6_K ql/qh uniform bytes (quants uniform in [-32, 31]), scales int8 uniform in
// [-127, 127], d = fp16(q6k_d); Q8_0 qs uniform in [-127, 127], d = fp16(q8_d); norm weights a
// constant; MoE router weights fp32 N(0, 0.02).
//
// Metadata written with exactly the types the reference loader demands
// (src/model/qwen3.cu:121-160): {arch}.block_count / embedding_length / feed_forward_length /
// attention.head_count / attention.head_count_kv / attention.key_length as UINT32,
// rope.freq_base and attention.layer_norm_rms_epsilon as FLOAT32, general.architecture STRING.
#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/fence_b200.h"
#include "gguf.h"

namespace fence {
int set_error(int code, const char* fmt, ...);

namespace {

inline uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
inline uint64_t stream_base(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ splitmix64(stream * 0xD1B54A32D192ED03ull + 0x8BB84B93962EACC9ull));
}

uint16_t f32_to_f16_bits(float f) {
    // round-to-nearest-even conversion of a normal/subnormal float to IEEE binary16
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t m = x & 0x7fffffu;
    if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0));
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const int shift = 14 - e;
        uint32_t hm = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1))) ++hm;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = m >> 13;
    const uint32_t rem = m & 0x1fffu;
    uint32_t out = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1))) ++out;
    return (uint16_t)out;
}

inline int8_t sym127(uint8_t r) { return (int8_t)((int)(r % 255u) - 127); }

void fill_q6k(uint8_t* dst, size_t b0, size_t nb, uint64_t base, uint16_t d) {
    for (size_t b = b0; b < b0 + nb; ++b) {
        uint8_t* blk = dst + (b - b0) * 210;
        uint64_t w[26];
        for (int k = 0; k < 26; ++k) w[k] = splitmix64(base + b * 26 + k);
        std::memcpy(blk, w, 192);  // ql[128] + qh[64]
        const uint8_t* sr = reinterpret_cast<const uint8_t*>(&w[24]);
        for (int k = 0; k < 16; ++k) blk[192 + k] = (uint8_t)sym127(sr[k]);
        std::memcpy(blk + 208, &d, 2);
    }
}
void fill_q8(uint8_t* dst, size_t b0, size_t nb, uint64_t base, uint16_t d) {
    for (size_t b = b0; b < b0 + nb; ++b) {
        uint8_t* blk = dst + (b - b0) * 34;
        uint64_t w[4];
        for (int k = 0; k < 4; ++k) w[k] = splitmix64(base + b * 4 + k);
        const uint8_t* r = reinterpret_cast<const uint8_t*>(w);
        std::memcpy(blk, &d, 2);
        for (int k = 0; k < 32; ++k) blk[2 + k] = (uint8_t)sym127(r[k]);
    }
}
void fill_normal(float* dst, size_t i0, size_t n, uint64_t base, float sigma) {
    for (size_t i = i0; i < i0 + n; ++i) {
        const uint64_t r = splitmix64(base + i);
        const double u1 = ((r >> 11) + 1.0) / 9007199254740993.0;            // (0, 1]
        const double u2 = (double)(splitmix64(base + i + 0x5bd1e995ull) >> 11) / 9007199254740992.0;
        dst[i - i0] = (float)(sigma * std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
    }
}

struct TensorPlan {
    std::string name;
    std::vector<uint64_t> dims;
    GGMLType type;
    uint64_t offset = 0;  // relative to data start
    uint64_t bytes = 0;
    int kind = 0;         // 0 quant, 1 const fp32, 2 normal fp32
    float value = 0.f;
};

uint64_t tensor_bytes(GGMLType t, const std::vector<uint64_t>& dims) {
    uint64_t n = 1;
    for (uint64_t d : dims) n *= d;
    const GGMLTypeInfo info = ggml_type_info(t);
    return (n + info.block_size - 1) / info.block_size * info.type_size;
}

struct Buf {
    std::vector<uint8_t> v;
    void u32(uint32_t x) { raw(&x, 4); }
    void u64(uint64_t x) { raw(&x, 8); }
    void f32(float x) { raw(&x, 4); }
    void raw(const void* p, size_t n) {
        const uint8_t* b = static_cast<const uint8_t*>(p);
        v.insert(v.end(), b, b + n);
    }
    void str(const std::string& s) {
        u64(s.size());
        raw(s.data(), s.size());
    }
    void kv_u32(const std::string& k, uint32_t x) { str(k); u32(4); u32(x); }
    void kv_f32(const std::string& k, float x) { str(k); u32(6); f32(x); }
    void kv_str(const std::string& k, const std::string& s) { str(k); u32(8); str(s); }
};

}  // namespace
}  // namespace fence

using namespace fence;

extern "C" void fence_synth_spec_default(fence_synth_spec* s) {
    std::memset(s, 0, sizeof *s);
    s->arch = "qwen3";
    s->n_layers = 2;
    s->embed_dim = 256;
    s->ff_dim = 512;
    s->n_heads = 4;
    s->n_kv_heads = 2;
    s->head_dim = 64;
    s->vocab_size = 1024;
    s->rope_freq_base = 1000000.0f;
    s->rms_eps = 1e-6f;
    s->linear_type = 14;
    s->embd_type = 8;
    s->qk_norm = 1;
    s->write_tokenizer = 0;
    s->gguf_version = 3;
    s->alignment = 32;
    s->seed = 1234;
    s->q6k_d = 1.5e-5f;
    s->q8_d = 1.6e-4f;
    s->norm_value = 1.0f;
}

extern "C" int fence_synth_fill_blocks(void* dst, int ggml_type, size_t n_blocks, uint64_t seed, uint64_t stream_id,
                                       float d) {
    if (!dst) return set_error(FENCE_E_ARG, "synth_fill_blocks: null destination");
    const uint64_t base = stream_base(seed, stream_id);
    const uint16_t dh = f32_to_f16_bits(d);
    if (ggml_type == 14) fill_q6k(static_cast<uint8_t*>(dst), 0, n_blocks, base, dh);
    else if (ggml_type == 8) fill_q8(static_cast<uint8_t*>(dst), 0, n_blocks, base, dh);
    else return set_error(FENCE_E_UNSUPPORTED, "synth_fill_blocks: type %d", ggml_type);
    return FENCE_OK;
}

extern "C" int fence_synth_write_gguf(const char* path, const fence_synth_spec* sp, int n_threads) {
    if (!path || !sp || !sp->arch) return set_error(FENCE_E_ARG, "synth: null argument");
    const fence_synth_spec& s = *sp;
    if (s.n_layers <= 0 || s.embed_dim <= 0 || s.ff_dim <= 0 || s.n_heads <= 0 || s.n_kv_heads <= 0 ||
        s.head_dim <= 0 || s.vocab_size <= 0 || s.n_heads % s.n_kv_heads)
        return set_error(FENCE_E_ARG, "synth: bad shape");
    const GGMLType lt = (GGMLType)s.linear_type, et = (GGMLType)s.embd_type;
    if ((lt != GGMLType::Q6_K && lt != GGMLType::Q8_0) || et != GGMLType::Q8_0)
        return set_error(FENCE_E_UNSUPPORTED, "synth: linear type must be Q6_K/Q8_0, embedding Q8_0");
    const uint32_t align = s.alignment ? s.alignment : 32;
    const std::string arch = s.arch;
    const uint64_t H = s.embed_dim, F = s.ff_dim, hd = s.head_dim, qd = (uint64_t)s.n_heads * hd,
                   kvd = (uint64_t)s.n_kv_heads * hd, V = s.vocab_size, E = s.n_experts;

    std::vector<TensorPlan> T;
    auto add = [&](const std::string& name, std::vector<uint64_t> dims, GGMLType t, int kind, float value) {
        TensorPlan p;
        p.name = name;
        p.dims = std::move(dims);
        p.type = t;
        p.kind = kind;
        p.value = value;
        p.bytes = tensor_bytes(t, p.dims);
        T.push_back(std::move(p));
    };
    add("token_embd.weight", {H, V}, et, 0, 0.f);
    add("output_norm.weight", {H}, GGMLType::F32, 1, s.norm_value);
    for (int l = 0; l < s.n_layers; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        add(p + "attn_norm.weight", {H}, GGMLType::F32, 1, s.norm_value);
        add(p + "attn_q.weight", {H, qd}, lt, 0, 0.f);
        add(p + "attn_k.weight", {H, kvd}, lt, 0, 0.f);
        add(p + "attn_v.weight", {H, kvd}, lt, 0, 0.f);
        if (s.qk_norm) {
            add(p + "attn_q_norm.weight", {hd}, GGMLType::F32, 1, s.norm_value);
            add(p + "attn_k_norm.weight", {hd}, GGMLType::F32, 1, s.norm_value);
        }
        add(p + "attn_output.weight", {qd, H}, lt, 0, 0.f);
        add(p + "ffn_norm.weight", {H}, GGMLType::F32, 1, s.norm_value);
        if (E > 0) {
            add(p + "ffn_gate_inp.weight", {H, E}, GGMLType::F32, 2, 0.02f);
            add(p + "ffn_gate_exps.weight", {H, F, E}, lt, 0, 0.f);
            add(p + "ffn_up_exps.weight", {H, F, E}, lt, 0, 0.f);
            add(p + "ffn_down_exps.weight", {F, H, E}, lt, 0, 0.f);
        } else {
            add(p + "ffn_gate.weight", {H, F}, lt, 0, 0.f);
            add(p + "ffn_up.weight", {H, F}, lt, 0, 0.f);
            add(p + "ffn_down.weight", {F, H}, lt, 0, 0.f);
        }
    }
    uint64_t off = 0;
    for (auto& t : T) {
        t.offset = off;
        off += (t.bytes + align - 1) / align * align;
    }
    const uint64_t data_bytes = off;

    Buf hb;
    hb.u32(0x46554747u);
    hb.u32(s.gguf_version == 2 ? 2u : 3u);
    hb.u64(T.size());
    uint64_t n_kv = 11 + (E > 0 ? 2 : 0) + (s.write_tokenizer ? 2 : 0);
    hb.u64(n_kv);
    hb.kv_str("general.architecture", arch);
    hb.kv_u32("general.alignment", align);
    hb.kv_u32(arch + ".block_count", (uint32_t)s.n_layers);
    hb.kv_u32(arch + ".context_length", 131072u);
    hb.kv_u32(arch + ".embedding_length", (uint32_t)H);
    hb.kv_u32(arch + ".feed_forward_length", (uint32_t)F);
    hb.kv_u32(arch + ".attention.head_count", (uint32_t)s.n_heads);
    hb.kv_u32(arch + ".attention.head_count_kv", (uint32_t)s.n_kv_heads);
    hb.kv_u32(arch + ".attention.key_length", (uint32_t)hd);
    hb.kv_f32(arch + ".rope.freq_base", s.rope_freq_base);
    hb.kv_f32(arch + ".attention.layer_norm_rms_epsilon", s.rms_eps);
    if (E > 0) {
        hb.kv_u32(arch + ".expert_count", (uint32_t)E);
        hb.kv_u32(arch + ".expert_used_count", (uint32_t)s.n_experts_used);
    }
    if (s.write_tokenizer) {
        // token strings "<id>" and an eos id outside the vocabulary so generation never stops early
        hb.str("tokenizer.ggml.tokens");
        hb.u32(9);
        hb.u32(8);
        hb.u64(V);
        for (uint64_t i = 0; i < V; ++i) hb.str("<" + std::to_string(i) + ">");
        hb.kv_u32("tokenizer.ggml.eos_token_id", (uint32_t)V);
    }
    for (auto& t : T) {
        hb.str(t.name);
        hb.u32((uint32_t)t.dims.size());
        for (uint64_t d : t.dims) hb.u64(d);
        hb.u32((uint32_t)t.type);
        hb.u64(t.offset);
    }
    const uint64_t header = hb.v.size();
    const uint64_t data_start = (header + align - 1) / align * align;
    const uint64_t total = data_start + data_bytes;

    const int fd = ::open(path, O_RDWR | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return set_error(FENCE_E_IO, "synth: cannot create '%s'", path);
    if (ftruncate(fd, (off_t)total) != 0) {
        ::close(fd);
        return set_error(FENCE_E_IO, "synth: cannot size '%s' to %llu bytes", path, (unsigned long long)total);
    }
    void* m = mmap(nullptr, total, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    if (m == MAP_FAILED) {
        ::close(fd);
        return set_error(FENCE_E_IO, "synth: mmap of '%s' failed", path);
    }
    uint8_t* base = static_cast<uint8_t*>(m);
    std::memcpy(base, hb.v.data(), header);
    std::memset(base + header, 0, data_start - header);

    // work list: (tensor, first block, block count) chunks of ~4 MB
    struct Job { size_t t; uint64_t b0, nb; };
    std::vector<Job> jobs;
    for (size_t i = 0; i < T.size(); ++i) {
        const GGMLTypeInfo info = ggml_type_info(T[i].type);
        const uint64_t nblocks = T[i].bytes / info.type_size;
        const uint64_t per = std::max<uint64_t>(1, (4u << 20) / info.type_size);
        for (uint64_t b = 0; b < nblocks; b += per) jobs.push_back({i, b, std::min(per, nblocks - b)});
        // zero the alignment padding after the tensor
        const uint64_t pad_end = (T[i].bytes + align - 1) / align * align;
        std::memset(base + data_start + T[i].offset + T[i].bytes, 0, pad_end - T[i].bytes);
    }
    const uint16_t d6 = f32_to_f16_bits(s.q6k_d), d8 = f32_to_f16_bits(s.q8_d);
    const int nt = n_threads > 0 ? n_threads : std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::thread> pool;
    std::atomic_size_t next{0};
    for (int w = 0; w < nt; ++w) {
        pool.emplace_back([&]() {
            for (;;) {
                const size_t j = next.fetch_add(1);
                if (j >= jobs.size()) break;
                const Job& jb = jobs[j];
                const TensorPlan& t = T[jb.t];
                const uint64_t sb = stream_base(s.seed, jb.t);
                uint8_t* dst = base + data_start + t.offset;
                if (t.kind == 0) {
                    if (t.type == GGMLType::Q6_K) fill_q6k(dst + jb.b0 * 210, jb.b0, jb.nb, sb, d6);
                    else fill_q8(dst + jb.b0 * 34, jb.b0, jb.nb, sb, d8);
                } else if (t.kind == 1) {
                    float* f = reinterpret_cast<float*>(dst) + jb.b0;
                    for (uint64_t i = 0; i < jb.nb; ++i) f[i] = t.value;
                } else {
                    fill_normal(reinterpret_cast<float*>(dst) + jb.b0, jb.b0, jb.nb, sb, t.value);
                }
            }
        });
    }
    for (auto& th : pool) th.join();
    const int rc = munmap(m, total);
    ::close(fd);
    if (rc != 0) return set_error(FENCE_E_IO, "synth: munmap failed");
    return FENCE_OK;
}
