/*
 * fence_oracle.c — CPU restatement of the reference's token loop (test infrastructure only; see
 * fence_oracle.h). Plain C11 + pthreads.
 */
#define _GNU_SOURCE
#include "fence_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------ half / bfloat16 */
float oracle_h2f(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
    float f;
    if (e == 0) {
        f = ldexpf((float)m, -24);
        return s ? -f : f;
    }
    uint32_t bits;
    if (e == 31) bits = s | 0x7f800000u | (m << 13);
    else bits = s | ((e + 112) << 23) | (m << 13);
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t oracle_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t ex = (int32_t)((x >> 23) & 0xff);
    uint32_t m = x & 0x7fffffu;
    if (ex == 0xff) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0));
    int32_t e = ex - 127 + 15;
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
    uint32_t out = sign | ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (out & 1))) ++out;
    return (uint16_t)out;
}

float oracle_bf2f(uint16_t h) {
    const uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t oracle_f2bf(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7f800000u) == 0x7f800000u && (x & 0x7fffffu)) return (uint16_t)((x >> 16) | 0x40u);
    const uint32_t lsb = (x >> 16) & 1u;
    x += 0x7fffu + lsb;
    return (uint16_t)(x >> 16);
}

/* ------------------------------------------------------------------ Q6_K / Q8_0 */
/* Element i of a super-block: half = i/128, col = (i%128)/32, l = i%32; low nibble from
 * ql[64*half + l + 32*(col&1)] (high nibble when col >= 2), high 2 bits from
 * qh[32*half + l] >> 2*col (tests/test_gemv_q6k.cu:82-109, src/kernels/q6k_dot.cuh:35-62). */
static inline int q6_at(const uint8_t* blk, int i) {
    const int half = i / 128, rem = i % 128, col = rem / 32, l = rem % 32;
    const int ql_idx = 64 * half + l + ((col & 1) ? 32 : 0);
    const int ql_shift = (col >= 2) ? 4 : 0;
    const int qh_idx = 32 * half + l;
    const int qh_shift = 2 * col;
    const int lo = (blk[ql_idx] >> ql_shift) & 0xF;
    const int hi = (blk[128 + qh_idx] >> qh_shift) & 0x3;
    return (lo | (hi << 4)) - 32;
}

void oracle_q6k_dequant(const uint8_t* blk, double* w) {
    uint16_t dh;
    memcpy(&dh, blk + 208, 2);
    const double d = oracle_h2f(dh);
    for (int i = 0; i < 256; ++i) w[i] = d * (double)(int8_t)blk[192 + i / 16] * (double)q6_at(blk, i);
}

double oracle_q6k_dot_block(const uint8_t* blk, const uint16_t* x) {
    uint16_t dh;
    memcpy(&dh, blk + 208, 2);
    const double d = oracle_h2f(dh);
    double sum = 0.0;
    for (int i = 0; i < 256; ++i) {
        const double sc = (double)(int8_t)blk[192 + i / 16];
        sum += d * sc * (double)q6_at(blk, i) * (double)oracle_h2f(x[i]);
    }
    return sum;
}

typedef struct {
    int kind; /* 0 = q6k, 1 = q8_0 */
    const uint8_t* W;
    const void* x;
    double* y;
    int M, K, r0, r1;
} gemv_job;

static void* gemv_worker(void* p) {
    gemv_job* j = (gemv_job*)p;
    if (j->kind == 0) {
        const int nb = j->K / 256;
        const uint16_t* x = (const uint16_t*)j->x;
        for (int r = j->r0; r < j->r1; ++r) {
            double s = 0.0;
            for (int b = 0; b < nb; ++b) s += oracle_q6k_dot_block(j->W + ((size_t)r * nb + b) * 210, x + b * 256);
            j->y[r] = s;
        }
    } else {
        const int nb = j->K / 32;
        const float* x = (const float*)j->x;
        for (int r = j->r0; r < j->r1; ++r) {
            double s = 0.0;
            for (int b = 0; b < nb; ++b) {
                const uint8_t* blk = j->W + ((size_t)r * nb + b) * 34;
                uint16_t dh;
                memcpy(&dh, blk, 2);
                double bs = 0.0;
                for (int i = 0; i < 32; ++i) bs += (double)(int8_t)blk[2 + i] * (double)x[b * 32 + i];
                s += (double)oracle_h2f(dh) * bs;
            }
            j->y[r] = s;
        }
    }
    return NULL;
}

static void run_gemv(int kind, const uint8_t* W, const void* x, double* y, int M, int K, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > M) nthreads = M;
    gemv_job jobs[256];
    pthread_t th[256];
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = (gemv_job){kind, W, x, y, M, K, (int)((long)M * t / nthreads), (int)((long)M * (t + 1) / nthreads)};
        if (t > 0) pthread_create(&th[t], NULL, gemv_worker, &jobs[t]);
    }
    gemv_worker(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
}

void oracle_gemv_q6k(const uint8_t* W, const uint16_t* x, double* y, int M, int K, int nthreads) {
    run_gemv(0, W, x, y, M, K, nthreads);
}
void oracle_gemv_q8_0(const uint8_t* W, const float* x, double* y, int M, int K, int nthreads) {
    run_gemv(1, W, x, y, M, K, nthreads);
}

void oracle_embed_q8_0(float* out, const uint8_t* W, int token, int dim) {
    const int nb = dim / 32;
    for (int i = 0; i < dim; ++i) {
        const uint8_t* blk = W + ((size_t)token * nb + i / 32) * 34;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        out[i] = oracle_h2f(dh) * (float)(int8_t)blk[2 + (i % 32)];
    }
}

/* ------------------------------------------------------------------ elementwise / norms */
void oracle_rms_norm(float* out, const float* x, const float* w, int n, float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    const double r = 1.0 / sqrt(ss / (double)n + (double)eps);
    for (int i = 0; i < n; ++i) out[i] = (float)((double)w[i] * (double)x[i] * r);
}

void oracle_rms_norm_per_head(float* x, const float* w, int n_heads, int hd, float eps) {
    for (int h = 0; h < n_heads; ++h) oracle_rms_norm(x + (size_t)h * hd, x + (size_t)h * hd, w, hd, eps);
}

void oracle_rope(float* q, float* k, int hd, int nq, int nkv, int pos, float base) {
    const int half = hd / 2;
    for (int t = 0; t < 2; ++t) {
        float* v = t == 0 ? q : k;
        const int nh = t == 0 ? nq : nkv;
        for (int h = 0; h < nh; ++h)
            for (int i = 0; i < half; ++i) {
                const double ang = (double)pos * pow((double)base, -2.0 * i / (double)hd);
                const double c = cos(ang), s = sin(ang);
                float* p = v + (size_t)h * hd;
                const double a = p[i], b = p[i + half];
                p[i] = (float)(a * (double)(float)c - b * (double)(float)s);
                p[i + half] = (float)(a * (double)(float)s + b * (double)(float)c);
            }
    }
}

void oracle_silu_mul(float* out, const float* g, const float* u, int n) {
    for (int i = 0; i < n; ++i) {
        const double gg = g[i];
        out[i] = (float)(gg / (1.0 + exp(-gg)) * (double)u[i]);
    }
}

void oracle_softmax(float* x, int n) {
    double mx = -1e30;
    for (int i = 0; i < n; ++i)
        if (x[i] > mx) mx = x[i];
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += exp((double)x[i] - mx);
    for (int i = 0; i < n; ++i) x[i] = (float)(exp((double)x[i] - mx) / s);
}

void oracle_attention(float* out, const float* q, const uint16_t* kc, const uint16_t* vc, int kv_bf16,
                      long stride_t, long stride_h, int hd, int nq, int nkv, int seq_len) {
    const int G = nq / nkv;
    double* sc = (double*)malloc(sizeof(double) * (size_t)seq_len);
    const double scale = 1.0 / sqrt((double)hd);
    for (int qh = 0; qh < nq; ++qh) {
        const int h = qh / G;
        const float* qv = q + (size_t)qh * hd;
        double mx = -INFINITY;
        for (int t = 0; t < seq_len; ++t) {
            const uint16_t* kr = kc + (size_t)t * stride_t + (size_t)h * stride_h;
            double dot = 0.0;
            for (int d = 0; d < hd; ++d) dot += (double)qv[d] * (double)(kv_bf16 ? oracle_bf2f(kr[d]) : oracle_h2f(kr[d]));
            sc[t] = dot * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        double sum = 0.0;
        for (int t = 0; t < seq_len; ++t) {
            sc[t] = exp(sc[t] - mx);
            sum += sc[t];
        }
        for (int d = 0; d < hd; ++d) {
            double acc = 0.0;
            for (int t = 0; t < seq_len; ++t) {
                const uint16_t* vr = vc + (size_t)t * stride_t + (size_t)h * stride_h;
                acc += sc[t] * (double)(kv_bf16 ? oracle_bf2f(vr[d]) : oracle_h2f(vr[d]));
            }
            out[(size_t)qh * hd + d] = (float)(acc / sum);
        }
    }
    free(sc);
}

/* Thread t (of 256) scans i = t, t+256, ... with strict '>' from -1e30; the 256 results are
 * tree-reduced with strict '>' keeping the lower thread on ties (ops.cuh:476-498). */
int oracle_argmax(const float* x, int n) {
    float bv[256];
    int bi[256];
    for (int t = 0; t < 256; ++t) {
        bv[t] = -1e30f;
        bi[t] = 0;
        for (int i = t; i < n; i += 256)
            if (x[i] > bv[t]) {
                bv[t] = x[i];
                bi[t] = i;
            }
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int t = 0; t < s; ++t)
            if (bv[t + s] > bv[t]) {
                bv[t] = bv[t + s];
                bi[t] = bi[t + s];
            }
    return bi[0];
}

/* ------------------------------------------------------------------ minimal GGUF reader */
typedef struct {
    char name[96];
    uint32_t n_dims;
    uint64_t dims[4];
    uint32_t type;
    uint64_t offset;
    const uint8_t* data;
} o_tensor;

typedef struct {
    char key[96];
    uint32_t type; /* 4 u32, 5 i32, 6 f32, 8 string */
    uint32_t u;
    float f;
    char s[64];
} o_kv;

struct oracle_model {
    void* map;
    size_t size;
    o_kv* kv;
    int n_kv;
    o_tensor* t;
    int n_t;
    int L, H, F, nh, nkv, hd, V, max_ctx, lin_type, qk_norm, kv_bf16, nthreads;
    float base, eps;
    uint16_t *kc, *vc;                 /* [L][max_ctx][nkv*hd] */
    float *hidden, *res, *normed, *q, *k, *v, *att, *gate, *up, *act, *final_hidden;
    uint16_t* xh;
    double* ybuf;
    const uint8_t *embd;
    const float* onorm;
    /* sparse MoE FFN (no counterpart in the reference: Mixtral routing, see oracle_forward) */
    int n_exp, n_used;
    float *moe_out, *moe_tmp;
    int* last_sel;       /* [L][n_used] experts chosen at the last forward */
    float route_margin;  /* smallest gap between the last chosen and the best unchosen router logit */
    struct {
        const uint8_t *q, *k, *v, *o, *g, *u, *d;
        int tq, to, tg, td;
        const float *an, *fn, *qn, *kn, *qb, *kb, *vb;
        const float* rt; /* router [n_exp][H] fp32 (MoE) */
    } * layer;
};

static int rd(const uint8_t** p, const uint8_t* end, void* dst, size_t n) {
    if ((size_t)(end - *p) < n) return -1;
    memcpy(dst, *p, n);
    *p += n;
    return 0;
}
static int skip_val(const uint8_t** p, const uint8_t* end, uint32_t ty) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (ty == 8) {
        uint64_t n;
        if (rd(p, end, &n, 8)) return -1;
        if ((uint64_t)(end - *p) < n) return -1;
        *p += n;
        return 0;
    }
    if (ty == 9) {
        uint32_t at;
        uint64_t n;
        if (rd(p, end, &at, 4) || rd(p, end, &n, 8)) return -1;
        for (uint64_t i = 0; i < n; ++i)
            if (skip_val(p, end, at)) return -1;
        return 0;
    }
    if (ty > 12) return -1;
    if ((size_t)(end - *p) < (size_t)sz[ty]) return -1;
    *p += sz[ty];
    return 0;
}
static const o_kv* find_kv(const oracle_model* m, const char* key) {
    for (int i = 0; i < m->n_kv; ++i)
        if (!strcmp(m->kv[i].key, key)) return &m->kv[i];
    return NULL;
}
static const o_tensor* find_t(const oracle_model* m, const char* name) {
    for (int i = 0; i < m->n_t; ++i)
        if (!strcmp(m->t[i].name, name)) return &m->t[i];
    return NULL;
}

static int parse_gguf(oracle_model* m) {
    const uint8_t* base = (const uint8_t*)m->map;
    const uint8_t *p = base, *end = base + m->size;
    uint32_t magic, ver;
    uint64_t nt, nkv;
    if (rd(&p, end, &magic, 4) || magic != 0x46554747u) return -1;
    if (rd(&p, end, &ver, 4) || ver < 2 || ver > 3) return -1;
    if (rd(&p, end, &nt, 8) || rd(&p, end, &nkv, 8)) return -1;
    m->kv = (o_kv*)calloc(nkv ? nkv : 1, sizeof(o_kv));
    uint32_t align = 32;
    for (uint64_t i = 0; i < nkv; ++i) {
        uint64_t kl;
        if (rd(&p, end, &kl, 8) || (uint64_t)(end - p) < kl) return -1;
        o_kv kv;
        memset(&kv, 0, sizeof kv);
        memcpy(kv.key, p, kl < 95 ? kl : 95);
        p += kl;
        uint32_t ty;
        if (rd(&p, end, &ty, 4)) return -1;
        kv.type = ty;
        if (ty == 4 || ty == 5) {
            if (rd(&p, end, &kv.u, 4)) return -1;
        } else if (ty == 6) {
            if (rd(&p, end, &kv.f, 4)) return -1;
        } else if (ty == 8) {
            uint64_t sl;
            if (rd(&p, end, &sl, 8) || (uint64_t)(end - p) < sl) return -1;
            memcpy(kv.s, p, sl < 63 ? sl : 63);
            p += sl;
        } else if (skip_val(&p, end, ty)) {
            return -1;
        }
        if (!strcmp(kv.key, "general.alignment") && ty == 4 && kv.u) align = kv.u;
        m->kv[m->n_kv++] = kv;
    }
    m->t = (o_tensor*)calloc(nt ? nt : 1, sizeof(o_tensor));
    for (uint64_t i = 0; i < nt; ++i) {
        o_tensor t;
        memset(&t, 0, sizeof t);
        uint64_t nl;
        if (rd(&p, end, &nl, 8) || (uint64_t)(end - p) < nl) return -1;
        memcpy(t.name, p, nl < 95 ? nl : 95);
        p += nl;
        if (rd(&p, end, &t.n_dims, 4) || t.n_dims > 4) return -1;
        for (uint32_t d = 0; d < 4; ++d) t.dims[d] = 1;
        for (uint32_t d = 0; d < t.n_dims; ++d)
            if (rd(&p, end, &t.dims[d], 8)) return -1;
        if (rd(&p, end, &t.type, 4) || rd(&p, end, &t.offset, 8)) return -1;
        m->t[m->n_t++] = t;
    }
    const size_t hdr = (size_t)(p - base);
    const size_t data = hdr + (align - hdr % align) % align;
    for (int i = 0; i < m->n_t; ++i) {
        if (data + m->t[i].offset >= m->size) return -1;
        m->t[i].data = base + data + m->t[i].offset;
    }
    return 0;
}

static uint32_t kv_u32(const oracle_model* m, const char* arch, const char* suffix, uint32_t dflt, int* ok) {
    char key[128];
    snprintf(key, sizeof key, "%s.%s", arch, suffix);
    const o_kv* kv = find_kv(m, key);
    if (!kv || kv->type != 4) {
        if (ok) *ok = 0;
        return dflt;
    }
    return kv->u;
}
static float kv_f32(const oracle_model* m, const char* arch, const char* suffix, float dflt) {
    char key[128];
    snprintf(key, sizeof key, "%s.%s", arch, suffix);
    const o_kv* kv = find_kv(m, key);
    return (kv && kv->type == 6) ? kv->f : dflt;
}

oracle_model* oracle_model_open(const char* path, int max_ctx, int kv_bf16, int nthreads) {
    oracle_model* m = (oracle_model*)calloc(1, sizeof(oracle_model));
    const int fd = open(path, O_RDONLY);
    if (fd < 0) {
        free(m);
        return NULL;
    }
    struct stat st;
    fstat(fd, &st);
    m->size = (size_t)st.st_size;
    m->map = mmap(NULL, m->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m->map == MAP_FAILED || parse_gguf(m)) {
        if (m->map != MAP_FAILED) munmap(m->map, m->size);
        free(m->kv);
        free(m->t);
        free(m);
        return NULL;
    }
    const o_kv* a = find_kv(m, "general.architecture");
    const char* arch = (a && a->type == 8) ? a->s : "qwen2";
    int ok = 1;
    m->L = (int)kv_u32(m, arch, "block_count", 0, &ok);
    m->H = (int)kv_u32(m, arch, "embedding_length", 0, &ok);
    m->F = (int)kv_u32(m, arch, "feed_forward_length", 0, &ok);
    m->nh = (int)kv_u32(m, arch, "attention.head_count", 0, &ok);
    m->nkv = (int)kv_u32(m, arch, "attention.head_count_kv", 0, &ok);
    if (!ok || !m->nh) {
        oracle_model_close(m);
        return NULL;
    }
    m->hd = (int)kv_u32(m, arch, "attention.key_length", (uint32_t)(m->H / m->nh), NULL);
    m->base = kv_f32(m, arch, "rope.freq_base", 10000.0f);
    m->eps = kv_f32(m, arch, "attention.layer_norm_rms_epsilon", 1e-5f);
    const o_tensor* e = find_t(m, "token_embd.weight");
    if (!e) {
        oracle_model_close(m);
        return NULL;
    }
    m->V = (int)e->dims[1];
    m->embd = e->data;
    m->max_ctx = max_ctx;
    m->kv_bf16 = kv_bf16;
    m->nthreads = nthreads > 0 ? nthreads : 1;
    const o_tensor* on = find_t(m, "output_norm.weight");
    m->onorm = on ? (const float*)on->data : NULL;
    m->n_exp = (int)kv_u32(m, arch, "expert_count", 0, NULL);
    m->n_used = m->n_exp > 0 ? (int)kv_u32(m, arch, "expert_used_count", 2, NULL) : 0;
    if (m->n_exp < 0 || m->n_exp > 64 || m->n_used < 0 || m->n_used > m->n_exp) {
        oracle_model_close(m);
        return NULL;
    }
    m->layer = calloc((size_t)m->L, sizeof(*m->layer));
    char name[128];
#define T(s) (snprintf(name, sizeof name, "blk.%d." s, l), find_t(m, name))
    for (int l = 0; l < m->L; ++l) {
        const o_tensor *q = T("attn_q.weight"), *k = T("attn_k.weight"), *v = T("attn_v.weight"),
                       *o = T("attn_output.weight"), *g = T("ffn_gate.weight"), *u = T("ffn_up.weight"),
                       *d = T("ffn_down.weight"), *an = T("attn_norm.weight"), *fn = T("ffn_norm.weight"),
                       *qn = T("attn_q_norm.weight"), *kn = T("attn_k_norm.weight"), *qb = T("attn_q.bias"),
                       *kb = T("attn_k.bias"), *vb = T("attn_v.bias"), *rt = T("ffn_gate_inp.weight");
        if (m->n_exp > 0) { /* experts: [K, M, n_exp] tensors, expert e's rows contiguous */
            g = T("ffn_gate_exps.weight");
            u = T("ffn_up_exps.weight");
            d = T("ffn_down_exps.weight");
            if (!rt || rt->type != 0 || rt->dims[0] != (uint64_t)m->H || rt->dims[1] != (uint64_t)m->n_exp) rt = NULL;
            if (!rt) {
                oracle_model_close(m);
                return NULL;
            }
            m->layer[l].rt = (const float*)rt->data;
        }
        if (!q || !k || !v || !o || !g || !u || !d || !an || !fn || !m->onorm) {
            oracle_model_close(m);
            return NULL;
        }
        m->layer[l].q = q->data;
        m->layer[l].k = k->data;
        m->layer[l].v = v->data;
        m->layer[l].o = o->data;
        m->layer[l].g = g->data;
        m->layer[l].u = u->data;
        m->layer[l].d = d->data;
        m->layer[l].tq = (int)q->type;
        m->layer[l].to = (int)o->type;
        m->layer[l].tg = (int)g->type;
        m->layer[l].td = (int)d->type;
        m->layer[l].an = (const float*)an->data;
        m->layer[l].fn = (const float*)fn->data;
        m->layer[l].qn = (qn && kn) ? (const float*)qn->data : NULL;
        m->layer[l].kn = (qn && kn) ? (const float*)kn->data : NULL;
        m->layer[l].qb = qb ? (const float*)qb->data : NULL;
        m->layer[l].kb = kb ? (const float*)kb->data : NULL;
        m->layer[l].vb = vb ? (const float*)vb->data : NULL;
        if (l == 0) {
            m->lin_type = (int)q->type;
            m->qk_norm = (qn && kn) ? 1 : 0;
        }
    }
#undef T
    const size_t qd = (size_t)m->nh * m->hd, kvd = (size_t)m->nkv * m->hd;
    const size_t mx = (size_t)(m->F > m->H ? m->F : m->H) + qd + (size_t)m->V;
    m->kc = (uint16_t*)calloc((size_t)m->L * max_ctx * kvd, 2);
    m->vc = (uint16_t*)calloc((size_t)m->L * max_ctx * kvd, 2);
    m->hidden = (float*)calloc(m->H, 4);
    m->res = (float*)calloc(m->H, 4);
    m->normed = (float*)calloc(m->H, 4);
    m->final_hidden = (float*)calloc(m->H, 4);
    m->q = (float*)calloc(qd, 4);
    m->k = (float*)calloc(kvd, 4);
    m->v = (float*)calloc(kvd, 4);
    m->att = (float*)calloc(qd, 4);
    m->gate = (float*)calloc(m->F, 4);
    m->up = (float*)calloc(m->F, 4);
    m->act = (float*)calloc(m->F, 4);
    m->xh = (uint16_t*)calloc(mx, 2);
    m->ybuf = (double*)calloc(mx, 8);
    m->moe_out = (float*)calloc(m->H, 4);
    m->moe_tmp = (float*)calloc(m->H, 4);
    m->last_sel = (int*)calloc((size_t)m->L * (m->n_used > 0 ? m->n_used : 1), sizeof(int));
    if (!m->kc || !m->vc) {
        oracle_model_close(m);
        return NULL;
    }
    return m;
}

void oracle_model_close(oracle_model* m) {
    if (!m) return;
    if (m->map && m->map != MAP_FAILED) munmap(m->map, m->size);
    free(m->kv);
    free(m->t);
    free(m->layer);
    free(m->kc);
    free(m->vc);
    free(m->hidden);
    free(m->res);
    free(m->normed);
    free(m->final_hidden);
    free(m->q);
    free(m->k);
    free(m->v);
    free(m->att);
    free(m->gate);
    free(m->up);
    free(m->act);
    free(m->xh);
    free(m->ybuf);
    free(m->moe_out);
    free(m->moe_tmp);
    free(m->last_sel);
    free(m);
}

/* Benchmark support (not in the reference): fills the K and V cache rows of positions [0, n_pos)
 * of every layer with seeded values (SplitMix64 words mapped to about N(0, 0.5) through a sum of
 * four uniforms), rounded to the cache type, as a stand-in for a prefill of n_pos tokens: the
 * decode steps after it do exactly the work they would do after a real prefill. */
static uint64_t o_splitmix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
int oracle_model_fill_kv(oracle_model* m, int n_pos, uint64_t seed) {
    if (!m || n_pos < 0 || n_pos > m->max_ctx) return -1;
    const size_t kvd = (size_t)m->nkv * m->hd;
    for (int l = 0; l < m->L; ++l)
        for (int c = 0; c < 2; ++c) {
            uint16_t* base = (c ? m->vc : m->kc) + (size_t)l * m->max_ctx * kvd;
            for (size_t i = 0; i < (size_t)n_pos * kvd; ++i) {
                const uint64_t r = o_splitmix(seed ^ ((uint64_t)(2 * l + c) << 40) ^ i);
                float u = 0.f;
                for (int j = 0; j < 4; ++j) u += (float)((r >> (16 * j)) & 0xffff) / 65536.0f;
                const float v = (u - 2.0f) * 0.866f;
                base[i] = m->kv_bf16 ? oracle_f2bf(v) : oracle_f2h(v);
            }
        }
    return 0;
}

void oracle_model_dims(const oracle_model* m, int* d) {
    d[0] = m->L;
    d[1] = m->H;
    d[2] = m->F;
    d[3] = m->nh;
    d[4] = m->nkv;
    d[5] = m->hd;
    d[6] = m->V;
    d[7] = m->max_ctx;
    d[8] = m->lin_type;
    d[9] = m->qk_norm;
}

void oracle_model_moe(const oracle_model* m, int* n_exp, int* n_used) {
    *n_exp = m->n_exp;
    *n_used = m->n_used;
}

float oracle_last_route(const oracle_model* m, int* sel) {
    if (sel && m->n_used > 0) memcpy(sel, m->last_sel, (size_t)m->L * m->n_used * sizeof(int));
    return m->route_margin;
}

void oracle_last_hidden(const oracle_model* m, float* out) { memcpy(out, m->final_hidden, (size_t)m->H * 4); }

/* y = W x for one linear of either type; Q6_K inputs are rounded to fp16 first, as the reference
 * does with f32_to_f16 before every gemv_q6k (qwen3.cu:278,310,325,336); Q8_0 takes fp32 x. */
static void linear(oracle_model* m, int type, const uint8_t* W, const float* x, float* y, int M, int K) {
    if (type == 14) {
        for (int i = 0; i < K; ++i) m->xh[i] = oracle_f2h(x[i]);
        oracle_gemv_q6k(W, m->xh, m->ybuf, M, K, m->nthreads);
    } else {
        oracle_gemv_q8_0(W, x, m->ybuf, M, K, m->nthreads);
    }
    for (int i = 0; i < M; ++i) y[i] = (float)m->ybuf[i];
}

static size_t o_row_bytes(int type, int K) { return type == 14 ? (size_t)K / 256 * 210 : (size_t)K / 32 * 34; }

/* Sparse MoE FFN of layer l on m->normed (no counterpart in the reference, which has no expert
 * tensors; Mixtral's published routing over the reference's per-op math): router logits
 * r_e = sum_k W_r[e][k] * normed[k] (fp32 weights, accumulated in double), the n_used largest
 * (ties to the smaller expert index), weights softmax over the chosen logits (the same as the
 * full softmax renormalised over them), and out = sum_s w_s * down_e(SwiGLU(gate_e x, up_e x)),
 * each expert's linears exactly the dense FFN's (qwen3.cu:317-341: fp16-rounded inputs for Q6_K).
 * No reference fixture exists for it (the reference has no expert tensors); tests/test_moe_hf_pin.py
 * pins it to the Mixtral sparse-MoE block of Hugging Face transformers, run in float64 on the same
 * dequantised weights. */
static void moe_ffn(oracle_model* m, int l) {
    const __typeof__(m->layer[0])* w = &m->layer[l];
    const int H = m->H, F = m->F, E = m->n_exp, K = m->n_used;
    double r[64];
    for (int e = 0; e < E; ++e) {
        double a = 0.0;
        for (int k = 0; k < H; ++k) a += (double)w->rt[(size_t)e * H + k] * (double)m->normed[k];
        r[e] = a;
    }
    int sel[64];
    int used[64] = {0};
    for (int s = 0; s < K; ++s) {
        int b = -1;
        for (int e = 0; e < E; ++e)
            if (!used[e] && (b < 0 || r[e] > r[b])) b = e;
        sel[s] = b;
        used[b] = 1;
    }
    double margin = 1e30;
    for (int e = 0; e < E; ++e)
        if (!used[e] && r[sel[K - 1]] - r[e] < margin) margin = r[sel[K - 1]] - r[e];
    if (l == 0 || margin < m->route_margin) m->route_margin = (float)margin;
    double z = 0.0, p[64];
    for (int s = 0; s < K; ++s) z += (p[s] = exp(r[sel[s]] - r[sel[0]]));
    for (int i = 0; i < H; ++i) m->moe_out[i] = 0.f;
    for (int s = 0; s < K; ++s) {
        const int e = sel[s];
        m->last_sel[(size_t)l * K + s] = e;
        const float ws = (float)(p[s] / z);
        linear(m, w->tg, w->g + (size_t)e * F * o_row_bytes(w->tg, H), m->normed, m->gate, F, H);
        linear(m, w->tg, w->u + (size_t)e * F * o_row_bytes(w->tg, H), m->normed, m->up, F, H);
        oracle_silu_mul(m->act, m->gate, m->up, F);
        linear(m, w->td, w->d + (size_t)e * H * o_row_bytes(w->td, F), m->act, m->moe_tmp, H, F);
        for (int i = 0; i < H; ++i) m->moe_out[i] += ws * m->moe_tmp[i];
    }
}

/* Test hook: moe_ffn of layer l (the function every MoE forward above runs) on a given normed
 * input; out[H] = the block's output before the residual add, sel[n_used] = the chosen experts.
 * Lets the tests set the oracle's MoE block beside a published implementation on the same input. */
int oracle_moe_ffn_apply(oracle_model* m, int l, const float* normed, float* out, int* sel) {
    if (!m || l < 0 || l >= m->L || m->n_exp <= 0 || !normed || !out) return -1;
    memcpy(m->normed, normed, (size_t)m->H * 4);
    moe_ffn(m, l);
    memcpy(out, m->moe_out, (size_t)m->H * 4);
    if (sel) memcpy(sel, m->last_sel + (size_t)l * m->n_used, (size_t)m->n_used * sizeof(int));
    return 0;
}

int oracle_forward(oracle_model* m, int token, int pos, float* logits) {
    if (token < 0 || token >= m->V || pos < 0 || pos >= m->max_ctx) return -1;
    const int H = m->H, F = m->F, hd = m->hd, nh = m->nh, nkv = m->nkv;
    const int qd = nh * hd, kvd = nkv * hd;
    oracle_embed_q8_0(m->hidden, m->embd, token, H);
    for (int l = 0; l < m->L; ++l) {
        const __typeof__(m->layer[0])* w = &m->layer[l];
        /* attention block, qwen3.cu:267-315 */
        memcpy(m->res, m->hidden, (size_t)H * 4);
        oracle_rms_norm(m->normed, m->hidden, w->an, H, m->eps);
        linear(m, w->tq, w->q, m->normed, m->q, qd, H);
        linear(m, w->tq, w->k, m->normed, m->k, kvd, H);
        linear(m, w->tq, w->v, m->normed, m->v, kvd, H);
        if (w->qb) for (int i = 0; i < qd; ++i) m->q[i] += w->qb[i];
        if (w->kb) for (int i = 0; i < kvd; ++i) m->k[i] += w->kb[i];
        if (w->vb) for (int i = 0; i < kvd; ++i) m->v[i] += w->vb[i];
        if (w->qn && w->kn) {
            oracle_rms_norm_per_head(m->q, w->qn, nh, hd, m->eps);
            oracle_rms_norm_per_head(m->k, w->kn, nkv, hd, m->eps);
        }
        oracle_rope(m->q, m->k, hd, nh, nkv, pos, m->base);
        uint16_t* kc = m->kc + (size_t)l * m->max_ctx * kvd;
        uint16_t* vc = m->vc + (size_t)l * m->max_ctx * kvd;
        for (int i = 0; i < kvd; ++i) {
            kc[(size_t)pos * kvd + i] = m->kv_bf16 ? oracle_f2bf(m->k[i]) : oracle_f2h(m->k[i]);
            vc[(size_t)pos * kvd + i] = m->kv_bf16 ? oracle_f2bf(m->v[i]) : oracle_f2h(m->v[i]);
        }
        oracle_attention(m->att, m->q, kc, vc, m->kv_bf16, kvd, hd, hd, nh, nkv, pos + 1);
        linear(m, w->to, w->o, m->att, m->hidden, H, qd);
        for (int i = 0; i < H; ++i) m->hidden[i] += m->res[i];
        /* MLP block, qwen3.cu:317-341 */
        memcpy(m->res, m->hidden, (size_t)H * 4);
        oracle_rms_norm(m->normed, m->hidden, w->fn, H, m->eps);
        if (m->n_exp > 0) {
            moe_ffn(m, l);
            for (int i = 0; i < H; ++i) m->hidden[i] = m->res[i] + m->moe_out[i];
            continue;
        }
        linear(m, w->tg, w->g, m->normed, m->gate, F, H);
        linear(m, w->tg, w->u, m->normed, m->up, F, H);
        oracle_silu_mul(m->act, m->gate, m->up, F);
        linear(m, w->td, w->d, m->act, m->hidden, H, F);
        for (int i = 0; i < H; ++i) m->hidden[i] += m->res[i];
    }
    oracle_rms_norm(m->final_hidden, m->hidden, m->onorm, H, m->eps);
    /* tied LM head: token_embd (Q8_0), fp32 input, qwen3.cu:261 */
    oracle_gemv_q8_0(m->embd, m->final_hidden, m->ybuf, m->V, H, m->nthreads);
    for (int i = 0; i < m->V; ++i) logits[i] = (float)m->ybuf[i];
    return 0;
}

/* ---- sample_nucleus, src/model/qwen3.cu:351-460 (see the header) ---- */
typedef struct {
    float p;
    int i;
} oracle_pi;
static int oracle_pi_desc(const void* a, const void* b) {
    const oracle_pi* x = (const oracle_pi*)a;
    const oracle_pi* y = (const oracle_pi*)b;
    if (x->p != y->p) return x->p > y->p ? -1 : 1;
    return x->i < y->i ? -1 : (x->i > y->i);
}

int oracle_sample_nucleus(const float* logits, int vocab, const int* history, int n_history, float temperature,
                          float top_p, int top_k, float rep_penalty, float min_p, int dynamic_temp, double u,
                          double* cut_margin, double* u_margin) {
    float* l = (float*)malloc(sizeof(float) * (size_t)vocab);
    oracle_pi* probs = (oracle_pi*)malloc(sizeof(oracle_pi) * (size_t)vocab);
    memcpy(l, logits, sizeof(float) * (size_t)vocab);
    if (rep_penalty > 1.0f && n_history > 0) /* qwen3.cu:358-369: once per occurrence */
        for (int h = 0; h < n_history; ++h) {
            const int t = history[h];
            if (t >= 0 && t < vocab) l[t] = l[t] > 0 ? l[t] / rep_penalty : l[t] * rep_penalty;
        }
    float mx = -1e30f;
    for (int i = 0; i < vocab; ++i) mx = l[i] > mx ? l[i] : mx;
    if (min_p > 0.0f) { /* qwen3.cu:376-384 */
        const float thr = mx + logf(min_p);
        for (int i = 0; i < vocab; ++i)
            if (l[i] < thr) l[i] = -1e30f;
    }
    float temp = temperature;
    if (dynamic_temp) { /* qwen3.cu:388-412 */
        float dyn = 0.0f;
        for (int i = 0; i < vocab; ++i)
            if (l[i] > -1e20f) dyn += expf(l[i] - mx);
        float ent = 0.0f;
        for (int i = 0; i < vocab; ++i)
            if (l[i] > -1e20f) {
                const float pr = expf(l[i] - mx) / dyn;
                if (pr > 1e-6f) ent -= pr * logf(pr);
            }
        float sc = ent / 2.0f;
        sc = sc < 0.5f ? 0.5f : (sc > 2.0f ? 2.0f : sc);
        temp *= sc;
    }
    float sum = 0.0f; /* qwen3.cu:414-426 */
    for (int i = 0; i < vocab; ++i) {
        if (l[i] < -1e20f) {
            l[i] = 0.0f;
            continue;
        }
        l[i] = expf((l[i] - mx) / temp);
        sum += l[i];
    }
    for (int i = 0; i < vocab; ++i) {
        probs[i].p = l[i] / sum;
        probs[i].i = i;
    }
    qsort(probs, (size_t)vocab, sizeof(oracle_pi), oracle_pi_desc); /* qwen3.cu:428-436, ties: smaller id */
    const int limit = top_k < vocab ? top_k : vocab;                  /* qwen3.cu:438-448 */
    float cum = 0.0f;
    int k = limit;
    double cm = 1e30;
    for (int i = 0; i < limit; ++i) {
        cum += probs[i].p;
        const double d = fabs((double)cum - (double)top_p);
        if (d < cm) cm = d;
        if (cum >= top_p) {
            k = i + 1;
            break;
        }
    }
    double w = 0.0, acc = 0.0, um = 1e30;
    for (int i = 0; i < k; ++i) w += probs[i].p;
    int pick = k - 1;
    for (int i = 0; i < k; ++i) { /* qwen3.cu:450-456: std::discrete_distribution (libstdc++: cumulative of the
                                     normalised weights in double, last set to 1, first >= u) */
        acc += probs[i].p / w;
        const double c = i == k - 1 ? 1.0 : acc;
        if (i < k - 1 && fabs(c - u) < um) um = fabs(c - u);
        if (i < k - 1 && c >= u) {
            pick = i;
            break;
        }
    }
    const int id = probs[pick].i;
    if (cut_margin) *cut_margin = cm;
    if (u_margin) *u_margin = um;
    free(l);
    free(probs);
    return id;
}
