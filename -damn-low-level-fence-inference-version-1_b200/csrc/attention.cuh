// attention.cuh — single-query grouped-query attention over a KV cache, split over the context
// (flash-decode), for sm_100a.
//
// Reference semantics (src/kernels/ops.cuh:320-403): for query head qh with kv head
// qh / (Hq/Hkv): s_t = (q . k_t) * head_dim^-1/2 for t < seq_len; p = softmax(s); out = sum_t p_t v_t,
// all in fp32 over an fp16 cache. The reference runs one CTA per query head over the whole
// context with thread-per-position dot products and re-reads every K/V row once per query head.
//
// Here one CTA handles one KV head and one chunk of positions for ALL query heads of its group,
// so every K/V byte is read from HBM once per token. Each CTA writes the chunk's running max,
// exp-sum and unnormalised output; chunks are merged in a fixed order (deterministic).
//  * K/V rows are staged in shared memory with 16-byte cp.async copies whose chunk index is XORed
//    with (row & 7), which makes the thread-per-position reads of K conflict-free.
//  * Fused engine mode additionally: applies q/k RMSNorm (ops.cuh:66-95) and NeoX RoPE
//    (ops.cuh:115-167) to the raw QKV-GEMV output, writes the new K/V row of position `pos` into the
//    cache (ops.cuh:419-433) — the CTA owning that position uses the rounded values itself — and
//    the last CTA of each KV head merges the chunks (arrival counter), so attention is one launch.
//    The chunk length adapts to the context so short contexts still spread over many SMs.
//  * KV element type: fp16 (reference numerics) or bf16.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace fence {

constexpr int ATTN_THREADS = 256;
constexpr int ATTN_CMAX = 64;   // positions per shared-memory tile (one fused-mode chunk)
constexpr int ATTN_MAX_G = 8;   // query heads per KV head supported
constexpr int ATTN_TPP = 4;     // threads per position in the score pass (each owns a quarter of head_dim)

template <typename T>
struct KVConv;
template <>
struct KVConv<__half> {
    static __device__ __forceinline__ __half from(float f) { return __float2half_rn(f); }
    static __device__ __forceinline__ float to(__half h) { return __half2float(h); }
    static __device__ __forceinline__ float2 pair(uint32_t w) {
        return __half22float2(*reinterpret_cast<const __half2*>(&w));
    }
};
template <>
struct KVConv<__nv_bfloat16> {
    static __device__ __forceinline__ __nv_bfloat16 from(float f) { return __float2bfloat16_rn(f); }
    static __device__ __forceinline__ float to(__nv_bfloat16 h) { return __bfloat162float(h); }
    static __device__ __forceinline__ float2 pair(uint32_t w) {
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
};

struct AttnArgs {
    const float* q;       // [Hq*HD]: final q (drop-in) or raw q from the QKV GEMV (fused)
    const void* kc;       // K cache base (element type KVT)
    const void* vc;
    long long stride_t;   // elements between positions
    long long stride_h;   // elements between KV heads
    int n_q_heads, n_kv_heads;
    int seq_len;          // drop-in: positions [0, seq_len)
    int nchunk;           // chunks per KV head in the grid (gridDim.x)
    int chunk_fixed;      // drop-in: positions per chunk; 0 = adaptive (fused)
    float* part;          // [Hkv][nchunk][G][HD+2] partials
    // fused mode
    const DecodeState* state;
    const float* k_new;   // raw k [Hkv*HD] of position pos
    const float* v_new;
    void* kc_w;           // writable cache bases (same as kc/vc)
    void* vc_w;
    const float* q_norm_w;  // [HD] or null
    const float* k_norm_w;
    float eps;
    const float2* rope;   // [max_ctx][HD/2] (cos, sin) table
    float* out;           // [Hq*HD] merged output (fp32)
    unsigned int* counter;  // [Hkv] arrival counters, zero between launches
};

// Fused-mode split of the context: chunks of 64 positions (one CTA each, a single shared-memory
// tile: the per-CTA work is a latency chain, so spreading the context over more CTAs is what
// shortens it), at most nchunk chunks (then longer ones), each a multiple of 16 positions. Up to
// 64 positions there is one chunk and no merge step.
constexpr int ATTN_CHUNK = 64;
__device__ __forceinline__ int attn_chunk_len(int seq_len, int nchunk) {
    int n = (seq_len + ATTN_CHUNK - 1) / ATTN_CHUNK;
    if (n > nchunk) n = nchunk;
    if (n < 1) n = 1;
    int c = (seq_len + n - 1) / n;
    c = (c + 15) & ~15;
    return c;
}

// RMSNorm of one head (HD values in smem row) by a warp, weight w[HD]; reference order w*x*rms.
template <int HD>
__device__ __forceinline__ void head_rmsnorm_warp(float* v, const float* w, float eps, int lane) {
    float ss = 0.f;
    for (int d = lane; d < HD; d += 32) ss += v[d] * v[d];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)HD + eps);
    __syncwarp();
    for (int d = lane; d < HD; d += 32) v[d] = w[d] * v[d] * r;
    __syncwarp();
}
// NeoX rotation of one head in smem with table row cs[HD/2].
template <int HD>
__device__ __forceinline__ void head_rope_warp(float* v, const float2* cs, int lane) {
    for (int i = lane; i < HD / 2; i += 32) {
        const float2 t = cs[i];
        const float a = v[i], b = v[i + HD / 2];
        v[i] = a * t.x - b * t.y;
        v[i + HD / 2] = a * t.y + b * t.x;
    }
    __syncwarp();
}

// One (KV head h, context chunk c) unit, run by threads 0 .. ATTN_THREADS-1 of the calling CTA,
// which synchronise on named barrier bar_id. STANDALONE: a kernel of its own (programmatic dependent
// launch around the loads that depend on the previous kernel); otherwise a phase of the persistent
// step kernel, whose grid barrier already orders it after the QKV phase.
template <typename KVT, int HD, bool FUSED, bool STANDALONE>
__device__ __forceinline__ void attn_chunk(const AttnArgs& a, int h, int c, uint8_t* sm, int bar_id,
                                           int known_pos = -1) {
    using C = KVConv<KVT>;
    constexpr int CH = HD * (int)sizeof(KVT) / 16;  // 16-byte chunks per row
    constexpr int EPC = 16 / (int)sizeof(KVT);      // elements per chunk
    constexpr int CPQ = CH / ATTN_TPP;              // chunks per quarter
    constexpr int KP = (ATTN_MAX_G * HD / 2 + ATTN_THREADS - 1) / ATTN_THREADS;  // PV pairs per thread
    constexpr int NW = ATTN_THREADS / 32;
    static_assert(CH >= 8 && CH % ATTN_TPP == 0, "head_dim too small for the swizzle");
    KVT* sk = reinterpret_cast<KVT*>(sm);
    KVT* sv = sk + ATTN_CMAX * HD;
    float* sq = reinterpret_cast<float*>(sv + ATTN_CMAX * HD);  // [G][HD]
    float* ss = sq + ATTN_MAX_G * HD;                            // [G][CMAX]
    float* skn = ss + ATTN_MAX_G * ATTN_CMAX;                    // [HD] new k row (fused)
    float* sqw = skn + HD;                                       // [HD] q-norm weight
    float* skw = sqw + HD;                                       // [HD] k-norm weight
    float2* srope = reinterpret_cast<float2*>(skw + HD);         // [HD/2] cos/sin at pos
    float* smax = reinterpret_cast<float*>(srope + HD / 2);      // [G] running max
    float* ssum = smax + ATTN_MAX_G;                             // [G] running exp-sum
    float* sresc = ssum + ATTN_MAX_G;                            // [G] rescale of the old accumulator
    int* sflag = reinterpret_cast<int*>(sresc + ATTN_MAX_G);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.n_q_heads / a.n_kv_heads;
    int seq_len, pos, clen;
    if (FUSED) {
        // written by the previous token step, independent of this step's GEMVs (the step kernel
        // reads it once and passes it in)
        pos = known_pos >= 0 ? known_pos : a.state->pos;
        seq_len = pos + 1;
        clen = attn_chunk_len(seq_len, a.nchunk);
    } else {
        seq_len = a.seq_len;
        pos = seq_len - 1;
        clen = a.chunk_fixed;
    }
    const int n_active = (seq_len + clen - 1) / clen;
    if (c >= n_active) {
        if (STANDALONE && tid == 0) pdl_launch_dependents();
        return;
    }
    const int t0 = c * clen;
    const int t1 = min(t0 + clen, seq_len);
    const bool owns_new = FUSED && (pos >= t0 && pos < t1);

    const KVT* kb = reinterpret_cast<const KVT*>(a.kc) + (long long)h * a.stride_h;
    const KVT* vb = reinterpret_cast<const KVT*>(a.vc) + (long long)h * a.stride_h;
    auto stage_tile = [&](int ts, int te) {  // rows [ts, te) -> smem rows 0.., chunk XOR (row & 7)
        for (int idx = tid; idx < (te - ts) * CH; idx += ATTN_THREADS) {
            const int r = idx / CH, ch = idx - r * CH;
            const int t = ts + r;
            const int pch = ch ^ (r & 7);
            cp_async16(reinterpret_cast<uint8_t*>(sk + r * HD) + pch * 16,
                       reinterpret_cast<const uint8_t*>(kb + (long long)t * a.stride_t) + ch * 16);
            cp_async16(reinterpret_cast<uint8_t*>(sv + r * HD) + pch * 16,
                       reinterpret_cast<const uint8_t*>(vb + (long long)t * a.stride_t) + ch * 16);
        }
        cp_async_commit();
    };

    // ---- everything that does not depend on the preceding kernel, before the wait:
    //      cached K/V rows of the first tile, norm weights, the RoPE row of `pos`
    {
        const int te = min(t0 + ATTN_CMAX, t1);
        // in the tile that holds `pos`, row pos is produced below (the others are cached)
        stage_tile(t0, (owns_new && pos < te) ? pos : te);
    }
    if (FUSED) {
        for (int d = tid; d < HD; d += ATTN_THREADS) {
            sqw[d] = a.q_norm_w ? a.q_norm_w[d] : 1.f;
            skw[d] = a.k_norm_w ? a.k_norm_w[d] : 1.f;
        }
        for (int i = tid; i < HD / 2; i += ATTN_THREADS) srope[i] = a.rope[(long long)pos * (HD / 2) + i];
    }
    if (tid < ATTN_MAX_G) {
        smax[tid] = -INFINITY;
        ssum[tid] = 0.f;
    }
    if (STANDALONE) {
        if (tid == 0) pdl_launch_dependents();
        pdl_wait();
    }

    // ---- q of the G heads (and the new K/V row) from the QKV GEMV
    const int qh0 = h * G;
    for (int i = tid; i < G * HD; i += ATTN_THREADS) sq[i] = a.q[(long long)qh0 * HD + i];
    if (owns_new)
        for (int d = tid; d < HD; d += ATTN_THREADS) skn[d] = a.k_new[(long long)h * HD + d];
    named_bar_sync(bar_id, ATTN_THREADS);
    if (FUSED) {
        // q/k RMSNorm (w * x * rms) then NeoX rotation, warp per head; one more warp for the new k
        for (int g = warp; g < G + (owns_new ? 1 : 0); g += NW) {
            float* v = (g < G) ? sq + g * HD : skn;
            const bool norm = (g < G) ? (a.q_norm_w != nullptr) : (a.k_norm_w != nullptr);
            const float* w = (g < G) ? sqw : skw;
            if (norm) {
                float s2 = 0.f;
                for (int d = lane; d < HD; d += 32) s2 += v[d] * v[d];
                s2 = warp_sum(s2);
                const float r = rsqrtf(s2 / (float)HD + a.eps);
                for (int d = lane; d < HD; d += 32) v[d] = w[d] * v[d] * r;
                __syncwarp();
            }
            for (int i = lane; i < HD / 2; i += 32) {
                const float2 t = srope[i];
                const float x0 = v[i], x1 = v[i + HD / 2];
                v[i] = x0 * t.x - x1 * t.y;
                v[i + HD / 2] = x0 * t.y + x1 * t.x;
            }
            __syncwarp();
            if (g == G) {
                // round to the cache type, store the new row (global) and into its tile slot; the
                // new v values are loaded before any store (the stores could otherwise alias them
                // and serialise every load behind the previous store)
                const int r = pos - t0;
                KVT* kw = reinterpret_cast<KVT*>(a.kc_w) + (long long)h * a.stride_h + (long long)pos * a.stride_t;
                KVT* vw = reinterpret_cast<KVT*>(a.vc_w) + (long long)h * a.stride_h + (long long)pos * a.stride_t;
                float vn[HD / 32];
#pragma unroll
                for (int i = 0; i < HD / 32; ++i) vn[i] = a.v_new[(long long)h * HD + lane + 32 * i];
#pragma unroll
                for (int i = 0; i < HD / 32; ++i) {
                    const int d = lane + 32 * i;
                    const KVT kq = C::from(v[d]);
                    const KVT vq = C::from(vn[i]);
                    kw[d] = kq;
                    vw[d] = vq;
                    if (r < ATTN_CMAX) {  // in the first tile; a later tile re-reads the row from global
                        const int ch = d / EPC, within = d % EPC;
                        const int pch = ch ^ (r & 7);
                        reinterpret_cast<KVT*>(reinterpret_cast<uint8_t*>(sk + r * HD) + pch * 16)[within] = kq;
                        reinterpret_cast<KVT*>(reinterpret_cast<uint8_t*>(sv + r * HD) + pch * 16)[within] = vq;
                    }
                }
            }
        }
    }

    const float scale = 1.0f / sqrtf((float)HD);
    float o[KP][2];
#pragma unroll
    for (int k = 0; k < KP; ++k) o[k][0] = o[k][1] = 0.f;

    for (int ts = t0; ts < t1; ts += ATTN_CMAX) {
        const int te = min(ts + ATTN_CMAX, t1);
        const int nt = te - ts;
        if (ts != t0) stage_tile(ts, te);
        cp_async_wait_all();
        named_bar_sync(bar_id, ATTN_THREADS);

        // ---- scores: ATTN_TPP threads per position, each over CPQ chunks, then a shuffle sum
        for (int base = 0; base < nt; base += ATTN_THREADS / ATTN_TPP) {
            const int r = base + tid / ATTN_TPP;
            const int qtr = tid % ATTN_TPP;
            float acc[ATTN_MAX_G];
#pragma unroll
            for (int g = 0; g < ATTN_MAX_G; ++g) acc[g] = 0.f;
            if (r < nt) {
                const uint8_t* krow = reinterpret_cast<const uint8_t*>(sk + r * HD);
#pragma unroll
                for (int i = 0; i < CPQ; ++i) {
                    const int ch = qtr + ATTN_TPP * i;
                    const uint4 w = *reinterpret_cast<const uint4*>(krow + ((ch ^ (r & 7)) * 16));
                    float kf[8];
                    const float2 f0 = C::pair(w.x), f1 = C::pair(w.y), f2 = C::pair(w.z), f3 = C::pair(w.w);
                    kf[0] = f0.x; kf[1] = f0.y; kf[2] = f1.x; kf[3] = f1.y;
                    kf[4] = f2.x; kf[5] = f2.y; kf[6] = f3.x; kf[7] = f3.y;
#pragma unroll
                    for (int g = 0; g < ATTN_MAX_G; ++g) {
                        if (g >= G) break;  // uniform: no predicated work for absent heads
                        const float4 qa = *reinterpret_cast<const float4*>(sq + g * HD + ch * EPC);
                        const float4 qb = *reinterpret_cast<const float4*>(sq + g * HD + ch * EPC + 4);
                        acc[g] = fmaf(qa.x, kf[0], acc[g]);
                        acc[g] = fmaf(qa.y, kf[1], acc[g]);
                        acc[g] = fmaf(qa.z, kf[2], acc[g]);
                        acc[g] = fmaf(qa.w, kf[3], acc[g]);
                        acc[g] = fmaf(qb.x, kf[4], acc[g]);
                        acc[g] = fmaf(qb.y, kf[5], acc[g]);
                        acc[g] = fmaf(qb.z, kf[6], acc[g]);
                        acc[g] = fmaf(qb.w, kf[7], acc[g]);
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < ATTN_MAX_G; ++g) {
                if (g >= G) break;
                acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
                acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 2);
            }
            if (r < nt && qtr == 0) {
#pragma unroll
                for (int g = 0; g < ATTN_MAX_G; ++g)
                    if (g < G) ss[g * ATTN_CMAX + r] = acc[g] * scale;
            }
        }
        named_bar_sync(bar_id, ATTN_THREADS);

        // ---- online softmax statistics per head (warp per head)
        for (int g = warp; g < G; g += NW) {
            float m = -INFINITY;
            for (int t = lane; t < nt; t += 32) m = fmaxf(m, ss[g * ATTN_CMAX + t]);
            m = warp_max(m);
            const float m_old = smax[g];
            const float m_new = fmaxf(m_old, m);
            float l = 0.f;
            for (int t = lane; t < nt; t += 32) {
                const float e = expf(ss[g * ATTN_CMAX + t] - m_new);
                ss[g * ATTN_CMAX + t] = e;
                l += e;
            }
            l = warp_sum(l);
            if (lane == 0) {
                const float f = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                sresc[g] = f;
                ssum[g] = ssum[g] * f + l;
                smax[g] = m_new;
            }
        }
        named_bar_sync(bar_id, ATTN_THREADS);

        // ---- P.V accumulate: thread <-> (head, dim pair)
#pragma unroll
        for (int k = 0; k < KP; ++k) {
            const int pidx = tid + k * ATTN_THREADS;
            if (pidx < G * (HD / 2)) {
                const int g = pidx / (HD / 2);
                const int d = 2 * (pidx - g * (HD / 2));
                const int ch = d / EPC, within = d % EPC;
                const float f = sresc[g];
                float o0 = o[k][0] * f, o1 = o[k][1] * f;
                const float* pg = ss + g * ATTN_CMAX;
                for (int r = 0; r < nt; ++r) {
                    const uint32_t w = *reinterpret_cast<const uint32_t*>(
                        reinterpret_cast<const uint8_t*>(sv + r * HD) + ((ch ^ (r & 7)) * 16) + within * sizeof(KVT));
                    const float2 vv = C::pair(w);
                    const float pr = pg[r];
                    o0 = fmaf(pr, vv.x, o0);
                    o1 = fmaf(pr, vv.y, o1);
                }
                o[k][0] = o0;
                o[k][1] = o1;
            }
        }
        named_bar_sync(bar_id, ATTN_THREADS);  // before the next tile overwrites sk/sv/ss
    }

    const int part_stride = HD + 2;
    if (n_active == 1) {
        // whole context in one chunk: normalise and write the output directly
#pragma unroll
        for (int k = 0; k < KP; ++k) {
            const int pidx = tid + k * ATTN_THREADS;
            if (pidx < G * (HD / 2)) {
                const int g = pidx / (HD / 2);
                const int d = 2 * (pidx - g * (HD / 2));
                const float inv = 1.0f / ssum[g];
                a.out[(long long)(qh0 + g) * HD + d] = o[k][0] * inv;
                a.out[(long long)(qh0 + g) * HD + d + 1] = o[k][1] * inv;
            }
        }
        return;
    }

    float* pbase = a.part + (((long long)h * a.nchunk + c) * G) * part_stride;
#pragma unroll
    for (int k = 0; k < KP; ++k) {
        const int pidx = tid + k * ATTN_THREADS;
        if (pidx < G * (HD / 2)) {
            const int g = pidx / (HD / 2);
            const int d = 2 * (pidx - g * (HD / 2));
            pbase[g * part_stride + d] = o[k][0];
            pbase[g * part_stride + d + 1] = o[k][1];
        }
    }
    if (tid < G) {
        pbase[tid * part_stride + HD] = smax[tid];
        pbase[tid * part_stride + HD + 1] = ssum[tid];
    }

    if (FUSED) {
        // ---- last CTA of this KV head merges all chunks
        __threadfence();
        named_bar_sync(bar_id, ATTN_THREADS);
        if (tid == 0) {
            const unsigned prev = atomicAdd(&a.counter[h], 1u);
            *sflag = (prev == (unsigned)n_active - 1) ? 1 : 0;
        }
        named_bar_sync(bar_id, ATTN_THREADS);
        if (*sflag) {
            __threadfence();
            // merge in two steps: (1) the chunks' max / exp-sum per head -> per-chunk scale factors
            // in shared memory (reusing the score buffer), (2) each output element adds its chunks'
            // partial outputs in chunk order (independent loads, deterministic). The partials are
            // read from L2: other CTAs wrote them before their counter increment.
            const float* hb = a.part + ((long long)h * a.nchunk * G) * part_stride;
            // the K tile and q are no longer needed: [G][n_active] chunk max (then scale factor) and
            // [G] 1/L in the K tile (>= 4096 floats), [G][n_active] exp-sums in q (1024 floats)
            float* fsc = reinterpret_cast<float*>(sk);
            float* fls = sq;
            for (int i = tid; i < G * n_active; i += ATTN_THREADS) {
                const int g = i / n_active, cc = i - g * n_active;
                const float* pr = hb + ((long long)cc * G + g) * part_stride;
                fsc[i] = __ldcg(pr + HD);
                fls[i] = __ldcg(pr + HD + 1);
            }
            named_bar_sync(bar_id, ATTN_THREADS);
            if (tid < G) {
                const int g = tid;
                float M = -INFINITY;
                for (int cc = 0; cc < n_active; ++cc) M = fmaxf(M, fsc[g * n_active + cc]);
                float L = 0.f;
                for (int cc = 0; cc < n_active; ++cc) {
                    const float f = expf(fsc[g * n_active + cc] - M);
                    L += fls[g * n_active + cc] * f;
                    fsc[g * n_active + cc] = f;
                }
                fsc[G * n_active + g] = 1.0f / L;
            }
            named_bar_sync(bar_id, ATTN_THREADS);
            for (int pidx = tid; pidx < G * HD; pidx += ATTN_THREADS) {
                const int g = pidx / HD, d = pidx - g * HD;
                float O = 0.f;
#pragma unroll 8
                for (int cc = 0; cc < n_active; ++cc)
                    O += __ldcg(hb + ((long long)cc * G + g) * part_stride + d) * fsc[g * n_active + cc];
                a.out[(long long)(qh0 + g) * HD + d] = O * fsc[G * n_active + g];
            }
            if (tid == 0) a.counter[h] = 0u;
        }
    }
}

template <typename KVT, int HD, bool FUSED>
__global__ void __launch_bounds__(ATTN_THREADS) attn_partial_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    attn_chunk<KVT, HD, FUSED, true>(a, blockIdx.y, blockIdx.x, sm, 0);
}

// Drop-in merge: one CTA per query head, thread per dimension.
template <int HD>
__global__ void attn_merge_kernel(const float* __restrict__ part, float* __restrict__ out, int n_q_heads,
                                  int n_kv_heads, int nchunk, int n_active) {
    const int qh = blockIdx.x;
    const int G = n_q_heads / n_kv_heads;
    const int h = qh / G, g = qh - h * G;
    const int part_stride = HD + 2;
    const float* hb = part + ((long long)h * nchunk * G) * part_stride;
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        float M = -INFINITY;
        for (int cc = 0; cc < n_active; ++cc) M = fmaxf(M, hb[((long long)cc * G + g) * part_stride + HD]);
        float L = 0.f, O = 0.f;
        for (int cc = 0; cc < n_active; ++cc) {
            const float* pr = hb + ((long long)cc * G + g) * part_stride;
            const float f = expf(pr[HD] - M);
            L += pr[HD + 1] * f;
            O += pr[d] * f;
        }
        out[(long long)qh * HD + d] = O / L;
    }
}

template <typename KVT, int HD>
constexpr int attn_smem_bytes() {
    return 2 * ATTN_CMAX * HD * (int)sizeof(KVT) + ATTN_MAX_G * HD * 4 + ATTN_MAX_G * ATTN_CMAX * 4 + 3 * HD * 4 +
           (HD / 2) * 8 + (3 * ATTN_MAX_G + 8) * 4;
}

}  // namespace fence
