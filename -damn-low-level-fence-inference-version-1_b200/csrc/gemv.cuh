// gemv.cuh — HBM-streaming dequant-GEMV for batch-1 decode on B200 (sm_100a).
//
// Computes y[row] = sum_k W[row][k] * x[k] for Q6_K (src/kernels/gemv_q6k.cuh:45-83 in the
// reference) and Q8_0 (src/kernels/gemv_q8_0.cuh:75-97) weights in their raw GGUF layouts, with
// the producer/consumer work that surrounds the GEMV in the token loop fused in:
//
//   prologue  x from fp16 / fp32 global memory, optionally RMSNorm'd (ops.cuh:17-45) and rounded to
//             fp16 (the reference's f32_to_f16 before every Q6_K GEMV, qwen3.cu:278,310,325,336)
//   epilogue  plain store (+bias), residual add (ops.cuh:256-263), SwiGLU of a gate/up row pair
//             (ops.cuh:183-195) written as the next GEMV's input, or LM-head logits + greedy argmax
//             (ops.cuh:467-499) with the decode state advanced on the device.
//
// Design (B200-first; the reference is one warp per row with byte loads):
//  * The weight bytes a CTA owns are streamed through a ring of shared-memory stages by one
//    producer thread issuing 1-D TMA bulk copies (cp.async.bulk, no multicast) that complete on
//    mbarriers, so tens of KB per SM are in flight with almost no issue cost. Stage boundaries are
//    rounded to 16 B in global memory; the sub-16 B tail of a tensor is fetched with plain loads.
//  * Each consumer thread owns one fixed 64-element "item" of the K dimension for every row it
//    touches: for Q6_K the elements {h*128 + c*32 + l16*16 + j | c<4, j<16} of one super-block
//    (h, l16 in {0,1}), so each of its four 16-element sub-blocks is complete inside the thread and
//    its scale is applied once; for Q8_0 two consecutive 32-element blocks.
//  * x is quantised per item to 16-bit integers split into a signed high byte and an unsigned low
//    byte, so the 6-bit (or 8-bit) weights are dotted with dp4a in exact integer arithmetic:
//    sum (q-32)*xq = 256*dp4a(q, xh) + dp4a(q, xl) - 32*sum(xq). The only rounding is xq itself
//    (|err| <= max|x_item| / 65534 per element), well inside the 1e-3 relative bound the reference
//    GEMV test applies (tests/test_gemv_q6k.cu:134-164).
//  * The 6-bit unpack is four 3-input logic ops per 16 weights on whole 32-bit words.
//  * Row sums are reduced through shared memory (double-buffered, one named barrier per stage) in
//    a fixed order, so results are deterministic.
//  * Programmatic dependent launch: the producer starts streaming weights before
//    griddepcontrol.wait; only the x prologue waits for the previous kernel.
#pragma once

#include "common.cuh"

namespace fence {

enum : int { WT_Q6K = 0, WT_Q80 = 1 };
enum : int { X_F16 = 0, X_F32 = 1, X_F32_R16 = 2, X_NORM = 3, X_NORM_R16 = 4 };
enum : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_LMHEAD = 3 };

constexpr int GEMV_NW = 8;                        // consumer warps per CTA
constexpr int GEMV_MAX_NT = GEMV_NW * 32 + 32;    // + one producer warp; two CTAs fit on an SM
constexpr int GEMV_MAX_SEG = 3;
constexpr int GEMV_STAGE_SLACK = 256;  // per-stage bytes: <= 3 pieces x (30 B alignment + 31 B padding) + over-read

struct GemvSeg {
    const uint8_t* W;   // tensor base, 16-byte aligned
    int rows;           // rows of this tensor covered by the launch
    float* y;           // EPI_STORE output, indexed by the tensor's row
    const float* bias;  // optional bias for EPI_STORE
};

// Device-resident decode state advanced by the LM head (token fed to the next step, its position).
struct DecodeState {
    int token;
    int pos;
    int step;
    int err;  // the device error word as the step that wrote token saw it at its end (0 = ok)
};

struct GemvArgs {
    GemvSeg seg[GEMV_MAX_SEG];
    int nseg;
    int dual;         // EPI_SWIGLU: seg[0] = gate, seg[1] = up, same rows
    int Mv;           // virtual rows (dual: rows of each tensor)
    int K;
    int rowB;         // bytes per row
    int I;            // items (64 elements) per row
    int S;            // virtual rows per stage (dual: gate/up pairs)
    int lpr;          // lanes per row: a warp works on 32/lpr row groups at once
    int ring;         // stages in the shared-memory ring
    int stage_bytes;  // bytes per ring slot (multiple of 128)
    // x source
    const void* x;
    const float* norm_w;
    float eps;
    // epilogue targets
    float* resid;      // EPI_RESID: resid[row] = dot + resid[row]
    void* act;         // EPI_SWIGLU output (fp16 when act_f16, else fp32)
    int act_f16;
    float* logits;     // EPI_LMHEAD
    float* cta_val;    // [gridDim.x] per-CTA best logit
    int* cta_idx;      // [gridDim.x] per-CTA best index
    unsigned int* counter;  // CTA arrival counter, zero between launches
    DecodeState* state;     // EPI_LMHEAD: token/pos/step advanced by the last CTA
    int* token_log;         // EPI_LMHEAD: token_log[step] = sampled id (may be null)
    int token_log_cap;
};

template <int WT>
struct WTraits;
template <>
struct WTraits<WT_Q6K> {
    static constexpr int BLOCK_ELEMS = 256;
    static constexpr int BLOCK_BYTES = 210;
    static constexpr int XWORDS = 16;  // xh / xl words per item
};
template <>
struct WTraits<WT_Q80> {
    static constexpr int BLOCK_ELEMS = 32;
    static constexpr int BLOCK_BYTES = 34;
    static constexpr int XWORDS = 17;  // 9 (block 0, shifted by the 2-byte scale) + 8 (block 1)
};

// --------------------------------------------------------------------------------------------
// Stage geometry: a stage covers `n` consecutive virtual rows starting at va, split into at most
// three contiguous pieces of global memory (one per tensor touched). All indexing is static so the
// pieces stay in registers.
struct Piece {
    const uint8_t* src;   // 16-byte aligned start of the bulk copy
    uint32_t copy_bytes;  // multiple of 16
    uint32_t tail_bytes;  // bytes after the bulk part fetched with plain loads (tensor end only)
    uint32_t smem_off;    // offset of the copy inside the stage slot
    uint32_t delta;       // offset of the first row inside the copy
    int first_row;        // first stage-row index in this piece
    int seg_row0;         // first tensor row
    int valid;
};

struct StageGeo {
    Piece p[GEMV_MAX_SEG];
};

__device__ __forceinline__ void make_piece(const GemvArgs& a, int s, int r0, int nr, int first, Piece& p) {
    const uint64_t total = (uint64_t)a.seg[s].rows * (uint64_t)a.rowB;
    const uint64_t g0 = (uint64_t)r0 * a.rowB;
    const uint64_t g1 = (uint64_t)(r0 + nr) * a.rowB;
    const uint64_t a0 = g0 & ~uint64_t(15);
    uint64_t end;
    uint32_t tail = 0;
    if (g1 >= total) {
        end = total & ~uint64_t(15);
        tail = (uint32_t)(total - end);
    } else {
        end = (g1 + 15) & ~uint64_t(15);
    }
    p.src = a.seg[s].W + a0;
    p.copy_bytes = (uint32_t)(end - a0);
    p.tail_bytes = tail;
    p.delta = (uint32_t)(g0 - a0);
    p.first_row = first;
    p.seg_row0 = r0;
    p.valid = 1;
}

__device__ __forceinline__ void stage_geo(const GemvArgs& a, int va, int n, StageGeo& g) {
#pragma unroll
    for (int k = 0; k < GEMV_MAX_SEG; ++k) g.p[k].valid = 0;
    if (a.dual) {
        make_piece(a, 0, va, n, 0, g.p[0]);
        make_piece(a, 1, va, n, n, g.p[1]);
    } else {
        int base = 0;
#pragma unroll
        for (int s = 0; s < GEMV_MAX_SEG; ++s) {
            if (s < a.nseg) {
                const int rs = a.seg[s].rows;
                const int lo = max(va, base), hi = min(va + n, base + rs);
                if (lo < hi) make_piece(a, s, lo - base, hi - lo, lo - va, g.p[s]);
                base += rs;
            }
        }
    }
    uint32_t off = 0;
#pragma unroll
    for (int k = 0; k < GEMV_MAX_SEG; ++k) {
        g.p[k].smem_off = off;
        if (g.p[k].valid) off = (off + g.p[k].copy_bytes + g.p[k].tail_bytes + 16u + 15u) & ~15u;
    }
}

// Piece index holding stage row r (pieces are ordered by first_row).
__device__ __forceinline__ int piece_of(const StageGeo& g, int r) {
    int k = 0;
#pragma unroll
    for (int j = 1; j < GEMV_MAX_SEG; ++j)
        if (g.p[j].valid && r >= g.p[j].first_row) k = j;
    return k;
}

// --------------------------------------------------------------------------------------------
// Per-thread quantised activation slice.
template <int WT>
struct XSlice {
    uint32_t xh[WTraits<WT>::XWORDS];
    uint32_t xl[WTraits<WT>::XWORDS];
    int corr[4];  // Q6_K: -32 * sum(xq) per column run
    float xs0, xs1;
};

__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// Quantise n floats (max |v| = amax) into xq (int), returns scale.
__device__ __forceinline__ float quant_scale(float amax, float& inv) {
    if (!isfinite(amax)) {  // propagate NaN/Inf like the reference's fp32 sums would
        inv = 0.f;
        return __int_as_float(0x7fc00000);
    }
    if (!(amax > 0.f)) {
        inv = 0.f;
        return 0.f;
    }
    inv = 32767.f / amax;
    return amax / 32767.f;
}
__device__ __forceinline__ void split16(int q, uint32_t& hb, uint32_t& lb) {
    hb = (uint32_t)((q >> 8) & 0xff);  // signed high byte (two's complement)
    lb = (uint32_t)(q & 0xff);          // unsigned low byte
}

// Loads the 64 x values of an item in the order the weight words deliver them.
//   Q6_K item (b, h, l16): v[c*16 + j] = x[b*256 + h*128 + c*32 + l16*16 + j]
//   Q8_0 item i:          v[e] = x[i*64 + e]
template <int WT, int XM>
__device__ __forceinline__ void load_item_x(const GemvArgs& a, int item, float v[64]) {
    int base[4];
    if (WT == WT_Q6K) {
        const int b = item >> 2, h = (item >> 1) & 1, l16 = item & 1;
#pragma unroll
        for (int c = 0; c < 4; ++c) base[c] = b * 256 + h * 128 + c * 32 + l16 * 16;
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) base[c] = item * 64 + c * 16;
    }
    if (XM == X_F16) {
        const uint16_t* x = static_cast<const uint16_t*>(a.x);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4* p = reinterpret_cast<const uint4*>(x + base[c]);
            const uint4 u0 = p[0], u1 = p[1];
            const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                v[c * 16 + 2 * k] = half_bits_to_float(w[k]);
                v[c * 16 + 2 * k + 1] = half_bits_to_float(w[k] >> 16);
            }
        }
    } else {
        const float* x = static_cast<const float*>(a.x);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float4* p = reinterpret_cast<const float4*>(x + base[c]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 f = p[k];
                v[c * 16 + 4 * k + 0] = f.x;
                v[c * 16 + 4 * k + 1] = f.y;
                v[c * 16 + 4 * k + 2] = f.z;
                v[c * 16 + 4 * k + 3] = f.w;
            }
        }
    }
    if (XM == X_NORM || XM == X_NORM_R16) {
        // w[i] * x[i] * rms in the reference's operation order (ops.cuh:43)
        const float* w = a.norm_w;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float4* p = reinterpret_cast<const float4*>(w + base[c]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 f = p[k];
                v[c * 16 + 4 * k + 0] *= f.x;
                v[c * 16 + 4 * k + 1] *= f.y;
                v[c * 16 + 4 * k + 2] *= f.z;
                v[c * 16 + 4 * k + 3] *= f.w;
            }
        }
    }
}

template <int WT, int XM>
__device__ __forceinline__ void make_slice(const GemvArgs& a, int item, float rms, XSlice<WT>& s) {
    float v[64];
    load_item_x<WT, XM>(a, item, v);
    if (XM == X_NORM || XM == X_NORM_R16) {
#pragma unroll
        for (int e = 0; e < 64; ++e) v[e] = v[e] * rms;
    }
    if (XM == X_F32_R16 || XM == X_NORM_R16) {
#pragma unroll
        for (int e = 0; e < 64; ++e) v[e] = round_f16(v[e]);
    }
    if (WT == WT_Q6K) {
        float amax = 0.f;
#pragma unroll
        for (int e = 0; e < 64; ++e) amax = fmaxf(amax, fabsf(v[e]));
        float inv;
        s.xs0 = quant_scale(amax, inv);
        s.xs1 = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            int sum = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t hw = 0, lw = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int q = __float2int_rn(v[c * 16 + 4 * k + j] * inv);
                    sum += q;
                    uint32_t hb, lb;
                    split16(q, hb, lb);
                    hw |= hb << (8 * j);
                    lw |= lb << (8 * j);
                }
                s.xh[c * 4 + k] = hw;
                s.xl[c * 4 + k] = lw;
            }
            s.corr[c] = -32 * sum;
        }
    } else {
        // two 32-element blocks with separate scales; block 0's words are shifted by the 2-byte
        // scale that precedes its quants: word m, byte n <-> element 4m + n - 2.
        float am0 = 0.f, am1 = 0.f;
#pragma unroll
        for (int e = 0; e < 32; ++e) am0 = fmaxf(am0, fabsf(v[e]));
#pragma unroll
        for (int e = 32; e < 64; ++e) am1 = fmaxf(am1, fabsf(v[e]));
        float inv0, inv1;
        s.xs0 = quant_scale(am0, inv0);
        s.xs1 = quant_scale(am1, inv1);
#pragma unroll
        for (int m = 0; m < 9; ++m) {
            uint32_t hw = 0, lw = 0;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                const int e = 4 * m + n - 2;
                if (e >= 0 && e < 32) {
                    const int q = __float2int_rn(v[e] * inv0);
                    uint32_t hb, lb;
                    split16(q, hb, lb);
                    hw |= hb << (8 * n);
                    lw |= lb << (8 * n);
                }
            }
            s.xh[m] = hw;
            s.xl[m] = lw;
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            uint32_t hw = 0, lw = 0;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                const int q = __float2int_rn(v[32 + 4 * m + n] * inv1);
                uint32_t hb, lb;
                split16(q, hb, lb);
                hw |= hb << (8 * n);
                lw |= lb << (8 * n);
            }
            s.xh[9 + m] = hw;
            s.xl[9 + m] = lw;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) s.corr[c] = 0;
    }
}

// Partial dot of one item of one row. `sb` is the 32-bit shared address of the item's super-block
// (Q6_K) or of the item's first block (Q8_0); 2-byte aligned (Q6_K) / 4-byte aligned (Q8_0).
template <int WT>
__device__ __forceinline__ float item_dot(uint32_t sb, int item, const XSlice<WT>& s) {
    if (WT == WT_Q6K) {
        const int h = (item >> 1) & 1, l16 = item & 1;
        uint32_t ql0[4], ql1[4], qh[4];
        lds_16B_a2(sb + h * 64 + l16 * 16, ql0);
        lds_16B_a2(sb + h * 64 + 32 + l16 * 16, ql1);
        lds_16B_a2(sb + 128 + h * 32 + l16 * 16, qh);
        const uint32_t sA = lds_u32_a2(sb + 192 + 8 * h);
        const uint32_t sB = lds_u32_a2(sb + 196 + 8 * h);
        const uint32_t dbits = lds_u16(sb + 208);
        int hi0 = 0, hi1 = 0, hi2 = 0, hi3 = 0;
        int lo0 = s.corr[0], lo1 = s.corr[1], lo2 = s.corr[2], lo3 = s.corr[3];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t qm = qh[k] & 0x33333333u;  // crumbs 0 (bits 0-1) and 2 (bits 4-5)
            const uint32_t qn = qh[k] & 0xCCCCCCCCu;  // crumbs 1 (bits 2-3) and 3 (bits 6-7)
            const uint32_t q0 = (ql0[k] & 0x0F0F0F0Fu) | ((qm << 4) & 0xF0F0F0F0u);
            const uint32_t q1 = (ql1[k] & 0x0F0F0F0Fu) | ((qn << 2) & 0xF0F0F0F0u);
            const uint32_t q2 = ((ql0[k] >> 4) & 0x0F0F0F0Fu) | (qm & 0xF0F0F0F0u);
            const uint32_t q3 = ((ql1[k] >> 4) & 0x0F0F0F0Fu) | ((qn >> 2) & 0xF0F0F0F0u);
            hi0 = dp4a_us(q0, s.xh[0 * 4 + k], hi0);
            lo0 = dp4a_uu(q0, s.xl[0 * 4 + k], lo0);
            hi1 = dp4a_us(q1, s.xh[1 * 4 + k], hi1);
            lo1 = dp4a_uu(q1, s.xl[1 * 4 + k], lo1);
            hi2 = dp4a_us(q2, s.xh[2 * 4 + k], hi2);
            lo2 = dp4a_uu(q2, s.xl[2 * 4 + k], lo2);
            hi3 = dp4a_us(q3, s.xh[3 * 4 + k], hi3);
            lo3 = dp4a_uu(q3, s.xl[3 * 4 + k], lo3);
        }
        // sub-block scales: column c uses scales[8h + l16 + 2c]
        const int sc0 = (int)(sA << (24 - 8 * l16)) >> 24;
        const int sc1 = (int)(sA << (8 - 8 * l16)) >> 24;
        const int sc2 = (int)(sB << (24 - 8 * l16)) >> 24;
        const int sc3 = (int)(sB << (8 - 8 * l16)) >> 24;
        const float t = (float)((hi0 * 256 + lo0) * sc0) + (float)((hi1 * 256 + lo1) * sc1) +
                        (float)((hi2 * 256 + lo2) * sc2) + (float)((hi3 * 256 + lo3) * sc3);
        return t * (half_bits_to_float(dbits) * s.xs0);
    } else {
        // 68 bytes = 17 words, 4-byte aligned (rows are 4-byte aligned when K % 64 == 0)
        int hi0 = 0, lo0 = 0, hi1 = 0, lo1 = 0;
        uint32_t w0 = 0, w8 = 0;
#pragma unroll
        for (int m = 0; m < 9; ++m) {
            const uint32_t q = lds32(sb + 4 * m);
            if (m == 0) w0 = q;
            if (m == 8) w8 = q;
            hi0 = dp4a_ss(q, s.xh[m], hi0);
            lo0 = dp4a_su(q, s.xl[m], lo0);
        }
#pragma unroll
        for (int m = 9; m < 17; ++m) {
            const uint32_t q = lds32(sb + 4 * m);
            hi1 = dp4a_ss(q, s.xh[m], hi1);
            lo1 = dp4a_su(q, s.xl[m], lo1);
        }
        const float d0 = half_bits_to_float(w0);
        const float d1 = half_bits_to_float(w8 >> 16);
        return (float)(hi0 * 256 + lo0) * (d0 * s.xs0) + (float)(hi1 * 256 + lo1) * (d1 * s.xs1);
    }
}

// Reference argmax order (ops.cuh:467-499): thread t of 256 keeps the first strict maximum of
// x[t], x[t+256], ...; the tree step `if (s[t+s] > s[t])` keeps position t on ties, so two tied
// threads meet at their lowest differing index bit and the one with a 0 there wins — i.e. the
// smaller 8-bit-reversed thread index. NaN and values <= -1e30 never win.
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
    if (!(v > -1e30f)) return false;
    if (bi < 0) return true;
    if (v > bv) return true;
    if (v < bv) return false;
    const unsigned ki = __brev((unsigned)(i & 255)) >> 24, kb = __brev((unsigned)(bi & 255)) >> 24;
    return ki < kb || (ki == kb && i < bi);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// --------------------------------------------------------------------------------------------
// Quantised-x record of one item in shared memory: xh[XW] | xl[XW] | corr[4] | xs0 | xs1 (40 words).
constexpr int XQ_WORDS = 40;

template <int WT>
__device__ __forceinline__ void store_slice(uint32_t rec, const XSlice<WT>& s) {
    constexpr int XW = WTraits<WT>::XWORDS;
    uint32_t w[XQ_WORDS];
#pragma unroll
    for (int k = 0; k < XW; ++k) {
        w[k] = s.xh[k];
        w[XW + k] = s.xl[k];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) w[2 * XW + k] = (uint32_t)s.corr[k];
    w[2 * XW + 4] = __float_as_uint(s.xs0);
    w[2 * XW + 5] = __float_as_uint(s.xs1);
#pragma unroll
    for (int k = 2 * XW + 6; k < XQ_WORDS; ++k) w[k] = 0u;
#pragma unroll
    for (int k = 0; k < XQ_WORDS / 4; ++k)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rec + 16 * k), "r"(w[4 * k]),
                     "r"(w[4 * k + 1]), "r"(w[4 * k + 2]), "r"(w[4 * k + 3])
                     : "memory");
}

template <int WT>
__device__ __forceinline__ void load_slice(uint32_t rec, XSlice<WT>& s) {
    constexpr int XW = WTraits<WT>::XWORDS;
    uint32_t w[XQ_WORDS];
#pragma unroll
    for (int k = 0; k < XQ_WORDS / 4; ++k) {
        const uint4 u = lds128(rec + 16 * k);
        w[4 * k] = u.x;
        w[4 * k + 1] = u.y;
        w[4 * k + 2] = u.z;
        w[4 * k + 3] = u.w;
    }
#pragma unroll
    for (int k = 0; k < XW; ++k) {
        s.xh[k] = w[k];
        s.xl[k] = w[XW + k];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) s.corr[k] = (int)w[2 * XW + k];
    s.xs0 = __uint_as_float(w[2 * XW + 4]);
    s.xs1 = __uint_as_float(w[2 * XW + 5]);
}

// Shared-memory carve-up (all regions 16-byte aligned); the host plan uses the same function.
// SR = rows per stage slot (dual: 2 x pairs).
struct GemvSmem {
    uint32_t xq, rowtab, rowinfo, bars, misc, total;
};
__host__ __device__ inline GemvSmem gemv_smem_layout(int ring, int stage_bytes, int SR, int I) {
    auto r16 = [](uint32_t x) { return (x + 15u) & ~15u; };
    GemvSmem L;
    L.xq = (uint32_t)ring * (uint32_t)stage_bytes;
    L.rowtab = L.xq + (uint32_t)I * XQ_WORDS * 4u;
    L.rowinfo = L.rowtab + r16(4u * ring * SR);
    L.bars = L.rowinfo + r16(4u * ring * SR);
    L.misc = L.bars + r16(16u * ring);
    L.total = L.misc + 512u;
    return L;
}

// Rows (dual: pairs) each lane group takes per batch: two independent rows share one x load;
// in dual mode the gate and up rows of a pair already share it.
__host__ __device__ inline int gemv_rows_per_group(int dual) { return dual ? 1 : 2; }

// One warp-autonomous streaming GEMV. Per CTA: one producer warp streams the CTA's contiguous rows
// through a ring of shared-memory stages (1-D TMA bulk copies on mbarriers); GEMV_NW consumer
// warps each take whole batches of rows (lane group of `lpr` lanes per row, each lane a strided
// subset of the row's 64-element items, shuffle reduction inside the group) and release every
// stage independently — no CTA-wide barrier in the steady state.
template <int WT, int XM, int EPI>
__global__ void __launch_bounds__(GEMV_MAX_NT, 2) gemv_stream_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    constexpr int NT_CONS = GEMV_NW * 32;
    const bool is_producer = (tid >= NT_CONS);
    const int I = a.I, S = a.S;
    const int SR = a.dual ? 2 * S : S;

    const GemvSmem SL = gemv_smem_layout(a.ring, a.stage_bytes, SR, I);
    const uint32_t smem_sa = smem_u32(smem);  // shared-window address of the dynamic allocation
    const uint32_t xq_sa = smem_sa + SL.xq;
    uint8_t* ring = smem;
    uint32_t* rowtab = reinterpret_cast<uint32_t*>(smem + SL.rowtab);  // [ring][SR] byte offset of each row
    int* rowinfo = reinterpret_cast<int*>(smem + SL.rowinfo);           // [ring][SR] (tensor << 28) | row
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL.bars);
    uint64_t* empty = full + a.ring;
    float* misc = reinterpret_cast<float*>(smem + SL.misc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 32);
    float* warp_best_v = misc + 40;                        // [GEMV_NW]
    int* warp_best_i = reinterpret_cast<int*>(misc + 72);  // [GEMV_NW]

    // ---- CTA range of virtual rows (dual: pairs)
    const int G = gridDim.x;
    const int c = blockIdx.x;
    const int v_begin = (int)(((long long)a.Mv * c) / G);
    const int v_end = (int)(((long long)a.Mv * (c + 1)) / G);
    const int nstages = (v_end - v_begin + S - 1) / S;

    if (tid == 0) {
        for (int s = 0; s < a.ring; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GEMV_NW);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) pdl_launch_dependents();

    if (is_producer) {
        // ================= producer warp: publishes each stage's row table, lane 0 streams the bytes
        for (int s = 0; s < nstages; ++s) {
            const int slot = s % a.ring;
            if (s >= a.ring) {
                int ok = 0;
                if (lane == 0) {
                    ok = mbar_try_wait(&empty[slot], ((s / a.ring) - 1) & 1) ? 1 : 0;
                    for (uint32_t it = 0; !ok && it < FENCE_WAIT_ROUNDS && !*abort_flag; ++it)
                        if (mbar_try_wait(&empty[slot], ((s / a.ring) - 1) & 1)) { ok = 1; break; }
                    if (!ok) {
                        if (!*abort_flag) set_device_error(-5);
                        *abort_flag = 1;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
            const int va = v_begin + s * S;
            const int n = min(S, v_end - va);
            StageGeo geo;
            stage_geo(a, va, n, geo);
            const int rows_in_stage = a.dual ? 2 * n : n;
            for (int rr = lane; rr < rows_in_stage; rr += 32) {
                const int k = piece_of(geo, rr);
                uint32_t off = 0, delta = 0;
                int first = 0, r0 = 0;
#pragma unroll
                for (int j = 0; j < GEMV_MAX_SEG; ++j)
                    if (j == k) {
                        off = geo.p[j].smem_off;
                        delta = geo.p[j].delta;
                        first = geo.p[j].first_row;
                        r0 = geo.p[j].seg_row0;
                    }
                rowtab[slot * SR + rr] = (uint32_t)slot * a.stage_bytes + off + delta + (uint32_t)(rr - first) * a.rowB;
                rowinfo[slot * SR + rr] = (k << 28) | (r0 + rr - first);
            }
            __syncwarp();
            if (lane == 0) {
                uint8_t* dst = ring + (size_t)slot * a.stage_bytes;
                uint32_t tx = 0;
#pragma unroll
                for (int k = 0; k < GEMV_MAX_SEG; ++k) {
                    const Piece& pk = geo.p[k];
                    if (!pk.valid) continue;
                    tx += pk.copy_bytes;
                    // sub-16-byte tail of a tensor: plain 2-byte loads (released by the arrive)
                    if (pk.tail_bytes) {
                        const uint16_t* src = reinterpret_cast<const uint16_t*>(pk.src + pk.copy_bytes);
                        uint16_t* d16 = reinterpret_cast<uint16_t*>(dst + pk.smem_off + pk.copy_bytes);
                        for (uint32_t b = 0; b < pk.tail_bytes / 2; ++b) d16[b] = src[b];
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(&full[slot], tx);
#pragma unroll
                for (int k = 0; k < GEMV_MAX_SEG; ++k)
                    if (geo.p[k].valid && geo.p[k].copy_bytes)
                        bulk_g2s(dst + geo.p[k].smem_off, geo.p[k].src, geo.p[k].copy_bytes, &full[slot]);
            }
        }
        pdl_wait();
        return;
    }

    // ================= consumers
    pdl_wait();  // x, residual and epilogue targets come from the previous kernel

    // ---- prologue: x of every item quantised once per CTA into shared memory
    float rms = 1.f;
    if (XM == X_NORM || XM == X_NORM_R16) {
        const float* x = static_cast<const float*>(a.x);
        float ss = 0.f;
        for (int i = tid * 16; i < a.K; i += NT_CONS * 16) {
            const float4* q4 = reinterpret_cast<const float4*>(x + i);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 f = q4[k];
                ss += f.x * f.x + f.y * f.y + f.z * f.z + f.w * f.w;
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) misc[warp] = ss;
        named_bar_sync(1, NT_CONS);
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < GEMV_NW; ++w) tot += misc[w];
        rms = rsqrtf(tot / (float)a.K + a.eps);
    }
    for (int it = tid; it < I; it += NT_CONS) {
        XSlice<WT> t;
        make_slice<WT, XM>(a, it, rms, t);
        store_slice<WT>(xq_sa + it * XQ_WORDS * 4, t);
    }
    named_bar_sync(1, NT_CONS);

    constexpr int RBM = 2;  // max rows per lane group per batch
    const int RB = gemv_rows_per_group(a.dual);
    const int lpr = a.lpr;
    const int grp = lane / lpr, sub = lane - grp * lpr;
    const int BR = (32 / lpr) * RB;  // rows (pairs) per warp batch
    float best_v = 0.f;
    int best_i = -1;

    for (int s = 0; s < nstages; ++s) {
        const int slot = s % a.ring;
        const int va = v_begin + s * S;
        const int n = min(S, v_end - va);

        // fast path: one try; the abort flag (a shared-memory load queued behind the weight
        // loads) is read only when the slot is not full yet
        bool ok = mbar_try_wait(&full[slot], (s / a.ring) & 1);
        if (!ok && !*abort_flag) {
            for (uint32_t it = 0; it < FENCE_WAIT_ROUNDS && !*abort_flag; ++it)
                if (mbar_try_wait(&full[slot], (s / a.ring) & 1)) { ok = true; break; }
            if (!ok) {
                if (!*abort_flag) set_device_error(-5);
                *abort_flag = 1;
            }
        }
        // batches are dealt to warps round-robin over the CTA's whole row range (a stage may hold
        // fewer batches than there are warps)
        const int nbatch = ok ? (n + BR - 1) / BR : 0;
        const int gb0 = s * (S / BR);  // global index of this stage's first batch
        int b = warp - gb0 % GEMV_NW;
        if (b < 0) b += GEMV_NW;
        for (; b < nbatch; b += GEMV_NW) {
            // rows of this lane group: b*BR + grp*RB + j
            uint32_t ra[RBM], rb2[RBM];
            bool valid[RBM];
#pragma unroll
            for (int j = 0; j < RBM; ++j) {
                const int rr = b * BR + grp * RB + j;
                valid[j] = (j < RB) && rr < n;
                ra[j] = valid[j] ? smem_sa + rowtab[slot * SR + rr] : smem_sa;
                rb2[j] = (valid[j] && a.dual) ? smem_sa + rowtab[slot * SR + n + rr] : smem_sa;
            }
            float acc[RBM], acc2[RBM];
#pragma unroll
            for (int j = 0; j < RBM; ++j) acc[j] = acc2[j] = 0.f;
            for (int it = sub; it < I; it += lpr) {
                XSlice<WT> xs;
                load_slice<WT>(xq_sa + it * XQ_WORDS * 4, xs);
                const uint32_t io = (WT == WT_Q6K) ? (uint32_t)(it >> 2) * 210u : (uint32_t)it * 68u;
#pragma unroll
                for (int j = 0; j < RBM; ++j) {
                    if (valid[j]) {
                        acc[j] += item_dot<WT>(ra[j] + io, it, xs);
                        if (a.dual) acc2[j] += item_dot<WT>(rb2[j] + io, it, xs);
                    }
                }
            }
            // reduce inside the lane group (fixed xor order -> deterministic)
#pragma unroll
            for (int j = 0; j < RBM; ++j) {
                for (int o = lpr >> 1; o > 0; o >>= 1) {
                    acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
                    acc2[j] += __shfl_xor_sync(0xffffffffu, acc2[j], o);
                }
            }
            if (sub == 0) {
#pragma unroll
                for (int j = 0; j < RBM; ++j) {
                    if (!valid[j]) continue;
                    const int rr = b * BR + grp * RB + j;
                    const int info = rowinfo[slot * SR + rr];
                    const int row = info & 0x0FFFFFFF;
                    const float sum = acc[j];
                    if (EPI == EPI_SWIGLU) {
                        const float o = silu_mul(sum, acc2[j]);
                        if (a.act_f16) reinterpret_cast<__half*>(a.act)[row] = __float2half_rn(o);
                        else reinterpret_cast<float*>(a.act)[row] = o;
                    } else if (EPI == EPI_STORE) {
                        const int sgi = info >> 28;
                        float* yk = sgi == 0 ? a.seg[0].y : (sgi == 1 ? a.seg[1].y : a.seg[2].y);
                        const float* bk = sgi == 0 ? a.seg[0].bias : (sgi == 1 ? a.seg[1].bias : a.seg[2].bias);
                        yk[row] = bk ? sum + bk[row] : sum;
                    } else if (EPI == EPI_RESID) {
                        a.resid[row] = sum + a.resid[row];
                    } else if (EPI == EPI_LMHEAD) {
                        a.logits[row] = sum;
                        if (argmax_better(sum, row, best_v, best_i)) {
                            best_v = sum;
                            best_i = row;
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }

    if (EPI == EPI_LMHEAD) {
        // lane -> warp -> CTA best; the last CTA to arrive reduces all CTAs and advances the state
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (oi >= 0 && argmax_better(ov, oi, best_v, best_i)) {
                best_v = ov;
                best_i = oi;
            }
        }
        if (lane == 0) {
            warp_best_v[warp] = best_v;
            warp_best_i[warp] = best_i;
        }
        named_bar_sync(1, NT_CONS);
        if (tid == 0) {
            float bv = 0.f;
            int bi = -1;
            for (int w = 0; w < GEMV_NW; ++w)
                if (warp_best_i[w] >= 0 && argmax_better(warp_best_v[w], warp_best_i[w], bv, bi)) {
                    bv = warp_best_v[w];
                    bi = warp_best_i[w];
                }
            a.cta_val[c] = bv;
            a.cta_idx[c] = bi;
            __threadfence();
            const unsigned int prev = atomicAdd(a.counter, 1u);
            if (prev == (unsigned)G - 1) {
                __threadfence();
                float gv = 0.f;
                int gi = -1;
                for (int k = 0; k < G; ++k) {
                    const int ik = ((volatile int*)a.cta_idx)[k];
                    const float vk = ((volatile float*)a.cta_val)[k];
                    if (ik >= 0 && argmax_better(vk, ik, gv, gi)) {
                        gv = vk;
                        gi = ik;
                    }
                }
                if (gi < 0) gi = 0;
                if (a.state) {
                    DecodeState* st = a.state;
                    st->token = gi;
                    st->pos = st->pos + 1;
                    if (a.token_log && st->step < a.token_log_cap) a.token_log[st->step] = gi;
                    st->step = st->step + 1;
                }
                *a.counter = 0u;
            }
        }
    }
}

// --------------------------------------------------------------------------------------------
// Register-resident Q6_K GEMV for the drop-in gemv_q6k (fp16 x, plain store, optional bias) when a
// CTA's rows fit its shared memory in chunk slots and K <= 4096: lane <-> item. Each CTA owns
// consecutive rows; its producer lane issues every chunk of rows (1-D bulk copies on mbarriers)
// before griddepcontrol.wait, so under programmatic dependent launch the whole CTA's weights load
// while the previous kernel runs. After the wait, the x prologue quantises each 64-element item
// with 8 threads (one 16-byte load of fp16 x each; the item's max by shuffles) into shared-memory
// records; every consumer lane then keeps ITS item's record in registers for all rows. A row is
// worked on by LPR lanes (one item each: 64 lanes for K > 2048, else 32), so a row costs one item
// dot per lane and one shuffle reduction per warp, with no x reloads; the two warps' pieces of a
// row are summed in a fixed order at the end (deterministic). Consumer warps: GQ_NW.
constexpr int GQ_NW = 16;
constexpr int GQ_NT = GQ_NW * 32 + 32;
constexpr int GQ_MAX_SLOTS = 8;

struct GQArgs {
    const uint8_t* W;  // 16-byte aligned, rows of rowB bytes (rowB % 16 == 0)
    const uint16_t* x;
    const float* bias;
    float* y;
    int M, K, I, rowB;
    int rows_cta;      // rows of the first CTAs (the last may have fewer)
    int RC, slots;     // rows per chunk, chunk slots
    int slot_bytes;
};

__host__ __device__ inline uint32_t gq_xrec_off(int slots, int slot_bytes) { return (uint32_t)(slots * slot_bytes); }

__global__ void __launch_bounds__(GQ_NT, 1) gemv_q6k_reg_kernel(const __grid_constant__ GQArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NTC = GQ_NW * 32;
    const int I = a.I;
    const int r0 = blockIdx.x * a.rows_cta;
    const int rows = max(0, min(a.rows_cta, a.M - r0));
    const int nch = (rows + a.RC - 1) / a.RC;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t xq_sa = sbase + gq_xrec_off(a.slots, a.slot_bytes);
    float* part = reinterpret_cast<float*>(smem + gq_xrec_off(a.slots, a.slot_bytes) + I * XQ_WORDS * 4);  // [rows][2]
    uint64_t* full = reinterpret_cast<uint64_t*>(part + 2 * a.rows_cta + 2);
    full = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(full) + 7) & ~uintptr_t(7));
    uint64_t* empty = full + GQ_MAX_SLOTS;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + GQ_MAX_SLOTS);
    if (tid == 0) {
        for (int s = 0; s < a.slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GQ_NW);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) pdl_launch_dependents();

    if (warp == GQ_NW) {
        // ---- producer lane: every chunk of this CTA's rows (weights never depend on the previous kernel)
        if (lane == 0) {
            for (int i = 0; i < nch; ++i) {
                const int slot = i % a.slots;
                if (i >= a.slots) {
                    bool ok = mbar_try_wait(&empty[slot], ((i / a.slots) - 1) & 1);
                    for (uint32_t it = 0; !ok && it < FENCE_WAIT_ROUNDS && !*abort_flag; ++it)
                        ok = mbar_try_wait(&empty[slot], ((i / a.slots) - 1) & 1);
                    if (!ok) {
                        if (!*abort_flag) set_device_error(-5);
                        *abort_flag = 1;
                        break;
                    }
                }
                const int n = min(a.RC, rows - i * a.RC);
                const uint32_t bytes = (uint32_t)n * (uint32_t)a.rowB;
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_g2s(smem + (size_t)slot * a.slot_bytes, a.W + (size_t)(r0 + i * a.RC) * a.rowB, bytes, &full[slot]);
            }
        }
        return;
    }

    // ---- consumers
    pdl_wait();  // x and y belong to the stream's previous work
    // x prologue: task t = (item, run c, half): 8 consecutive fp16 of run c of the item
    for (int t0 = 0; t0 < I * 8; t0 += NTC) {
        const int t = t0 + tid;
        const bool on = t < I * 8;
        const int item = on ? t >> 3 : 0, c = (t >> 1) & 3, hh = t & 1;
        const int b = item >> 2, h = (item >> 1) & 1, l16 = item & 1;
        const int base = b * 256 + h * 128 + c * 32 + l16 * 16 + hh * 8;
        float v[8];
        if (on) {
            const uint4 u = *reinterpret_cast<const uint4*>(a.x + base);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[2 * k] = half_bits_to_float(w[k]);
                v[2 * k + 1] = half_bits_to_float(w[k] >> 16);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = 0.f;
        }
        float amax = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));  // the item's 8 tasks
        float inv;
        const float xs = quant_scale(amax, inv);
        uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
        int sum = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int q = __float2int_rn(v[k] * inv);
            sum += q;
            uint32_t hb, lb;
            split16(q, hb, lb);
            hw[k >> 2] |= hb << (8 * (k & 3));
            lw[k >> 2] |= lb << (8 * (k & 3));
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // the run's two halves
        if (on) {
            const uint32_t rec = xq_sa + (uint32_t)item * XQ_WORDS * 4;
            const int wi = c * 4 + hh * 2;  // XSlice word index of the first of this task's two words
            asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(rec + wi * 4), "r"(hw[0]), "r"(hw[1]) : "memory");
            asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(rec + (16 + wi) * 4), "r"(lw[0]), "r"(lw[1]) : "memory");
            if (hh == 0) asm volatile("st.shared.b32 [%0], %1;" ::"r"(rec + (32 + c) * 4), "r"(-32 * sum) : "memory");
            if (hh == 0 && c == 0) {
                asm volatile("st.shared.b32 [%0], %1;" ::"r"(rec + 36 * 4), "r"(__float_as_uint(xs)) : "memory");
                asm volatile("st.shared.b32 [%0], %1;" ::"r"(rec + 37 * 4), "r"(0u) : "memory");
            }
        }
    }
    named_bar_sync(1, NTC);

    const int LPR = I > 32 ? 64 : 32, WPG = LPR / 32, NG = GQ_NW / WPG;
    const int g = warp / WPG, item = (warp % WPG) * 32 + lane;
    const bool has_item = item < I;
    XSlice<WT_Q6K> xs;
    load_slice<WT_Q6K>(xq_sa + (uint32_t)(has_item ? item : 0) * XQ_WORDS * 4, xs);
    const uint32_t ioff = (uint32_t)(item >> 2) * 210u;
    for (int i = 0; i < nch; ++i) {
        const int slot = i % a.slots;
        bool ok = mbar_try_wait(&full[slot], (i / a.slots) & 1);
        if (!ok && !*abort_flag) {
            for (uint32_t it = 0; it < FENCE_WAIT_ROUNDS && !*abort_flag; ++it)
                if (mbar_try_wait(&full[slot], (i / a.slots) & 1)) { ok = true; break; }
            if (!ok) {
                if (!*abort_flag) set_device_error(-5);
                *abort_flag = 1;
            }
        }
        const int n = min(a.RC, rows - i * a.RC);
        if (ok) {
            const uint32_t cb = sbase + (uint32_t)slot * a.slot_bytes;
            for (int rr = g; rr < n; rr += NG) {
                float d = has_item ? item_dot<WT_Q6K>(cb + (uint32_t)rr * a.rowB + ioff, item, xs) : 0.f;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                if (lane == 0) part[(i * a.RC + rr) * 2 + (warp % WPG)] = d;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    named_bar_sync(1, NTC);
    if (*abort_flag) return;
    for (int r = tid; r < rows; r += NTC) {
        float v = part[r * 2] + (WPG > 1 ? part[r * 2 + 1] : 0.f);
        if (a.bias) v += a.bias[r0 + r];
        a.y[r0 + r] = v;
    }
}

// --------------------------------------------------------------------------------------------
// Simple kernels for shapes the streaming kernel does not take (K % 64 != 0 for Q8_0, huge K,
// misaligned weights): one warp per row, fp32 accumulation in the reference's per-lane order.
__global__ void gemv_q6k_simple_kernel(const uint8_t* __restrict__ W, const uint16_t* __restrict__ x,
                                       const float* __restrict__ bias, float* __restrict__ y, int M,
                                       int K);
__global__ void gemv_q8_0_simple_kernel(const uint8_t* __restrict__ W, const float* __restrict__ x,
                                        float* __restrict__ y, int M, int K);

// Host-side launch planning for the streaming kernel.
struct GemvPlan {
    int ok;
    int grid, block, smem;
    int S, lpr, ring, stage_bytes, I, rowB;
};

}  // namespace fence
