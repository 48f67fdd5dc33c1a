// rgemv.cuh — the engine's streaming GEMV over REPACKED weights (sm_100a).
//
// The drop-in launchers read the reference's GGUF blocks as they are (gemv.cuh), whose Q6_K
// super-blocks are 210 bytes long and so sit at 2-byte alignment in shared memory; every 16-byte
// load then costs five 4-byte loads and four funnel shifts, and the access pattern hits few banks.
// The engine owns its weights, so at load time it rewrites every linear once into an aligned,
// bank-friendly layout with the SAME bytes per weight (repack kernels in rgemv.cu):
//
//   Q6_K  (K/256 super-blocks of 210 B per row; item = 64 weights = (super-block j, half h, l16))
//     q[row][item][48]  ql[64h+16*l16 .. +16] | ql[64h+32+16*l16 .. +16] | qh[32h+16*l16 .. +16]
//     s[row][item][4]   int8 scales of the item's four 16-element columns: sc[8h + 2c + l16]
//     d[row][K/256]     fp16 super-block scale d
//   Q8_0  (K/32 blocks of 34 B per row; item = 64 weights = blocks 2i, 2i+1)
//     q[row][item][64]  the item's 64 int8 quants in four 16-byte chunks; chunk k is stored at
//                       position k ^ ((item >> 1) & 3), so the 8 lanes of a quarter warp reading
//                       position p of 8 consecutive items hit 8 different 16-byte bank groups
//     d[row][item][2]   fp16 d of block 2i, then of block 2i+1
//
// The arithmetic per item is the drop-in kernels' (gemv.cuh item_dot) operation for operation:
// the integer dot products are exact and the float expression is the same, so the engine's
// results do not depend on the layout.
//
// Kernel (one CTA per SM, 7 consumer warps + 1 producer warp, so that the next phase's kernel fits
// beside it on the SM and streams its weights under programmatic dependent launch):
//  * producer: streams the CTA's rows in stages of R rows (3 bulk copies per stage: q, s, d slices)
//    into a ring of shared-memory slots guarded by mbarriers;
//  * consumers: quantise x once per CTA, then every stage is worked on by ALL consumer lanes: lane
//    gl owns one (row, item) of the stage — the same item for the whole kernel, its x held in
//    registers; a row longer than the lanes is split into equal parts — and a segmented shuffle
//    reduction sums each row part inside a warp; the first lane of each segment stores that
//    per-warp piece in shared memory. Nothing else (no atomics, no global traffic) sits in the
//    stage loop: after the last stage one thread per row adds the row's pieces in a fixed order
//    (deterministic) and runs the fused epilogue with coalesced global accesses.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace fence {

constexpr int RG_NW = 7;                 // consumer warps
constexpr int RG_NT = RG_NW * 32 + 32;   // + producer warp
constexpr int RG_NL = RG_NW * 32;        // consumer lanes
constexpr int RG_MAX_R = 64;             // row slots per stage
constexpr int RG_MAX_RING = 12;

// Repacked matrix (see the layout above). Arrays are padded by 64 bytes so stage copies rounded up
// to 16 bytes stay inside the allocation.
struct RMat {
    const uint8_t* q;
    const uint8_t* s;  // Q6_K only
    const uint8_t* d;
    int rows;
    int iph;           // Q6_K column slice starting inside a super-block: its first item's index
                       // within that super-block (0..3); local item i uses d entry (i + iph) / 4
};

struct RGemvArgs {
    RMat w;
    int wt;
    int I;            // items (64 weights) per row
    int np;           // parts per row (rows longer than the consumer lanes are split in np equal parts)
    int ipl;          // (unused by the tiled step kernel; kept 1)
    int R;            // rows per stage (dual: even; rows 2p, 2p+1 are gate/up of pair p)
    int dual;
    int Mv;           // virtual rows (dual: gate/up pairs)
    int ring;         // slots in the ring
    int slot_bytes;
    int mp;           // max per-warp pieces of one row's reduction
    int rows_cta;     // max rows (dual: 2 x pairs) of one CTA
    // x source
    const void* x;
    const float* norm_w;
    float eps;
    // epilogues
    float* y;            // EPI_STORE (row-indexed)
    const float* bias;   // EPI_STORE, optional
    float* resid;        // EPI_RESID
    void* act;           // EPI_SWIGLU (pair-indexed)
    int act_f16;
    float* logits;       // EPI_LMHEAD
    float* cta_val;
    int* cta_idx;
    unsigned int* counter;
    DecodeState* state;
    int* token_log;
    int token_log_cap;
    // step kernel: the matrix re-tiled per CTA into row blocks of RB rows x K-slices of CI items,
    // each tile contiguous (sk_tile_bytes) and streamed by one bulk copy; tcta[c] = byte offset of
    // CTA c's first tile in tb
    const uint8_t* tb;
    const unsigned long long* tcta;
    int RB, CI;
    int pad_[2];
};

// ---- tiles of the step kernel's weights (one (row block, K-slice) of one CTA's rows)
// Q8_0: q [n][64] (chunk k of record (row, slot s) at 16-byte position k ^ ((s >> 1) & 3)) | d [n][4]
// Q6_K: q [n][48] | s [n][4] | d [rows][ndq] (fp16 d of the super-blocks the slice overlaps)
// with n = rows x items records in (row, slot) order, every part 16-byte aligned.
__host__ __device__ inline int sk_ndq(int CI) { return (CI + 3) / 4 + 1; }
__host__ __device__ inline uint32_t sk_tile_bytes(int wt, int rows, int items, int CI, uint32_t* s_off = nullptr,
                                                  uint32_t* d_off = nullptr) {
    const uint32_t n = (uint32_t)rows * (uint32_t)items;
    const uint32_t q = n * (uint32_t)(wt == WT_Q6K ? 48 : 64);
    const uint32_t so = q;
    const uint32_t doff = (wt == WT_Q6K) ? ((so + 4u * n + 15u) & ~15u) : q;
    const uint32_t db = (wt == WT_Q6K) ? (uint32_t)rows * (uint32_t)sk_ndq(CI) * 2u : 4u * n;
    if (s_off) *s_off = so;
    if (d_off) *d_off = doff;
    return (doff + db + 15u) & ~15u;
}

// Launch plan (host).
struct RGemvPlan {
    int ok;
    int grid, block, smem;
};

__host__ __device__ inline int rg_qbytes(int wt) { return wt == WT_Q6K ? 48 : 64; }
__host__ __device__ inline int rg_dbytes_row(int wt, int I, int iph = 0) {
    return wt == WT_Q6K ? ((I + iph + 3) >> 2) * 2 : I * 4;
}
// Q6_K scale bytes of one row (4 per item), padded to 16 so that every row starts 16-byte aligned
// for the bulk copies (a tensor-parallel column slice may hold a number of items not divisible by 4)
__host__ __device__ inline int rg_sbytes_row(int wt, int I) { return wt == WT_Q6K ? (I * 4 + 15) & ~15 : 0; }

// Shared-memory layout of one slot: [q | s | d] each 16-aligned, d copied from a 16-aligned source
// below its first row (the offset of that row inside the copy is recomputed by the consumers).
struct RSlot {
    uint32_t s_off, d_off, bytes;
};
__host__ __device__ inline RSlot rg_slot(int wt, int I, int R, int iph = 0) {
    RSlot L;
    const uint32_t qb = (uint32_t)R * I * rg_qbytes(wt);
    const uint32_t sb = (uint32_t)R * rg_sbytes_row(wt, I);
    const uint32_t db = (uint32_t)R * rg_dbytes_row(wt, I, iph);
    L.s_off = (qb + 15u) & ~15u;
    L.d_off = (L.s_off + sb + 15u) & ~15u;
    L.bytes = (L.d_off + db + 16u + 15u) & ~15u;  // + up to 15 bytes of d alignment slack
    return L;
}

struct RGSmem {
    uint32_t xq, acc, bars, misc, total;
};
__host__ __device__ inline RGSmem rg_smem_layout(int ring, int slot_bytes, int I, int rows_cta, int mp) {
    auto r16 = [](uint32_t x) { return (x + 15u) & ~15u; };
    RGSmem L;
    L.xq = (uint32_t)ring * (uint32_t)slot_bytes;
    L.acc = L.xq + r16((uint32_t)I * XQ_WORDS * 4u);
    L.bars = L.acc + r16(4u * (uint32_t)rows_cta * (uint32_t)mp);
    L.misc = L.bars + r16(16u * ring);
    L.total = L.misc + 512u;
    return L;
}

// Per-warp pieces of row slot rs's reduction (np parts of ip items, lanes rs*np*ip ..).
__host__ __device__ inline int rg_part_pieces(int rs, int pt, int np, int ip) {
    const int lo = (rs * np + pt) * ip;
    return ((lo + ip - 1) >> 5) - (lo >> 5) + 1;
}
__host__ __device__ inline int rg_row_pieces(int rs, int np, int ip) {
    int n = 0;
    for (int pt = 0; pt < np; ++pt) n += rg_part_pieces(rs, pt, np, ip);
    return n;
}

// ---------------------------------------------------------------------------------------------
// x: one 40-word record per item in shared memory, built by a group of lanes.
//   Q6_K: xh[16] | xl[16] | corr[4] | xs | 0 0 0 ; word 4c+k = elements 4k..4k+3 of column c
//   Q8_0: xh[16] | xl[16] | 0 0 0 0 | xs0 | xs1 | 0 0 ; word w = elements 4w..4w+3 of the item
// Every record is built by 4 lanes of one warp, 16 values each: Q6_K lane q holds column q, Q8_0
// lane q elements 16q..16q+15 (block q / 2, whose scale is a max over the lane pair).
// The arithmetic is make_slice's (gemv.cuh) element for element; the group's amax is an exact max.
constexpr int RG_LPI = 4;   // lanes per x record
constexpr int RG_NV = 16;   // x values per lane
template <int WT>
__device__ __forceinline__ int rg_task_base(int item, int q) {
    if (WT == WT_Q6K) {
        const int b = item >> 2, h = (item >> 1) & 1, l16 = item & 1;
        return b * 256 + h * 128 + q * 32 + l16 * 16;
    }
    return item * 64 + q * 16;
}

// Raw x values of one record-building task (Q6_K: 16 values of column q; Q8_0: elements 16q..).
template <int WT, int XM>
__device__ __forceinline__ void rg_load_task(const void* xsrc, int base, float (&v)[RG_NV]) {
    constexpr int NV = RG_NV;
    if (XM == X_F16) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xsrc) + base);
#pragma unroll
        for (int c = 0; c < NV / 8; ++c) {
            const uint4 u = p[c];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[c * 8 + 2 * k] = half_bits_to_float(w[k]);
                v[c * 8 + 2 * k + 1] = half_bits_to_float(w[k] >> 16);
            }
        }
    } else {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(xsrc) + base);
#pragma unroll
        for (int c = 0; c < NV / 4; ++c) {
            const float4 f = p[c];
            v[4 * c] = f.x;
            v[4 * c + 1] = f.y;
            v[4 * c + 2] = f.z;
            v[4 * c + 3] = f.w;
        }
    }
}

// Normalise / round the task's values as make_slice does (gemv.cuh), quantise them with the
// item's scale (a max over the lane group: exact) and store the task's words of the record.
// All lanes of the warp call this (shuffles); lanes with active == false store nothing.
template <int WT, int XM>
__device__ __forceinline__ void rg_quant_store(float (&v)[RG_NV], const float (&w)[RG_NV], int q, float rms,
                                               uint32_t rec, bool active) {
    constexpr int NV = RG_NV;
    if (XM == X_NORM || XM == X_NORM_R16) {  // w[i] * x[i] * rms, the reference's order (ops.cuh:43)
#pragma unroll
        for (int e = 0; e < NV; ++e) v[e] = (v[e] * w[e]) * rms;
    }
    if (XM == X_F32_R16 || XM == X_NORM_R16) {
#pragma unroll
        for (int e = 0; e < NV; ++e) v[e] = round_f16(v[e]);
    }
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < NV; ++e) amax = fmaxf(amax, fabsf(v[e]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));      // Q8_0: the block's lane pair
    if (WT == WT_Q6K) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));  // Q6_K: the item
    float inv;
    const float xs = quant_scale(amax, inv);
    if (!active) return;
    int sum = 0;
#pragma unroll
    for (int k = 0; k < NV / 4; ++k) {
        uint32_t hw = 0u, lw = 0u;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int qv = __float2int_rn(v[4 * k + j] * inv);
            sum += qv;
            uint32_t hb, lb;
            split16(qv, hb, lb);
            hw |= hb << (8 * j);
            lw |= lb << (8 * j);
        }
        const uint32_t wi = (uint32_t)(4 * q + k);
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(rec + 4u * wi), "r"(hw) : "memory");
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(rec + 64u + 4u * wi), "r"(lw) : "memory");
    }
    if (WT == WT_Q6K) {
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(rec + 128u + 4u * q), "r"(-32 * sum) : "memory");
        if (q == 0)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rec + 144u), "r"(__float_as_uint(xs)),
                         "r"(0u), "r"(0u), "r"(0u) : "memory");
    } else {
        if ((q & 1) == 0)
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(rec + 144u + 2u * q), "r"(__float_as_uint(xs)) : "memory");
        if (q == 0)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rec + 128u), "r"(0u), "r"(0u), "r"(0u),
                         "r"(0u) : "memory");
        else if (q == 1)
            asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(rec + 152u), "r"(0u), "r"(0u) : "memory");
    }
}

// Per-lane x of its item, in the order its weight loads deliver them.
struct RX {
    uint32_t xh[16], xl[16];
    int corr[4];     // Q6_K: -32 * sum of the column's quantised x
    float xsA, xsB;  // Q6_K: xsA; Q8_0: scale of block 0 (chunks 0-1) / block 1 (chunks 2-3)
    uint32_t sw;     // Q8_0: byte offset of chunk k in the item record is (16 k) ^ sw
};

template <int WT>
__device__ __forceinline__ void rg_load_x(uint32_t rec, int item, RX& x) {
    if (WT == WT_Q6K) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 a = lds128(rec + 16u * k), b = lds128(rec + 64u + 16u * k);
            x.xh[4 * k] = a.x; x.xh[4 * k + 1] = a.y; x.xh[4 * k + 2] = a.z; x.xh[4 * k + 3] = a.w;
            x.xl[4 * k] = b.x; x.xl[4 * k + 1] = b.y; x.xl[4 * k + 2] = b.z; x.xl[4 * k + 3] = b.w;
        }
        const uint4 c = lds128(rec + 128u);
        x.corr[0] = (int)c.x; x.corr[1] = (int)c.y; x.corr[2] = (int)c.z; x.corr[3] = (int)c.w;
        x.xsA = __uint_as_float(lds32(rec + 144u));
        x.xsB = 0.f;
        x.sw = 0u;
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 a = lds128(rec + 16u * k), b = lds128(rec + 64u + 16u * k);
            x.xh[4 * k] = a.x; x.xh[4 * k + 1] = a.y; x.xh[4 * k + 2] = a.z; x.xh[4 * k + 3] = a.w;
            x.xl[4 * k] = b.x; x.xl[4 * k + 1] = b.y; x.xl[4 * k + 2] = b.z; x.xl[4 * k + 3] = b.w;
        }
        x.xsA = __uint_as_float(lds32(rec + 144u));
        x.xsB = __uint_as_float(lds32(rec + 148u));
        // the repack stores chunk k of item i at slot k ^ ((i >> 1) & 3): reading chunk k there, the
        // eight lanes of a quarter-warp (consecutive items, 64-byte records) hit eight different
        // 16-byte bank groups
        x.sw = ((uint32_t)(item >> 1) & 3u) << 4;
        x.corr[0] = x.corr[1] = x.corr[2] = x.corr[3] = 0;
    }
}

// The words of one item a lane needs from a stage: Q6_K ql0 | ql1 | qh (12 words), its scale word
// and the super-block d; Q8_0 the 4 quant chunks (16 words) and the item's two d.
template <int WT>
struct RWT {
    uint32_t w[WT == WT_Q6K ? 12 : 16];
    uint32_t sc, d;
};

// Loads an item's words: q, s, d are 32-bit shared addresses of the item's record, its scale word
// (Q6_K) and its d (Q6_K: the super-block's fp16; Q8_0: the item's two fp16).
template <int WT>
__device__ __forceinline__ void rg_item_load(uint32_t q, uint32_t s, uint32_t d, uint32_t sw, RWT<WT>& r) {
    if constexpr (WT == WT_Q6K) {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const uint4 u = lds128(q + 16u * k);
            r.w[4 * k] = u.x; r.w[4 * k + 1] = u.y; r.w[4 * k + 2] = u.z; r.w[4 * k + 3] = u.w;
        }
        r.sc = lds32(s);
        r.d = lds_u16(d);
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 u = lds128(q + ((16u * k) ^ sw));
            r.w[4 * k] = u.x; r.w[4 * k + 1] = u.y; r.w[4 * k + 2] = u.z; r.w[4 * k + 3] = u.w;
        }
        r.sc = 0u;
        r.d = lds32(d);
    }
}

// 64-weight item dot of loaded words with the lane's x.
template <int WT>
__device__ __forceinline__ float rg_item_compute(const RWT<WT>& r, const RX& x) {
    if constexpr (WT == WT_Q6K) {
        int hi0 = 0, hi1 = 0, hi2 = 0, hi3 = 0;
        int lo0 = x.corr[0], lo1 = x.corr[1], lo2 = x.corr[2], lo3 = x.corr[3];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t ql0 = r.w[k], ql1 = r.w[4 + k], qh = r.w[8 + k];
            const uint32_t qm = qh & 0x33333333u;  // crumbs of columns 0 (bits 0-1) and 2 (bits 4-5)
            const uint32_t qn = qh & 0xCCCCCCCCu;  // crumbs of columns 1 (bits 2-3) and 3 (bits 6-7)
            const uint32_t q0 = (ql0 & 0x0F0F0F0Fu) | ((qm << 4) & 0xF0F0F0F0u);
            const uint32_t q1 = (ql1 & 0x0F0F0F0Fu) | ((qn << 2) & 0xF0F0F0F0u);
            const uint32_t q2 = ((ql0 >> 4) & 0x0F0F0F0Fu) | (qm & 0xF0F0F0F0u);
            const uint32_t q3 = ((ql1 >> 4) & 0x0F0F0F0Fu) | ((qn >> 2) & 0xF0F0F0F0u);
            hi0 = dp4a_us(q0, x.xh[0 * 4 + k], hi0);
            lo0 = dp4a_uu(q0, x.xl[0 * 4 + k], lo0);
            hi1 = dp4a_us(q1, x.xh[1 * 4 + k], hi1);
            lo1 = dp4a_uu(q1, x.xl[1 * 4 + k], lo1);
            hi2 = dp4a_us(q2, x.xh[2 * 4 + k], hi2);
            lo2 = dp4a_uu(q2, x.xl[2 * 4 + k], lo2);
            hi3 = dp4a_us(q3, x.xh[3 * 4 + k], hi3);
            lo3 = dp4a_uu(q3, x.xl[3 * 4 + k], lo3);
        }
        const uint32_t sc = r.sc;
        const int sc0 = (int)(sc << 24) >> 24, sc1 = (int)(sc << 16) >> 24;
        const int sc2 = (int)(sc << 8) >> 24, sc3 = (int)sc >> 24;
        const float t = (float)((hi0 * 256 + lo0) * sc0) + (float)((hi1 * 256 + lo1) * sc1) +
                        (float)((hi2 * 256 + lo2) * sc2) + (float)((hi3 * 256 + lo3) * sc3);
        return t * (half_bits_to_float(r.d) * x.xsA);
    } else {
        int hiA = 0, loA = 0, hiB = 0, loB = 0;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            if (m < 8) {
                hiA = dp4a_ss(r.w[m], x.xh[m], hiA);
                loA = dp4a_su(r.w[m], x.xl[m], loA);
            } else {
                hiB = dp4a_ss(r.w[m], x.xh[m], hiB);
                loB = dp4a_su(r.w[m], x.xl[m], loB);
            }
        }
        const float dA = half_bits_to_float(r.d & 0xffffu);
        const float dB = half_bits_to_float(r.d >> 16);
        return (float)(hiA * 256 + loA) * (dA * x.xsA) + (float)(hiB * 256 + loB) * (dB * x.xsB);
    }
}

// 64-weight item dot of repacked weights straight from shared memory.
template <int WT>
__device__ __forceinline__ float rg_item_dot(uint32_t q, uint32_t s, uint32_t d, const RX& x) {
    RWT<WT> r;
    rg_item_load<WT>(q, s, d, x.sw, r);
    return rg_item_compute<WT>(r, x);
}

// Epilogue of one finished row (or gate/up pair).
template <int EPI>
__device__ __forceinline__ void rg_epilogue(const RGemvArgs& a, int row, float sum, float sum2, float& best_v,
                                            int& best_i) {
    if (EPI == EPI_SWIGLU) {
        const float o = silu_mul(sum, sum2);
        if (a.act_f16) reinterpret_cast<__half*>(a.act)[row] = __float2half_rn(o);
        else reinterpret_cast<float*>(a.act)[row] = o;
    } else if (EPI == EPI_STORE) {
        a.y[row] = a.bias ? sum + a.bias[row] : sum;
    } else if (EPI == EPI_RESID) {
        a.resid[row] = sum + a.resid[row];
    } else {
        a.logits[row] = sum;
        if (argmax_better(sum, row, best_v, best_i)) {
            best_v = sum;
            best_i = row;
        }
    }
}

template <int WT, int XM, int EPI>
__global__ void __launch_bounds__(RG_NT, 2) rgemv_kernel(const __grid_constant__ RGemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool is_producer = tid >= RG_NL;
    const int I = a.I, R = a.R, ring = a.ring;
    const bool dual = a.dual != 0;
    const int S = dual ? R / 2 : R;  // virtual rows per stage
    const RGSmem SL = rg_smem_layout(ring, a.slot_bytes, I, a.rows_cta, a.mp);
    const RSlot SS = rg_slot(WT, I, R, a.w.iph);
    const uint32_t smem_sa = smem_u32(smem);
    const uint32_t xq_sa = smem_sa + SL.xq;
    float* acc = reinterpret_cast<float*>(smem + SL.acc);  // [rows of the CTA][mp] reduction pieces
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL.bars);
    uint64_t* empty = full + ring;
    float* misc = reinterpret_cast<float*>(smem + SL.misc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 32);
    float* warp_best_v = misc + 40;
    int* warp_best_i = reinterpret_cast<int*>(misc + 72);

    const int G = gridDim.x, c = blockIdx.x;
    const int v_begin = (int)(((long long)a.Mv * c) / G), v_end = (int)(((long long)a.Mv * (c + 1)) / G);
    const int nstages = (v_end - v_begin + S - 1) / S;
    const int qb = rg_qbytes(WT), sbr = rg_sbytes_row(WT, I), dbr = rg_dbytes_row(WT, I, a.w.iph);

    if (tid == 0) {
        for (int s = 0; s < ring; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], RG_NW);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) pdl_launch_dependents();

    if (is_producer) {
        // ================= producer: weights never depend on the previous kernel, so it streams
        // before griddepcontrol.wait
        if (lane == 0) {
            for (int s = 0; s < nstages; ++s) {
                const int slot = s % ring;
                if (s >= ring) {
                    bool ok = mbar_try_wait(&empty[slot], ((s / ring) - 1) & 1);
                    for (uint32_t it = 0; !ok && it < FENCE_WAIT_ROUNDS && !*abort_flag; ++it)
                        if (mbar_try_wait(&empty[slot], ((s / ring) - 1) & 1)) { ok = true; break; }
                    if (!ok) {
                        if (!*abort_flag) set_device_error(-5);
                        *abort_flag = 1;
                        break;
                    }
                }
                const int v0 = v_begin + s * S;
                const int nv = min(S, v_end - v0);
                const long long row0 = dual ? 2ll * v0 : v0;
                const uint32_t nrows = dual ? 2u * nv : (uint32_t)nv;
                uint8_t* dst = smem + (size_t)slot * a.slot_bytes;
                const uint32_t qbytes = nrows * (uint32_t)I * qb;
                const uint32_t sbytes = nrows * (uint32_t)sbr;
                const uint64_t d0 = (uint64_t)row0 * dbr;
                const uint64_t d0a = d0 & ~uint64_t(15);
                const uint32_t dbytes = ((uint32_t)(d0 - d0a) + nrows * (uint32_t)dbr + 15u) & ~15u;
                mbar_arrive_expect_tx(&full[slot], qbytes + sbytes + dbytes);
                bulk_g2s(dst, a.w.q + (uint64_t)row0 * I * qb, qbytes, &full[slot]);
                if (sbytes) bulk_g2s(dst + SS.s_off, a.w.s + (uint64_t)row0 * sbr, sbytes, &full[slot]);
                bulk_g2s(dst + SS.d_off, a.w.d + d0a, dbytes, &full[slot]);
            }
        }
        __syncwarp();
        pdl_wait();
        return;
    }

    // ================= consumers
    constexpr int NT = RG_NL;
    constexpr int LPI = RG_LPI;  // lanes per x record
    constexpr int NV = RG_NV;
    constexpr bool NORM = (XM == X_NORM || XM == X_NORM_R16);
    const int ntask = I * LPI;
    // norm weights do not depend on the previous kernel: fetch them before the wait
    constexpr int PASSES = 2;  // task passes kept in registers (more re-read x)
    float wv[PASSES][NV];
    if (NORM) {
#pragma unroll
        for (int ps = 0; ps < PASSES; ++ps) {
            const int idx = ps * NT + tid;
            const int base = idx < ntask ? rg_task_base<WT>(idx / LPI, idx % LPI) : 0;
            const float4* p = reinterpret_cast<const float4*>(a.norm_w + base);
#pragma unroll
            for (int cc = 0; cc < NV / 4; ++cc) {
                const float4 f = p[cc];
                wv[ps][4 * cc] = f.x;
                wv[ps][4 * cc + 1] = f.y;
                wv[ps][4 * cc + 2] = f.z;
                wv[ps][4 * cc + 3] = f.w;
            }
        }
    }
    pdl_wait();  // x, residual and epilogue targets come from the previous kernel

    // ---- x prologue: load (sum of squares for RMSNorm), quantise once per CTA into shared memory
    {
        float xv[PASSES][NV];
        float ss = 0.f;
#pragma unroll
        for (int ps = 0; ps < PASSES; ++ps) {
            const int idx = ps * NT + tid;
            const int base = idx < ntask ? rg_task_base<WT>(idx / LPI, idx % LPI) : 0;
            rg_load_task<WT, XM>(a.x, base, xv[ps]);
            if (NORM && idx < ntask) {
#pragma unroll
                for (int e = 0; e < NV; ++e) ss += xv[ps][e] * xv[ps][e];
            }
        }
        float rms = 1.f;
        if (NORM) {
            for (int b0 = PASSES * NT + tid; b0 < ntask; b0 += NT) {  // beyond the register passes
                float t[NV];
                rg_load_task<WT, XM>(a.x, rg_task_base<WT>(b0 / LPI, b0 % LPI), t);
#pragma unroll
                for (int e = 0; e < NV; ++e) ss += t[e] * t[e];
            }
            ss = warp_sum(ss);
            if (lane == 0) misc[warp] = ss;
            named_bar_sync(1, NT);
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < RG_NW; ++w) tot += misc[w];
            rms = rsqrtf(tot / (float)(I * 64) + a.eps);
        }
        // quantise: register passes (static index), then any remaining tasks straight from memory;
        // trip counts are warp-uniform (shuffles inside)
#pragma unroll
        for (int ps = 0; ps < PASSES; ++ps) {
            const int b0 = ps * NT + warp * 32;
            if (b0 < ntask) {
                const int idx = b0 + lane;
                const bool active = idx < ntask;
                const int item = active ? idx / LPI : 0, q = idx % LPI;
                rg_quant_store<WT, XM>(xv[ps], wv[ps], q, rms, xq_sa + item * XQ_WORDS * 4, active);
            }
        }
        for (int b0 = PASSES * NT + warp * 32; b0 < ntask; b0 += NT) {
            const int idx = b0 + lane;
            const bool active = idx < ntask;
            const int item = active ? idx / LPI : 0, q = idx % LPI;
            float t[NV], tw[NV];
            const int base = active ? rg_task_base<WT>(item, q) : 0;
            rg_load_task<WT, XM>(a.x, base, t);
            if (NORM) {
                const float4* p = reinterpret_cast<const float4*>(a.norm_w + base);
#pragma unroll
                for (int cc = 0; cc < NV / 4; ++cc) {
                    const float4 f = p[cc];
                    tw[4 * cc] = f.x;
                    tw[4 * cc + 1] = f.y;
                    tw[4 * cc + 2] = f.z;
                    tw[4 * cc + 3] = f.w;
                }
            }
            rg_quant_store<WT, XM>(t, tw, q, rms, xq_sa + item * XQ_WORDS * 4, active);
        }
    }
    named_bar_sync(1, NT);

    // ---- lane <-> (slot, item): slot = (row of the stage, part of the row), IP items per part
    const int NP = a.np, IP = I / NP, MP = a.mp;
    const int sl = tid / IP, itp = tid - sl * IP;
    const int rs = sl / NP, pt = sl - rs * NP, it = pt * IP + itp;
    const bool lane_on = rs < R;
    RX x;
    if (lane_on) rg_load_x<WT>(xq_sa + it * XQ_WORDS * 4, it, x);
    const int slot_lo = sl * IP;
    const int seg_hi = min(slot_lo + IP - 1 - warp * 32, 31);
    const bool head = lane == max(slot_lo - warp * 32, 0);
    int pidx = warp - (slot_lo >> 5);  // this segment's piece index in its row's reduction
    for (int p2 = 0; p2 < pt; ++p2) pidx += rg_part_pieces(rs, p2, NP, IP);
    const uint32_t q_off = (uint32_t)(rs * I + it) * qb;
    const uint32_t s_off = SS.s_off + (uint32_t)(rs * rg_sbytes_row(WT, I) + it * 4);
    const int nsbl = rg_dbytes_row(WT, I, a.w.iph) / 2;  // Q6_K d entries per row
    const uint32_t d_off = SS.d_off + (WT == WT_Q6K ? (uint32_t)(rs * nsbl + ((it + a.w.iph) >> 2)) * 2u
                                                     : (uint32_t)(rs * I + it) * 4u);
    const long long row_begin = dual ? 2ll * v_begin : v_begin;

    for (int s = 0; s < nstages; ++s) {
        const int slot = s % ring;
        const int v0 = v_begin + s * S;
        const int nv = min(S, v_end - v0);
        const long long row0 = dual ? 2ll * v0 : v0;
        const int nrows = dual ? 2 * nv : nv;
        // fast path: one try; the abort flag (a shared-memory load queued behind the weight
        // loads) is read only when the slot is not full yet
        bool ok = mbar_try_wait(&full[slot], (s / ring) & 1);
        if (!ok && !*abort_flag) {
            for (uint32_t w = 0; w < FENCE_WAIT_ROUNDS && !*abort_flag; ++w)
                if (mbar_try_wait(&full[slot], (s / ring) & 1)) { ok = true; break; }
            if (!ok) {
                if (!*abort_flag) set_device_error(-5);
                *abort_flag = 1;
            }
        }
        const bool on = ok && lane_on && rs < nrows;
        float v = 0.f;
        if (on) {
            const uint32_t base = smem_sa + (uint32_t)slot * a.slot_bytes;
            const uint32_t ddelta = (uint32_t)(((uint64_t)row0 * dbr) & 15u);
            v = rg_item_dot<WT>(base + q_off, base + s_off, base + d_off + ddelta, x);
        }
        // segmented reduction: lanes of one row part inside this warp, fixed tree (deterministic)
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float t = __shfl_down_sync(0xffffffffu, v, o);
            if (lane + o <= seg_hi) v += t;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // the slot's bytes are no longer read
        if (on && head) acc[(size_t)(row0 - row_begin + rs) * MP + pidx] = v;
    }
    named_bar_sync(1, NT);  // every piece of every row is in shared memory

    // ---- epilogues, one thread per row (pair): pieces added in part, then warp order
    auto row_sum = [&](int rl) {
        const int r_s = rl % R;
        const int n = rg_row_pieces(r_s, NP, IP);
        float t = 0.f;
        for (int k = 0; k < n; ++k) t += acc[(size_t)rl * MP + k];
        return t;
    };
    float best_v = 0.f;
    int best_i = -1;
    const int nvr = v_end - v_begin;
    for (int vr = tid; vr < nvr; vr += NT) {
        if (dual) {
            rg_epilogue<EPI>(a, v_begin + vr, row_sum(2 * vr), row_sum(2 * vr + 1), best_v, best_i);
        } else {
            rg_epilogue<EPI>(a, v_begin + vr, row_sum(vr), 0.f, best_v, best_i);
        }
    }

    if (EPI == EPI_LMHEAD) {
        // thread -> warp -> CTA best; the last CTA to arrive reduces all CTAs and advances the state
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
        named_bar_sync(1, NT);
        if (tid == 0) {
            float bv = 0.f;
            int bi = -1;
            for (int w = 0; w < RG_NW; ++w)
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
                    st->err = *reinterpret_cast<volatile int*>(&g_device_error);
                }
                *a.counter = 0u;
            }
        }
    }
}

}  // namespace fence
