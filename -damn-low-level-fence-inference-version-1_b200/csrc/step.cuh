// step.cuh — the whole batch-1 token step (reference: Qwen3Model::forward,
// src/model/qwen3.cu:241-341) as ONE persistent kernel on B200.
//
// A token is ~180 dependent phases (per layer: QKV, attention, O + residual, gate/up + SwiGLU,
// down + residual; then the LM head), each only a few MB of weights. As separate kernels every
// phase pays launch, DRAM ramp-up, drain and the completion hand-off. Here the weights of ALL
// phases stream through one shared-memory ring per SM — weights never depend on activations — and
// the consumer warps run the phases in order, separated by a grid-wide phase counter.
//
//  * grid: one CTA per SM (cooperative launch: all CTAs co-resident, which the counter needs);
//    block: SK_NW = 11 consumer warps + 1 producer warp (384 threads: 168 registers each, so the
//    stage loop, the x prologue and the attention unit run without register spills; measured
//    faster than 15 consumer warps at 128 registers and than 8 at 168).
//  * producer warp (lane 0): walks every GEMV phase's rows of this CTA in order and streams them
//    (rgemv.cuh repacked layout: q, s, d slices of R rows per stage, 1-D bulk copies, no
//    multicast) into the ring; it only ever waits for free slots.
//  * consumers, per GEMV phase (the rgemv.cuh design with 352 lanes): norm weights pulled into L2
//    by the producer a ring ahead; wait for the counter; x quantised once per CTA into shared
//    memory (4 lanes per 64-value record); every stage
//    worked on by all lanes (lane <-> (row, item), x in registers, segmented shuffle reduction,
//    one shared-memory piece per (row, warp)); after the last stage one thread per row adds the
//    pieces in a fixed order and runs the fused epilogue; then the CTA counts itself done.
//  * attention phase: (KV head, context chunk) units over the CTAs, each run by 256 threads (q/k
//    RMSNorm, RoPE, KV store, q.K^T and P.V on mma.sync, online softmax over 64-position tiles);
//    a unit's first tile is loaded across the phase change, and the last unit of each KV head
//    merges its chunks.
//  * LM head: logits + argmax; the CTA that completes the step last reduces the argmax and
//    advances the device decode state (token, pos, step).
//
// Counter protocol: every CTA adds 1 after each phase and 1 after publishing its argmax, so a step
// adds (n_phases + 1) * G. A CTA takes the step's base as the counter at kernel start rounded down
// to that multiple (no CTA can be a whole step ahead within one launch); phase k may start once the
// counter reaches base + k * G. Every wait is bounded; on expiry the device error word is set and
// the CTA stops waiting (its results are then invalid, but the kernel ends).
#pragma once

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "rgemv.cuh"

namespace fence {

constexpr int SK_NW = 11;                 // consumer warps
constexpr int SK_NT = SK_NW * 32 + 32;    // + producer warp
constexpr int SK_NL = SK_NW * 32;         // consumer lanes (352)
constexpr int SK_MAX_R = 64;              // rows per stage
// x records of the step kernel: 176 bytes apart (an odd number of 16-byte chunks), so the lanes of a
// quarter-warp reading eight consecutive items' records hit eight different bank groups
constexpr uint32_t SK_XQB = 176;
constexpr uint32_t SK_BAR_SPINS = 1u << 20;
// Exchange buffer of one rank (tensor parallel): an argmax counter, one argmax (value bits |
// index << 32) per rank, then partials [2][tp_n][tp_h] (a rank's rows adjacent, so the writing
// warps store 256 contiguous bytes per row block), each a 64-bit (value bits | tag << 32)
// stored with one 8-byte access: the tag (the step's reduction number, never 0) tells a reader
// that the value is this reduction's, so no fence or counter sits between the ranks' partials.
constexpr int SK_TP_MAX = 8;
constexpr uint32_t SK_XB_ACNT = 8, SK_XB_ARG = 256, SK_XB_PART = 1024;
__host__ __device__ inline size_t sk_xb_bytes(int tp_n, int tp_h) {
    return SK_XB_PART + (size_t)2 * tp_n * tp_h * 8;
}
constexpr int kStepAttnSolo = 128;  // StepArgs::attn_solo used by the engine (a two-tile walk beats split + merge)
constexpr int SK_WAIT_ERR = -5;           // FENCE_E_DEVICE_WAIT in the device error word

enum : int { SP_GEMV = 0, SP_ATTN = 1 };
constexpr int SK_TRACE = 8;  // trace words per CTA and phase

struct __align__(16) SPhase {
    int kind;
    RGemvArgs g;      // GEMV: matrix, geometry (I, np, R, mp, rows_cta), x, epilogue targets
    int xm, epi;
    int embed;        // first phase: x = dequantised token_embd row of state->token
    const uint8_t* embd;
    float* hidden_out;
    AttnArgs at;      // attention
    // tensor parallel (StepArgs::tp_n > 1)
    int tp_red;       // row-parallel matrix: the epilogue sends its partial rows to every rank's
                      // exchange buffer (slot red_idx & 1) instead of adding the residual
    int tp_sum;       // x prologue: x = hin + the ranks' partials of reduction red_idx, summed in
                      // rank order (identical on every rank); this CTA's share of it goes to hout
    int red_idx;      // the step's reduction this phase produces (tp_red) or consumes (tp_sum)
    const float* hin;
    float* hout;
    // sparse MoE FFN (no counterpart in the reference): a layer's FFN is one gate/up phase and one
    // down phase per routed expert slot (slot 0 = the router's first choice). The gate/up phase of
    // slot 0 computes the routing in its x prologue (every CTA, identically) from the normed x;
    // the producer streams the tiles of the chosen expert (tb + local expert * estride).
    int moe;          // 0 dense; SK_MOE_GU gate/up of an expert slot; SK_MOE_DN down of an expert slot
    int moe_slot;
    int moe_seq;      // the step's routing number this phase uses (1-based: layer + 1)
    int moe_chain;    // no grid-counter wait: the phase reads nothing another CTA wrote since the last wait
    int moe_reuse_x;  // the x records of the previous phase are this phase's (gate/up of a later slot)
    int moe_last;     // down: the last slot (adds the residual / sends the partial row)
    int n_exp, n_used;
    int e_lo, e_n;    // local experts: global ids [e_lo, e_lo + e_n) (expert parallel: a rank's share)
    long long estride;       // bytes between consecutive local experts' tile sets
    const float* route_w;    // router [n_exp][H] fp32 (slot-0 gate/up phase)
    float* moe_acc;          // tensor parallel: the slots' partial rows summed before the last slot sends
    int pad_moe_[2];
};
enum : int { SK_MOE_GU = 1, SK_MOE_DN = 2 };
constexpr int SK_MOE_EMAX = 16;   // experts a router may have
constexpr int SK_MISC_ROUTE = 112; // misc floats: chosen experts [2] (int), weights [2], routing number

struct StepArgs {
    const SPhase* ph;
    int nph;
    int ring, slot_bytes;
    int attn_solo;       // contexts up to this many positions: one attention unit per KV head
    int scratch_bytes;   // union: x records (+ embedding row) / attention tile
    int acc_floats;      // reduction pieces of the largest phase
    unsigned long long* bar;
    DecodeState* state;
    float* cta_val;
    int* cta_idx;
    int* token_log;
    int token_log_cap;
    // optional trace, null = off: [G][nph][SK_TRACE] per CTA: globaltimer ns at the phase start
    // (after the counter wait), when x is quantised (GEMV) / the first unit is done (attention),
    // when the last stage is consumed, and at the end (before the count); SM cycles the consumers
    // waited for filled slots and cycles the producer waited for free slots
    unsigned long long* trace;
    // tensor parallel: tp_n ranks (one GPU each, one step kernel each), exchanging over NVLink
    // through every rank's exchange buffer xb[p] (mapped into this process): SK_XB_* layout
    int tp_n, tp_rank;
    int tp_h;            // floats per rank per reduction (the hidden size)
    int n_red;           // reductions per step (2 per layer)
    int vocab0;          // first vocabulary row of this rank's LM-head shard
    uint8_t* xb[SK_TP_MAX];
    unsigned long long* launch;  // steps this rank has finished (read at the start, +1 at the end)
    int stall_phase;     // test only: this phase's counter wait gets an unreachable target (-1 = off)
};

constexpr uint32_t SK_DESC = (sizeof(SPhase) + 15u) & ~15u;  // one phase descriptor in shared memory
static_assert(sizeof(SPhase) % 16 == 0 && alignof(SPhase) == 16, "descriptors are copied in 16-byte words");
constexpr int SK_RPRE = SK_NL;                               // prefetched residual rows per CTA

struct SKSmem {
    uint32_t scratch, acc, desc, rpre, bars, misc, total;
};
__host__ __device__ inline SKSmem sk_smem_layout(int ring, int slot_bytes, int scratch_bytes, int acc_floats) {
    auto r16 = [](uint32_t x) { return (x + 15u) & ~15u; };
    SKSmem L;
    L.scratch = (uint32_t)ring * (uint32_t)slot_bytes;
    L.acc = L.scratch + r16((uint32_t)scratch_bytes);
    L.desc = L.acc + r16(4u * (uint32_t)acc_floats);
    L.rpre = L.desc + 2u * SK_DESC;
    L.bars = L.rpre + r16(4u * SK_RPRE);
    L.misc = L.bars + r16(16u * ring);
    L.total = L.misc + 512u;
    return L;
}

__device__ __forceinline__ unsigned long long sk_ld_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long sk_ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// +v on a (possibly peer-mapped) counter, releasing this thread's earlier writes (and, after a CTA
// barrier, the CTA's) to every GPU of the system
__device__ __forceinline__ void sk_red_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Rank p's tagged partials of reduction slot buf, as mapped here: [tp_n][tp_h]
__device__ __forceinline__ unsigned long long* sk_xpart(const StepArgs& A, int p, int buf) {
    return reinterpret_cast<unsigned long long*>(A.xb[p] + SK_XB_PART) + (size_t)buf * A.tp_n * A.tp_h;
}
__device__ __forceinline__ void sk_st_sys64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long sk_ld_sys64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// The tag of reduction red of the step counted launch0 (1-based, so a zeroed buffer never matches).
__device__ __forceinline__ unsigned sk_red_tag(const StepArgs& A, unsigned long long launch0, int red) {
    return (unsigned)(launch0 * (unsigned long long)A.n_red + (unsigned long long)red) + 1u;
}
__device__ __forceinline__ unsigned long long sk_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Row range of this CTA in a GEMV phase: virtual rows (dual: gate/up pairs) and actual rows.
struct SKRows {
    int v_begin, v_end;
    long long r_begin, r_end;
};
__device__ __forceinline__ SKRows sk_rows(const RGemvArgs& g, int c, int G) {
    SKRows r;
    r.v_begin = (int)(((long long)g.Mv * c) / G);
    r.v_end = (int)(((long long)g.Mv * (c + 1)) / G);
    r.r_begin = g.dual ? 2ll * r.v_begin : r.v_begin;
    r.r_end = g.dual ? 2ll * r.v_end : r.v_end;
    return r;
}

// ---- x prologue of a GEMV phase (consumers): records of all items in shared memory.
template <int WT, int XM>
__device__ __forceinline__ void sk_quantise(const void* xsrc, const float* norm_w, float eps, int I, uint32_t xq_sa,
                                            float* misc) {
    constexpr int NT = SK_NL;
    constexpr int LPI = RG_LPI;
    constexpr int NV = RG_NV;
    constexpr bool NORM = (XM == X_NORM || XM == X_NORM_R16);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ntask = I * LPI;
    float xv[NV], wv[NV];
    const bool mine = tid < ntask;  // one register pass; further tasks re-read x below
    const int base0 = mine ? rg_task_base<WT>(tid / LPI, tid % LPI) : 0;
    rg_load_task<WT, XM>(xsrc, base0, xv);
    float rms = 1.f;
    if (NORM) {
        const float4* p = reinterpret_cast<const float4*>(norm_w + base0);
#pragma unroll
        for (int cc = 0; cc < NV / 4; ++cc) {
            const float4 f = p[cc];
            wv[4 * cc] = f.x;
            wv[4 * cc + 1] = f.y;
            wv[4 * cc + 2] = f.z;
            wv[4 * cc + 3] = f.w;
        }
        float ss = 0.f;
        if (mine) {
#pragma unroll
            for (int e = 0; e < NV; ++e) ss += xv[e] * xv[e];
        }
        for (int b = NT + tid; b < ntask; b += NT) {
            float t[NV];
            rg_load_task<WT, XM>(xsrc, rg_task_base<WT>(b / LPI, b % LPI), t);
#pragma unroll
            for (int e = 0; e < NV; ++e) ss += t[e] * t[e];
        }
        ss = warp_sum(ss);
        if (lane == 0) misc[warp] = ss;
        named_bar_sync(1, NT);
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < SK_NW; ++w) tot += misc[w];
        rms = rsqrtf(tot / (float)(I * 64) + eps);
    }
    if (warp * 32 < ntask) {  // warp-uniform (shuffles inside)
        const int item = mine ? tid / LPI : 0;
        rg_quant_store<WT, XM>(xv, wv, tid % LPI, rms, xq_sa + item * SK_XQB, mine);
    }
    for (int b0 = NT + warp * 32; b0 < ntask; b0 += NT) {
        const int idx = b0 + lane;
        const bool active = idx < ntask;
        const int item = active ? idx / LPI : 0, q = idx % LPI;
        const int base = active ? rg_task_base<WT>(item, q) : 0;
        float t[NV], tw[NV];
        rg_load_task<WT, XM>(xsrc, base, t);
        if (NORM) {
            const float4* p = reinterpret_cast<const float4*>(norm_w + base);
#pragma unroll
            for (int cc = 0; cc < NV / 4; ++cc) {
                const float4 f = p[cc];
                tw[4 * cc] = f.x;
                tw[4 * cc + 1] = f.y;
                tw[4 * cc + 2] = f.z;
                tw[4 * cc + 3] = f.w;
            }
        }
        rg_quant_store<WT, XM>(t, tw, q, rms, xq_sa + item * SK_XQB, active);
    }
    named_bar_sync(1, NT);  // records complete; misc free again
}

// Out of line: the prologue's register use stays out of the stage loop's allocation.
template <int WT>
__device__ __noinline__ void sk_quantise_xm(int xm, const void* xsrc, const float* norm_w, float eps, int I,
                                               uint32_t xq_sa, float* misc) {
    switch (xm) {
        case X_F16: sk_quantise<WT, X_F16>(xsrc, norm_w, eps, I, xq_sa, misc); break;
        case X_F32: sk_quantise<WT, X_F32>(xsrc, norm_w, eps, I, xq_sa, misc); break;
        case X_F32_R16: sk_quantise<WT, X_F32_R16>(xsrc, norm_w, eps, I, xq_sa, misc); break;
        case X_NORM: sk_quantise<WT, X_NORM>(xsrc, norm_w, eps, I, xq_sa, misc); break;
        default: sk_quantise<WT, X_NORM_R16>(xsrc, norm_w, eps, I, xq_sa, misc); break;
    }
}

// Routing of a sparse-MoE layer (consumers, every CTA the same way): r_e = W_r[e] . RMSNorm(x)
// (fp32 router weights, per-thread partial sums in a fixed order, fixed reduction tree: the same
// bits in every CTA), the n_used largest r_e (ties to the smaller expert id), weights = softmax
// over the chosen logits (= the full softmax renormalised over them). Chosen ids and weights go to
// misc[SK_MISC_ROUTE..+3], then the routing number `seq` to misc[SK_MISC_ROUTE + 4] for the
// producer warp. red: SK_NW * SK_MOE_EMAX floats of free shared memory.
__device__ __noinline__ void sk_route(const float* x, const float* nw, float eps, const float* Wr, int E, int K,
                                      int H, float* red, float* misc, int seq) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float ss = 0.f;
    for (int k = tid; k < H; k += SK_NL) {
        const float v = x[k];
        ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    named_bar_sync(1, SK_NL);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < SK_NW; ++w) tot += red[w];
    const float rms = rsqrtf(tot / (float)H + eps);
    named_bar_sync(1, SK_NL);  // red is reused below
    float p[SK_MOE_EMAX];
#pragma unroll
    for (int e = 0; e < SK_MOE_EMAX; ++e) p[e] = 0.f;
    // 16-byte loads, a group of 4 expert rows' loads issued before any use (H % 64 == 0): a few L2
    // round trips per thread instead of one per element. Groups of 4, not all rows at once: this
    // function's register footprint is what the step kernel must keep clear around the call, and
    // 16 loads in flight made it spill its own loop state.
    const int H4 = H >> 2;
    for (int k4 = tid; k4 < H4; k4 += SK_NL) {
        const float4 xv = reinterpret_cast<const float4*>(x)[k4];
        const float4 wv = reinterpret_cast<const float4*>(nw)[k4];
        const float x0 = xv.x * rms * wv.x, x1 = xv.y * rms * wv.y, x2 = xv.z * rms * wv.z, x3 = xv.w * rms * wv.w;
#pragma unroll
        for (int e0 = 0; e0 < SK_MOE_EMAX; e0 += 4) {
            if (e0 >= E) break;
            float4 wr[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e0 + e < E) wr[e] = __ldg(reinterpret_cast<const float4*>(Wr + (size_t)(e0 + e) * H) + k4);
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e0 + e < E) p[e0 + e] += wr[e].x * x0 + wr[e].y * x1 + wr[e].z * x2 + wr[e].w * x3;
        }
    }
#pragma unroll
    for (int e = 0; e < SK_MOE_EMAX; ++e) {
        if (e < E) {
            const float v = warp_sum(p[e]);
            if (lane == 0) red[warp * SK_MOE_EMAX + e] = v;
        }
    }
    named_bar_sync(1, SK_NL);
    if (tid == 0) {
        float r[SK_MOE_EMAX];
        for (int e = 0; e < E; ++e) {
            float t = 0.f;
            for (int w = 0; w < SK_NW; ++w) t += red[w * SK_MOE_EMAX + e];
            r[e] = t;
        }
        int s0 = 0, s1 = -1;
        for (int e = 1; e < E; ++e)
            if (r[e] > r[s0]) s0 = e;
        if (K > 1)
            for (int e = 0; e < E; ++e)
                if (e != s0 && (s1 < 0 || r[e] > r[s1])) s1 = e;
        float w0 = 1.f, w1 = 0.f;
        if (K > 1) {
            const float a = expf(r[s1] - r[s0]);
            w0 = 1.f / (1.f + a);
            w1 = a / (1.f + a);
        }
        int* rs = reinterpret_cast<int*>(misc + SK_MISC_ROUTE);
        rs[0] = s0;
        rs[1] = s1;
        misc[SK_MISC_ROUTE + 2] = w0;
        misc[SK_MISC_ROUTE + 3] = w1;
        __threadfence_block();
        *reinterpret_cast<volatile int*>(misc + SK_MISC_ROUTE + 4) = seq;
    }
    named_bar_sync(1, SK_NL);
}

// Bounded wait for a filled ring slot (the consumer side). Fast path: one try (the abort flag, a
// shared-memory load queued behind the other warps' weight loads, is read only when the slot is not
// full yet). Returns false when the CTA gave up (abort flag set, device error recorded).
__device__ __forceinline__ bool sk_wait_full(uint64_t* bar, uint32_t par, volatile int* abort_flag) {
    if (mbar_try_wait(bar, par)) return true;
    if (*abort_flag) return false;
    for (uint32_t w = 0; w < FENCE_WAIT_ROUNDS && !*abort_flag; ++w)
        if (mbar_try_wait(bar, par)) return true;
    if (!*abort_flag) set_device_error(SK_WAIT_ERR);
    *abort_flag = 1;
    return false;
}

// ---- the stage loop of a GEMV phase (consumers) over the CTA's tiles (row block b x K-slice j, in
// that order). Lane <-> (row rl of the block, item slot is of the slice): per tile it loads its
// item's x record (shared by the lanes of the other rows: a broadcast) and its weight record, does
// the exact integer item dot and adds it to a register accumulator; after a block's last slice a
// segmented shuffle reduction over the row's CI lanes leaves one shared-memory piece per (row,
// warp). No reduction sits between the tiles of a block. Returns the ring stages consumed. Out of
// line: the loop gets the whole register budget.
template <int WT>
__device__ __noinline__ uint32_t sk_stages(const RGemvArgs& g, const SKRows& rr, uint32_t use, int ring,
                                           int slot_bytes, uint32_t smem_sa, uint32_t xq_sa, float* acc,
                                           uint64_t* full, uint64_t* empty, volatile int* abort_flag) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int I = g.I, RB = g.RB, CI = g.CI, MP = g.mp;
    const int rows = (int)(rr.r_end - rr.r_begin);
    const int ns = (I + CI - 1) / CI, ndq = sk_ndq(CI);
    const int rl = tid / CI, is = tid - rl * CI;
    const bool lane_on = rl < RB;
    const int slot_lo = rl * CI;
    const int seg_hi = min(slot_lo + CI - 1 - warp * 32, 31);
    const bool head = lane == max(slot_lo - warp * 32, 0);
    const int pidx = warp - (slot_lo >> 5);  // this segment's piece index in its row's reduction
    const uint32_t sw = ((uint32_t)(is >> 1) & 3u) << 4;  // Q8_0 chunk position swizzle of this slot
    const uint32_t acc_sa = smem_u32(acc) + (uint32_t)(rl * MP + pidx) * 4u;
    const uint32_t ring_u = (uint32_t)ring;
    uint32_t slot = use % ring_u, par = (use / ring_u) & 1u;  // advanced incrementally below
    for (int r0 = 0; r0 < rows; r0 += RB) {
        const int rows_b = min(RB, rows - r0);
        const bool row_on = lane_on && rl < rows_b;
        float a = 0.f;
        for (int j = 0; j < ns; ++j, ++use) {
            const int items = min(CI, I - j * CI);
            uint32_t s_off, d_off;
            sk_tile_bytes(WT, rows_b, items, CI, &s_off, &d_off);
            const bool ok = sk_wait_full(&full[slot], par, abort_flag);
            if (ok && row_on && is < items) {
                const int it = j * CI + is;
                const uint32_t base = smem_sa + slot * (uint32_t)slot_bytes;
                const uint32_t rec = (uint32_t)(rl * items + is);
                RX x;
                rg_load_x<WT>(xq_sa + (uint32_t)it * SK_XQB, it, x);
                x.sw = sw;
                RWT<WT> w;
                const uint32_t dad = WT == WT_Q6K
                    ? base + d_off + (uint32_t)(rl * ndq + ((it + g.w.iph) >> 2) - ((j * CI + g.w.iph) >> 2)) * 2u
                    : base + d_off + rec * 4u;
                rg_item_load<WT>(base + rec * (uint32_t)rg_qbytes(WT), base + s_off + rec * 4u, dad, x.sw, w);
                a += rg_item_compute<WT>(w, x);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);  // the slot's bytes are no longer read
            if (++slot == ring_u) {
                slot = 0;
                par ^= 1u;
            }
        }
        // the row's CI lanes, inside this warp: fixed tree (deterministic)
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float t = __shfl_down_sync(0xffffffffu, a, o);
            if (lane + o <= seg_hi) a += t;
        }
        if (row_on && head)
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(acc_sa + (uint32_t)(r0 * MP) * 4u), "f"(a) : "memory");
    }
    return use;
}

// mma.sync m16n8k16 on KVT operands (f16 or bf16) with fp32 accumulators. Only rows 0..7 of A are
// used (at most ATTN_MAX_G = 8 query heads per KV head), so A's rows 8..15 registers are zero.
template <typename KVT>
struct SKMma;
template <>
struct SKMma<__half> {
    static __device__ __forceinline__ uint32_t pack(float x, float y) {
        const __half2 h = __floats2half2_rn(x, y);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
    static __device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
    }
};
template <>
struct SKMma<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float x, float y) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
    static __device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
    }
};

// Tiles of 64 positions one attention unit of the step kernel holds in shared memory at once: all
// of its K tiles are in flight together, and each V tile later reuses its K tile's buffer.
constexpr int SK_ATT_TILES = 4;
constexpr int SK_ATT_MAXLEN = SK_ATT_TILES * ATTN_CMAX;  // 256 positions per unit at most

// Positions per attention unit of the step kernel: up to `solo` positions one unit per KV head
// walks the whole context (no merge); beyond, the context of each KV head is spread over the CTAs
// available to it (ctas / n_kv_heads), in whole 64-position tiles, at most SK_ATT_MAXLEN per unit,
// never more chunks than the partials hold (nchunk; the engine sizes them so that nchunk units of
// SK_ATT_MAXLEN cover max_ctx).
__host__ __device__ __forceinline__ int sk_attn_clen(int seq, int nchunk, int ctas, int n_kv_heads, int solo) {
    if (seq <= solo) return (seq + ATTN_CMAX - 1) / ATTN_CMAX * ATTN_CMAX;
    const int per_head = ctas / n_kv_heads > 1 ? ctas / n_kv_heads : 1;
    int clen = (seq + per_head - 1) / per_head;
    const int cmin = (seq + nchunk - 1) / nchunk;
    if (clen < cmin) clen = cmin;
    clen = (clen + ATTN_CMAX - 1) / ATTN_CMAX * ATTN_CMAX;
    return clen < SK_ATT_MAXLEN ? clen : SK_ATT_MAXLEN;
}

// Floats per (KV head, chunk, query head) record of the step kernel's attention partials: 128
// unnormalised outputs, the max and the exp-sum, padded so that every record is 16-byte aligned.
constexpr int SK_PART_STRIDE = 132;

// Shared memory of one attention unit (sk_attn_unit's carve-up): SK_ATT_TILES K/V tile buffers,
// the scores / softmax weights [G][SK_ATT_MAXLEN] (the fp32 q [G][128] before them), q as (high,
// remainder) pairs, new k / v, norm weights, RoPE row, softmax state and a flag.
// Tile rows are padded to 136 elements (272 bytes): the eight rows an mma fragment or an ldmatrix
// reads sit 4 banks apart, so the row-contiguous layout the bulk copies write is conflict-free.
constexpr int SK_ATT_RSTR = 136;
constexpr int SK_ATT_TILE_BYTES = ATTN_CMAX * SK_ATT_RSTR * 2;
constexpr int sk_attn_scratch_bytes() {
    return SK_ATT_TILES * SK_ATT_TILE_BYTES + ATTN_MAX_G * SK_ATT_MAXLEN * 4 + 2 * ATTN_MAX_G * 64 * 4 +
           4 * 128 * 4 + 64 * 8 + 3 * ATTN_MAX_G * 4 + 16;
}
// Partial records the merging unit stages at a time (in the tile buffers and scores)
constexpr int SK_MERGE_RECS = (SK_ATT_TILES * SK_ATT_TILE_BYTES + ATTN_MAX_G * SK_ATT_MAXLEN * 4) / (SK_PART_STRIDE * 4);
static_assert(SK_MERGE_RECS >= ATTN_MAX_G, "merge staging holds at least one chunk");

// Rows [ts, te) of a K or V head into a tile buffer: ONE 1-D bulk copy (TMA, no multicast) of the
// rows as they lie in the cache (rows of SK_ATT_RSTR elements, the engine's padded layout),
// completing on the tile's mbarrier; issued by one thread. The row at pos may arrive stale or new:
// the unit writes it into the tile itself after the copy has landed.
template <typename KVT>
__device__ __forceinline__ void sk_attn_rows(KVT* dst, const KVT* src, long long stride_t, int ts, int te, uint64_t* bar) {
    const uint32_t bytes = (uint32_t)(te - ts) * (uint32_t)(SK_ATT_RSTR * sizeof(KVT));
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(dst, src + (long long)ts * stride_t, bytes, bar);
}

// Tile buffers of a chunk of T tiles: K tile i in buffer i; V tile i in buffer i + SK_ATT_TILES / 2
// when the chunk has at most SK_ATT_TILES / 2 tiles (its K and V then load together), else in
// buffer i once the scores of K tile i are done.
__device__ __forceinline__ int sk_attn_vbuf(int T, int i) { return T <= SK_ATT_TILES / 2 ? i + SK_ATT_TILES / 2 : i; }

// Issues the tiles of attention unit (h, c) that can load before its scores: the K tiles, and the V
// tiles when they have buffers of their own (thread 0). Run at the end of the phase before attention,
// so they load across the phase change; the cache rows before pos are not written by that phase and
// the row at pos is replaced by the unit. Returns the tile count T.
template <typename KVT>
__device__ __forceinline__ int sk_attn_issue_early(const AttnArgs& a, int h, int c, int clen, int pos, uint8_t* sm,
                                                   uint64_t* abar) {
    constexpr int TILE = ATTN_CMAX;
    KVT* kt = reinterpret_cast<KVT*>(sm);
    const int t0 = c * clen, t1 = min(t0 + clen, pos + 1);
    const int T = (t1 - t0 + TILE - 1) / TILE;
    const KVT* kb = reinterpret_cast<const KVT*>(a.kc) + (long long)h * a.stride_h;
    const KVT* vb = reinterpret_cast<const KVT*>(a.vc) + (long long)h * a.stride_h;
    if (threadIdx.x == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // after the generic use of the scratch
        for (int ts = t0, i = 0; ts < t1; ts += TILE, ++i) {
            sk_attn_rows<KVT>(kt + i * TILE * SK_ATT_RSTR, kb, a.stride_t, ts, min(ts + TILE, t1), &abar[i]);
            if (T <= SK_ATT_TILES / 2) {
                const int vbi = sk_attn_vbuf(T, i);
                sk_attn_rows<KVT>(kt + vbi * TILE * SK_ATT_RSTR, vb, a.stride_t, ts, min(ts + TILE, t1), &abar[vbi]);
            }
        }
    }
    return T;
}

// One attention unit of the step kernel (KV head h, context chunk c of clen <= SK_ATT_MAXLEN
// positions), run by threads 0..ATTN_THREADS-1 (named barrier 2). The semantics are attention.cuh's
// fused chunk (q/k RMSNorm, NeoX RoPE, KV store of the new row, softmax(q.K^T / sqrt(hd)) V in fp32,
// reference src/kernels/ops.cuh:66-177,320-443); the schedule is cut for latency:
//  * every K tile of the chunk is in flight at once (issued across the phase change when `pre`),
//    together with the small inputs (q, new k/v, norm weights, RoPE row);
//  * pass 1, every position of the chunk at once: q.K^T on the tensor cores (mma.sync m16n8k16,
//    fp32 accumulators, up to four independent chains per warp; query heads = rows of A; the fp32
//    q is split into a KVT high part and a KVT remainder, two products summed, so it keeps ~22
//    (f16) / ~16 (bf16) bits while K enters exactly as cached); the tile buffers then take the V
//    rows, which load during the softmax;
//  * the chunk's exact softmax (max, exp, sum over all its positions, a warp per head);
//  * pass 2: P.V on the tensor cores over the whole chunk, P split the same way as q;
//  * the unit writes its chunk's unnormalised output, max and exp-sum to the partials; the last
//    unit of the KV head to arrive (arrival counter) merges the head's chunks, so attention is a
//    single phase; for a single chunk the unit writes the normalised output itself.
template <typename KVT>
__device__ __noinline__ void sk_attn_unit(const AttnArgs& a, int h, int c, int clen, int n_active, int pos,
                                          uint8_t* sm, bool pre, uint64_t* abar, uint32_t& apar,
                                          volatile int* abort_flag, unsigned long long* tr) {
    using C = KVConv<KVT>;
    using M = SKMma<KVT>;
    constexpr int HD = 128;
    constexpr int NT = ATTN_THREADS, NW = NT / 32, TILE = ATTN_CMAX, ML = SK_ATT_MAXLEN;
    static_assert(TILE == 64 && NT == 256 && NW == 8 && ATTN_MAX_G <= 8, "unit geometry");
    constexpr int RSTR = SK_ATT_RSTR;
    KVT* kv = reinterpret_cast<KVT*>(sm);                                      // [SK_ATT_TILES][TILE][RSTR]
    float* ss = reinterpret_cast<float*>(sm + SK_ATT_TILES * SK_ATT_TILE_BYTES);  // [G][ML] scores, then P
    float* sq = ss;                                                             // [G][HD] fp32 q (before the scores)
    uint32_t* sqa = reinterpret_cast<uint32_t*>(ss + ATTN_MAX_G * ML);          // [2][G][HD/2] q high / remainder
    float* skn = reinterpret_cast<float*>(sqa + 2 * ATTN_MAX_G * (HD / 2));     // [HD] new k (rotated, cache-rounded)
    float* svn = skn + HD;                                                      // [HD] new v
    float* sqw = svn + HD;
    float* skw = sqw + HD;
    float2* srope = reinterpret_cast<float2*>(skw + HD);                        // [HD/2]
    float* smax = reinterpret_cast<float*>(srope + HD / 2);
    float* ssum = smax + ATTN_MAX_G;
    float* sinv = ssum + ATTN_MAX_G;
    int* flag = reinterpret_cast<int*>(sinv + ATTN_MAX_G);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.n_q_heads / a.n_kv_heads;
    const int t0 = c * clen, t1 = min(t0 + clen, pos + 1);
    const int n = t1 - t0, T = (n + TILE - 1) / TILE;
    const bool owns_new = pos >= t0 && pos < t1;
    const KVT* kb = reinterpret_cast<const KVT*>(a.kc) + (long long)h * a.stride_h;
    const KVT* vb = reinterpret_cast<const KVT*>(a.vc) + (long long)h * a.stride_h;
    auto tile = [&](int i) { return kv + i * TILE * RSTR; };
    auto vtile = [&](int i) { return tile(sk_attn_vbuf(T, i)); };
    // a buffer's mbarrier completes once per fill; apar (the same in every unit thread) holds the
    // parity of each buffer's next completion
    auto wait_buf = [&](int b) {
        if (!mbar_wait(&abar[b], (apar >> b) & 1u)) *abort_flag = 1;
        apar ^= 1u << b;
    };
    // the new row (cache-rounded floats) into its tile slot, when pos lies in tile i
    auto put_new = [&](int i, int buf, const float* row) {  // tile i held in buffer buf
        const int r = pos - (t0 + i * TILE);
        if (r < 0 || r >= TILE || tid >= HD) return;
        const int d = tid;
        tile(buf)[r * RSTR + d] = C::from(row[d]);
    };
    // rows [m, round16(m)) of a partial V tile: zero, so that P.V's last k-step reads finite values
    auto zero_tail = [&](int i, int m) {
        const int m16 = (m + 15) & ~15;
        for (int idx = tid; idx < (m16 - m) * 16; idx += NT) {
            const int r = m + (idx >> 4), ch = idx & 15;
            *reinterpret_cast<uint4*>(tile(i) + r * RSTR + ch * 8) = make_uint4(0u, 0u, 0u, 0u);
        }
    };

    // ---- small inputs (one group); without `pre` the K tiles follow, one group each
    const int qh0 = h * G;
    for (int i = tid; i < G * (HD / 4); i += NT) cp_async16(sq + 4 * i, a.q + (long long)qh0 * HD + 4 * i);
    if (tid < HD / 4) {
        const int i = tid;
        if (owns_new) {
            cp_async16(skn + 4 * i, a.k_new + (long long)h * HD + 4 * i);
            cp_async16(svn + 4 * i, a.v_new + (long long)h * HD + 4 * i);
        }
        if (a.q_norm_w) cp_async16(sqw + 4 * i, a.q_norm_w + 4 * i);
        if (a.k_norm_w) cp_async16(skw + 4 * i, a.k_norm_w + 4 * i);
        // RoPE row: HD/2 (cos, sin) pairs = HD/4 chunks of 16 bytes
        cp_async16(reinterpret_cast<float*>(srope) + 4 * i,
                   reinterpret_cast<const float*>(a.rope + (long long)pos * (HD / 2)) + 4 * i);
    }
    cp_async_commit();
    if (!pre) sk_attn_issue_early<KVT>(a, h, c, clen, pos, sm, abar);  // else issued at the previous phase's end
    cp_async_wait_group<0>();  // the small inputs
    named_bar_sync(2, NT);
    // ---- q/k RMSNorm (w * x * rms) and NeoX rotation, a warp per head; the new K/V row
    for (int g = warp; g < G + (owns_new ? 1 : 0); g += NW) {
        const float* v = (g < G) ? sq + g * HD : skn;
        const float* nw = (g < G) ? a.q_norm_w : a.k_norm_w;
        const float* w = (g < G) ? sqw : skw;
        float x4[HD / 32];
#pragma unroll
        for (int i = 0; i < HD / 32; ++i) x4[i] = v[lane + 32 * i];
        if (nw) {
            float s2 = 0.f;
#pragma unroll
            for (int i = 0; i < HD / 32; ++i) s2 += x4[i] * x4[i];
            s2 = warp_sum(s2);
            const float r = rsqrtf(s2 / (float)HD + a.eps);
#pragma unroll
            for (int i = 0; i < HD / 32; ++i) x4[i] = w[lane + 32 * i] * x4[i] * r;
        }
        // rotation pairs (j, j + 64): lane holds j = lane, lane + 32 and their partners
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float2 t = srope[lane + 32 * i];
            const float x0 = x4[i], x1 = x4[i + 2];
            x4[i] = x0 * t.x - x1 * t.y;
            x4[i + 2] = x0 * t.y + x1 * t.x;
        }
        __syncwarp();
        if (g < G) {  // q as (high, remainder) pairs: element pair (2j, 2j + 1) in word j
#pragma unroll
            for (int i = 0; i < HD / 32; ++i) {
                const float hi = M::round(x4[i]);
                const float lo = x4[i] - hi;
                const float hi_n = __shfl_down_sync(0xffffffffu, hi, 1);
                const float lo_n = __shfl_down_sync(0xffffffffu, lo, 1);
                if ((lane & 1) == 0) {
                    const int j = (lane + 32 * i) >> 1;
                    sqa[g * (HD / 2) + j] = M::pack(hi, hi_n);
                    sqa[(ATTN_MAX_G + g) * (HD / 2) + j] = M::pack(lo, lo_n);
                }
            }
        } else {  // round to the cache type and store the row (the tiles take it from skn / svn)
            KVT* kw = reinterpret_cast<KVT*>(a.kc_w) + (long long)h * a.stride_h + (long long)pos * a.stride_t;
            KVT* vw = reinterpret_cast<KVT*>(a.vc_w) + (long long)h * a.stride_h + (long long)pos * a.stride_t;
#pragma unroll
            for (int i = 0; i < HD / 32; ++i) {
                const int d = lane + 32 * i;
                const KVT kq = C::from(x4[i]);
                kw[d] = kq;
                vw[d] = C::from(svn[d]);
                skn[d] = C::to(kq);
            }
        }
    }
    named_bar_sync(2, NT);  // sq is dead: ss takes the scores from here on

    const float scale = 1.0f / sqrtf((float)HD);
    const int gr = lane >> 2, q4 = lane & 3;  // fragment row (query head) and column pair
    const bool live = gr < G;
    // ---- pass 1: scores of every position of the chunk at once: warp w takes the 8-position groups
    //      w, w + 8, w + 16, w + 24 (group p: tile p / 8, rows 8 (p % 8) ..), independent mma chains
    for (int i = 0; i < T; ++i) wait_buf(i);  // every K tile
    for (int i = 0; i < T; ++i) put_new(i, i, skn);
    named_bar_sync(2, NT);
    if (tr && tid == 0) tr[4] = sk_ns();  // trace: inputs ready, K tiles landed
    {
        constexpr int GPW = SK_ATT_TILES;  // position groups per warp
        float dh[GPW][4], dl[GPW][4];
#pragma unroll
        for (int j = 0; j < GPW; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) dh[j][e] = dl[j][e] = 0.f;
        const uint32_t* qa = sqa + gr * (HD / 2);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t ah0 = live ? qa[8 * ks + q4] : 0u, ah2 = live ? qa[8 * ks + 4 + q4] : 0u;
            const uint32_t al0 = live ? qa[ATTN_MAX_G * (HD / 2) + 8 * ks + q4] : 0u;
            const uint32_t al2 = live ? qa[ATTN_MAX_G * (HD / 2) + 8 * ks + 4 + q4] : 0u;
#pragma unroll
            for (int j = 0; j < GPW; ++j) {
                const int p = warp + NW * j;  // position group
                if (8 * p >= n) continue;     // warp-uniform
                const int r = 8 * (p & 7) + gr;
                const uint32_t* krow = reinterpret_cast<const uint32_t*>(tile(p >> 3) + r * RSTR);
                const uint32_t b0 = krow[8 * ks + q4];
                const uint32_t b1 = krow[8 * ks + 4 + q4];
                M::mma(dh[j], ah0, ah2, b0, b1);
                M::mma(dl[j], al0, al2, b0, b1);
            }
        }
        if (live) {  // d[0], d[1]: head gr, chunk positions 8 p + 2 q4 + {0, 1}
#pragma unroll
            for (int j = 0; j < GPW; ++j) {
                const int col = 8 * (warp + NW * j) + 2 * q4;
                if (col < n) ss[gr * ML + col] = (dh[j][0] + dl[j][0]) * scale;
                if (col + 1 < n) ss[gr * ML + col + 1] = (dh[j][1] + dl[j][1]) * scale;
            }
        }
    }
    named_bar_sync(2, NT);  // the K tiles are dead: long chunks load their V rows into those buffers
    if (tid == 0 && T > SK_ATT_TILES / 2) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // after the generic reads of the K rows
        for (int i = 0; i < T; ++i)
            sk_attn_rows<KVT>(tile(i), vb, a.stride_t, t0 + i * TILE, min(t0 + (i + 1) * TILE, t1), &abar[i]);
    }
    if (tr && tid == 0) tr[5] = sk_ns();  // trace: scores done
    // ---- the chunk's softmax, a warp per head: max, exp, sum; P (zero beyond n) back into ss
    for (int g = warp; g < G; g += NW) {
        float* sr = ss + g * ML;
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sr[j]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < T * TILE; j += 32) {
            const float e = j < n ? expf(sr[j] - m) : 0.f;
            sr[j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            smax[g] = m;
            ssum[g] = l;
        }
    }
    // ---- pass 2: P.V over the chunk; warp w -> dims 16w .. 16w + 15 (two n-tiles), k-steps of 16 positions
    for (int i = 0; i < T; ++i) wait_buf(sk_attn_vbuf(T, i));  // every V tile
    for (int i = 0; i < T; ++i) put_new(i, sk_attn_vbuf(T, i), svn);
    if (n < T * TILE) zero_tail(sk_attn_vbuf(T, T - 1), n - (T - 1) * TILE);
    named_bar_sync(2, NT);
    if (tr && tid == 0) tr[6] = sk_ns();  // trace: V tiles landed
    float oh[2][2][4] = {}, ol[2][2][4] = {};  // [k-step parity][n-tile j]: dims 16 warp + 8 j + 2 q4 + {0, 1}
    // ldmatrix.trans addresses: lane -> row (lane & 7) + 8 (bit 3) of tile rows 16 ks.., chunk 2w + (bit 4)
    const int lr = (lane & 7) + ((lane >> 3) & 1) * 8, lch = 2 * warp + (lane >> 4);
    const float* prow = ss + gr * ML;
    for (int kp = 0; kp < (n + 15) / 16; ++kp) {  // k-step kp: chunk positions 16 kp ..
        const int r = 16 * (kp & 3) + lr;
        const uint32_t addr = smem_u32(vtile(kp >> 2) + r * RSTR + lch * 8);
        uint32_t b[4];
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                     : "r"(addr));
        const float2 p0 = live ? *reinterpret_cast<const float2*>(prow + 16 * kp + 2 * q4) : make_float2(0.f, 0.f);
        const float2 p2 = live ? *reinterpret_cast<const float2*>(prow + 16 * kp + 8 + 2 * q4) : make_float2(0.f, 0.f);
        const float h0x = M::round(p0.x), h0y = M::round(p0.y), h2x = M::round(p2.x), h2y = M::round(p2.y);
        const uint32_t ah0 = M::pack(h0x, h0y), ah2 = M::pack(h2x, h2y);
        const uint32_t al0 = M::pack(p0.x - h0x, p0.y - h0y), al2 = M::pack(p2.x - h2x, p2.y - h2y);
        const int e = kp & 1;  // two accumulator sets: half the dependent chain length
        M::mma(oh[e][0], ah0, ah2, b[0], b[1]);
        M::mma(ol[e][0], al0, al2, b[0], b[1]);
        M::mma(oh[e][1], ah0, ah2, b[2], b[3]);
        M::mma(ol[e][1], al0, al2, b[2], b[3]);
    }
    // ---- output (single chunk) or this chunk's partials: head gr, dims 16 warp + 8 j + 2 q4 + {0, 1}
    float* pbase = a.part + (((long long)h * a.nchunk + c) * G) * SK_PART_STRIDE;
    if (gr < G) {
        const float inv = n_active == 1 ? 1.0f / ssum[gr] : 1.0f;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int d = 16 * warp + 8 * j + 2 * q4;
            const float2 o = make_float2(((oh[0][j][0] + ol[0][j][0]) + (oh[1][j][0] + ol[1][j][0])) * inv,
                                         ((oh[0][j][1] + ol[0][j][1]) + (oh[1][j][1] + ol[1][j][1])) * inv);
            if (n_active == 1) *reinterpret_cast<float2*>(a.out + (long long)(qh0 + gr) * HD + d) = o;
            else *reinterpret_cast<float2*>(pbase + gr * SK_PART_STRIDE + d) = o;
        }
    }
    if (tr && tid == 0) tr[7] = sk_ns();  // trace: P.V done, output / partial written
    if (n_active == 1) return;  // (the caller's barrier orders the next unit's reuse of the buffers)
    if (tid < G) *reinterpret_cast<float2*>(pbase + tid * SK_PART_STRIDE + HD) = make_float2(smax[tid], ssum[tid]);
    // ---- the last unit of KV head h to arrive merges the head's chunks: output (query head
    //      qh0 + g, dim d) = sum_c o_c e^(m_c - M) / sum_c l_c e^(m_c - M), the weights e^(m_c - M)
    //      computed once per (head, chunk), chunks in order (deterministic whichever unit merges;
    //      more chunks than one staging batch holds rescale per batch). The arrival is one
    //      acq_rel atomic after the CTA barrier (cumulative release of the unit's partials); the
    //      last unit stages the head's partial records in shared memory with one batch of async
    //      copies per SK_MERGE_RECS records.
    named_bar_sync(2, NT);
    if (tid == 0) {
        unsigned old;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.counter + h) : "memory");
        *flag = old == (unsigned)(n_active - 1);
    }
    named_bar_sync(2, NT);
    if (!*flag) return;
    constexpr int RS = SK_PART_STRIDE, NO = ATTN_MAX_G * HD / NT;  // outputs per thread (<= 4)
    float* sp = reinterpret_cast<float*>(sm);                     // [batch][G][RS] staged records
    float* sw = reinterpret_cast<float*>(sqa);                    // [G][per_batch] chunk weights
    const float* hb = a.part + (long long)h * a.nchunk * G * RS;
    const int per_batch = SK_MERGE_RECS / G;
    float Ox[NO];
#pragma unroll
    for (int j = 0; j < NO; ++j) Ox[j] = 0.f;
    if (tid < G) {
        smax[tid] = -INFINITY;  // running max and exp-sum of head tid (this unit's own were stored)
        ssum[tid] = 0.f;
    }
    for (int cb = 0; cb < n_active; cb += per_batch) {
        const int nb = min(per_batch, n_active - cb);
        const int n16 = nb * G * (RS / 4);  // 16-byte pieces of nb chunks' records
        const float* src = hb + (long long)cb * G * RS;
        for (int i = tid; i < n16; i += NT) cp_async16(sp + 4 * i, src + 4 * i);
        cp_async_commit();
        cp_async_wait_group<0>();
        named_bar_sync(2, NT);
        if (tid < G) {  // head g = tid: the batch's chunk weights e^(m_c - M) and the new running max / sum
            const int g = tid;
            float mb = smax[g];
            for (int cc = 0; cc < nb; ++cc) mb = fmaxf(mb, sp[(cc * G + g) * RS + HD]);
            const float f = smax[g] == -INFINITY ? 0.f : expf(smax[g] - mb);
            float l = ssum[g] * f;
            for (int cc = 0; cc < nb; ++cc) {
                const float w = expf(sp[(cc * G + g) * RS + HD] - mb);
                sw[g * per_batch + cc] = w;
                l += sp[(cc * G + g) * RS + HD + 1] * w;
            }
            smax[g] = mb;
            ssum[g] = l;
            sinv[g] = f;  // rescale of the outputs accumulated over earlier batches
        }
        named_bar_sync(2, NT);
#pragma unroll
        for (int j = 0; j < NO; ++j) {
            const int i = tid + j * NT, g = i / HD, d = i - g * HD;
            if (g < G) {
                float o = Ox[j] * sinv[g];
                for (int cc = 0; cc < nb; ++cc) o += sp[(cc * G + g) * RS + d] * sw[g * per_batch + cc];
                Ox[j] = o;
            }
        }
        named_bar_sync(2, NT);  // the next batch overwrites the staging area and the weights
    }
#pragma unroll
    for (int j = 0; j < NO; ++j) {
        const int i = tid + j * NT, g = i / HD;
        if (g < G) a.out[(long long)qh0 * HD + i] = Ox[j] / ssum[g];
    }
    if (tid == 0) a.counter[h] = 0u;  // every unit of head h has arrived: zero for the next layer
}

// x of a phase after a tensor-parallel reduction: hbuf[i] = hin[i] + sum over ranks (rank order)
// of the tagged partials of row i; rows [h0, h1) also to hout (this CTA's share of the residual
// stream). A pass reads every row with no load depending on another (four rows of a thread in
// flight together, each rank's rows coalesced across the warp); passes repeat, bounded, until
// every tag matched.
template <int N>
__device__ __forceinline__ bool sk_tp_gather(const float* hin, float* hout, const unsigned long long* parts,
                                             unsigned tag, float* hbuf, int H, int h0, int h1) {
    for (uint32_t pass = 0; pass < SK_BAR_SPINS; ++pass) {
        bool bad = false;
#pragma unroll 4
        for (int i = (int)threadIdx.x; i < H; i += SK_NL) {
            float v = __ldcg(hin + i);
#pragma unroll
            for (int p = 0; p < N; ++p) {
                const unsigned long long w = sk_ld_sys64(parts + (size_t)p * H + i);
                bad |= (unsigned)(w >> 32) != tag;
                v += __uint_as_float((unsigned)w);
            }
            hbuf[i] = v;
            if (i >= h0 && i < h1) hout[i] = v;  // the residual stream, for the next reduction
        }
        if (!bad) return true;
    }
    return false;
}

// Epilogues of a GEMV phase, one consumer thread per virtual row; rpre holds the residual rows
// prefetched at the phase start (rows up to SK_RPRE).
template <bool TP>
__device__ __forceinline__ void sk_epilogues(const RGemvArgs& g, int epi, const SKRows& rr, const float* acc,
                                             const float* rpre, float& best_v, int& best_i, const StepArgs& A,
                                             const SPhase& ph, unsigned tag, bool moe_owned, float moe_w) {
    const int LP = g.CI, R = g.RB, MP = g.mp;
    auto row_sum = [&](int rl) {
        const int n = rg_part_pieces(rl % R, 0, 1, LP);
        float t = 0.f;
        for (int k = 0; k < n; ++k) t += acc[(size_t)rl * MP + k];
        return t;
    };
    const int nvr = rr.v_end - rr.v_begin;
    if (ph.moe == SK_MOE_DN) {
        // routed expert slot: its rows scaled by the slot's routing weight (0 when this rank holds
        // none of the expert: expert parallel); one GPU: added to the residual stream slot by slot;
        // tensor parallel: summed over the slots here, the last slot sends the partial rows
        const float scale = moe_owned ? moe_w : 0.f;
        for (int vr = threadIdx.x; vr < nvr; vr += SK_NL) {
            const int row = rr.v_begin + vr;
            const float v = moe_owned ? row_sum(vr) * scale : 0.f;
            if (!TP) {
                g.resid[row] = v + (vr < SK_RPRE ? rpre[vr] : g.resid[row]);
            } else {
                const float t = ph.moe_slot > 0 ? v + ph.moe_acc[row] : v;
                if (!ph.moe_last) {
                    ph.moe_acc[row] = t;
                } else {
                    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(t);
                    for (int p = 0; p < A.tp_n; ++p)
                        sk_st_sys64(sk_xpart(A, p, ph.red_idx & 1) + (size_t)A.tp_rank * A.tp_h + row, w);
                }
            }
        }
        return;
    }
    for (int vr = threadIdx.x; vr < nvr; vr += SK_NL) {
        const int row = rr.v_begin + vr;
        if (epi == EPI_SWIGLU) {
            const float o = silu_mul(row_sum(2 * vr), row_sum(2 * vr + 1));
            if (g.act_f16) reinterpret_cast<__half*>(g.act)[row] = __float2half_rn(o);
            else reinterpret_cast<float*>(g.act)[row] = o;
        } else {
            const float sum = row_sum(vr);
            if (epi == EPI_STORE) {
                g.y[row] = g.bias ? sum + g.bias[row] : sum;
            } else if (TP && epi == EPI_RESID && ph.tp_red) {  // tagged partial row -> every rank (NVLink stores)
                const unsigned long long v = ((unsigned long long)tag << 32) | __float_as_uint(sum);
                for (int p = 0; p < A.tp_n; ++p) sk_st_sys64(sk_xpart(A, p, ph.red_idx & 1) + (size_t)A.tp_rank * A.tp_h + row, v);
            } else if (epi == EPI_RESID) {
                g.resid[row] = sum + (vr < SK_RPRE ? rpre[vr] : g.resid[row]);
            } else {
                g.logits[row] = sum;
                if (argmax_better(sum, row, best_v, best_i)) {
                    best_v = sum;
                    best_i = row;
                }
            }
        }
    }
}

// TP: tensor-parallel build (StepArgs::tp_n > 1); the single-GPU build carries none of its code.
template <typename KVT, bool TP>
__global__ void __launch_bounds__(SK_NT, 1) step_kernel(const __grid_constant__ StepArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NT = SK_NL;
    const bool is_producer = tid >= NT;
    const int G = gridDim.x, c = blockIdx.x;
    const int ring = A.ring, NPH = A.nph;
    const SKSmem SL = sk_smem_layout(ring, A.slot_bytes, A.scratch_bytes, A.acc_floats);
    const uint32_t smem_sa = smem_u32(smem);
    uint8_t* scratch = smem + SL.scratch;
    const uint32_t xq_sa = smem_sa + SL.scratch;
    float* acc = reinterpret_cast<float*>(smem + SL.acc);
    uint8_t* desc = smem + SL.desc;  // [2] phase descriptors: phase k in buffer k & 1
    float* rpre = reinterpret_cast<float*>(smem + SL.rpre);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL.bars);
    uint64_t* empty = full + ring;
    float* misc = reinterpret_cast<float*>(smem + SL.misc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 32);
    float* warp_best_v = misc + 40;
    int* warp_best_i = reinterpret_cast<int*>(misc + 72);
    uint64_t* dbar = reinterpret_cast<uint64_t*>(misc + 96);  // [2] descriptor copies (phase k: k & 1)
    uint64_t* abar = reinterpret_cast<uint64_t*>(misc + 104); // [SK_ATT_TILES] attention tile buffers

    if (tid == 0) {
        for (int s = 0; s < ring; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], SK_NW);
        }
        mbar_init(&dbar[0], 1);
        mbar_init(&dbar[1], 1);
        for (int i = 0; i < SK_ATT_TILES; ++i) mbar_init(&abar[i], 1);
        *abort_flag = 0;
        *reinterpret_cast<volatile int*>(misc + SK_MISC_ROUTE + 4) = 0;  // no routing yet in this step
        fence_barrier_init();
    }
    __syncthreads();
    const unsigned long long per_step = (unsigned long long)(NPH + 1) * (unsigned long long)G;
    const unsigned long long base = (sk_ld_acquire(A.bar) / per_step) * per_step;

    if (is_producer) {
        // ================= producer (lane 0): stream every GEMV phase's rows of this CTA
        if (lane == 0) {
            uint32_t use = 0;
            for (int k = 0; k < NPH && !*abort_flag; ++k) {
                const SPhase& ph = A.ph[k];
                if (ph.kind == SP_ATTN) {
                    // the next MoE routing's router weights into L2 (every CTA reads all of them)
                    for (int k2 = k + 1; k2 < NPH && k2 <= k + 3; ++k2) {
                        const SPhase& nx = A.ph[k2];
                        if (nx.moe == SK_MOE_GU && nx.moe_slot == 0 && c < 4) {
                            const uint32_t rb = (uint32_t)nx.n_exp * (uint32_t)nx.g.I * 256u;
                            for (uint32_t o = (uint32_t)c * 32768u; o < rb; o += 4u * 32768u)
                                bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(nx.route_w) + o, min(32768u, rb - o));
                        }
                    }
                    // (the attention phase's K/V rows are not pulled into L2 here: on config 2 at 4000
                    // positions that prefetch competed with the QKV phase's weights and made the step
                    // 0.9 % slower; the units' own tile copies, issued at the QKV phase's end, read them)
                }
                if (ph.kind != SP_GEMV) continue;
                const RGemvArgs& g = ph.g;
                // the phase's norm weights are read by every CTA in its x prologue: into L2 now,
                // a ring's depth ahead (they are otherwise evicted by the weight stream)
                if (g.norm_w && c < 8) bulk_prefetch_l2(g.norm_w, (uint32_t)g.I * 256u);
                const SKRows rr = sk_rows(g, c, G);
                const int rows = (int)(rr.r_end - rr.r_begin), I = g.I, RB = g.RB, CI = g.CI;
                const uint8_t* src = g.tb + g.tcta[c];  // this CTA's tiles, in (row block, K-slice) order
                if (ph.moe) {
                    // the routed expert of this slot: wait (bounded) for this CTA's routing of the layer
                    volatile int* rseq = reinterpret_cast<volatile int*>(misc + SK_MISC_ROUTE + 4);
                    bool ok = *rseq >= ph.moe_seq;
                    for (uint32_t it = 0; !ok && it < FENCE_WAIT_ROUNDS && !*abort_flag; ++it) {
                        __nanosleep(32);
                        ok = *rseq >= ph.moe_seq;
                    }
                    if (!ok) {
                        if (!*abort_flag) set_device_error(SK_WAIT_ERR);
                        *abort_flag = 1;
                        break;
                    }
                    __threadfence_block();
                    const int e = reinterpret_cast<volatile int*>(misc + SK_MISC_ROUTE)[ph.moe_slot] - ph.e_lo;
                    if (e < 0 || e >= ph.e_n) continue;  // expert parallel: another rank's expert
                    src += (size_t)e * (size_t)ph.estride;
                }
                unsigned long long pwait = 0;
                bool stop = false;
                for (int r0 = 0; r0 < rows && !stop; r0 += RB) {
                    const int rows_b = min(RB, rows - r0);
                    for (int j = 0; j * CI < I; ++j, ++use) {
                        const int slot = use % ring;
                        if (use >= (uint32_t)ring) {
                            const long long w0 = A.trace ? clock64() : 0;
                            bool ok = mbar_try_wait(&empty[slot], ((use / ring) - 1) & 1);
                            for (uint32_t it = 0; !ok && it < FENCE_WAIT_ROUNDS && !*abort_flag; ++it)
                                if (mbar_try_wait(&empty[slot], ((use / ring) - 1) & 1)) { ok = true; break; }
                            if (A.trace) pwait += (unsigned long long)(clock64() - w0);
                            if (!ok) {
                                if (!*abort_flag) set_device_error(SK_WAIT_ERR);
                                *abort_flag = 1;
                                stop = true;
                                break;
                            }
                        }
                        const uint32_t bytes = sk_tile_bytes(g.wt, rows_b, min(CI, I - j * CI), CI);
                        mbar_arrive_expect_tx(&full[slot], bytes);
                        bulk_g2s(smem + (size_t)slot * A.slot_bytes, src, bytes, &full[slot]);
                        src += bytes;
                    }
                }
                if (A.trace) A.trace[((size_t)c * NPH + k) * SK_TRACE + 5] = pwait;
                if (stop) break;
            }
            // leave no bulk copy in flight (immediately true on the normal path, where the
            // consumers waited for every stage); bounded
            const uint32_t first = use > (uint32_t)ring ? use - ring : 0u;
            for (uint32_t u = first; u < use; ++u)
                for (uint32_t it = 0; it < FENCE_WAIT_ROUNDS; ++it)
                    if (mbar_try_wait(&full[u % ring], (u / ring) & 1)) break;
        }
        return;
    }

    // ================= consumers
    uint32_t use = 0;
    float best_v = 0.f;
    int best_i = -1;
    const int pos = A.state->pos;  // fixed for the whole step (advanced only at its very end)
    const unsigned long long launch0 = TP ? *reinterpret_cast<volatile unsigned long long*>(A.launch) : 0ull;
    // descriptor k arrives on dbar[k & 1], completing that barrier's phase k >> 1
    if (tid == 0) {
        mbar_arrive_expect_tx(&dbar[0], SK_DESC);
        bulk_g2s(desc, &A.ph[0], SK_DESC, &dbar[0]);
    }
    int attn_pre = 0;  // tiles of this CTA's first attention unit issued at the end of the phase before
    uint32_t apar = 0;  // attention tile buffers: parity of each one's next mbarrier completion
    for (int k = 0; k < NPH; ++k) {
        // the next phase's descriptor: one bulk copy into the buffer phase k - 1 used (every consumer
        // thread is past that phase's end barrier), landing while this phase runs
        if (tid == 0 && k + 1 < NPH) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(&dbar[(k + 1) & 1], SK_DESC);
            bulk_g2s(desc + ((k + 1) & 1) * SK_DESC, &A.ph[k + 1], SK_DESC, &dbar[(k + 1) & 1]);
        }
        if (!mbar_wait(&dbar[k & 1], (uint32_t)(k >> 1) & 1u)) *abort_flag = 1;
        const SPhase& ph = *reinterpret_cast<const SPhase*>(desc + (k & 1) * SK_DESC);
        if (k > 0 && !ph.moe_chain) {  // wait until every CTA has finished phase k-1
            if (tid == 0) {
                // acquire: the other CTAs' phase k-1 writes (released by their counts) become
                // visible to this thread and, through the CTA barrier below, to the whole CTA
                const unsigned long long target =
                    k == A.stall_phase ? ~0ull : base + (unsigned long long)k * G;
                bool ok = false;
                for (uint32_t it = 0; it < SK_BAR_SPINS; ++it) {
                    if (sk_ld_acquire(A.bar) >= target) { ok = true; break; }
                    if ((it & 63u) == 63u && *abort_flag) break;
                }
                if (!ok) {
                    if (!*abort_flag) set_device_error(SK_WAIT_ERR);
                    *abort_flag = 1;
                }
            }
            named_bar_sync(1, NT);
        }
        if (A.trace && tid == 0) A.trace[((size_t)c * NPH + k) * SK_TRACE] = sk_ns();
        unsigned long long wcyc = 0;
        if (ph.kind == SP_GEMV) {
            const RGemvArgs& g = ph.g;
            const SKRows rr = sk_rows(g, c, G);
            const void* xsrc = g.x;
            if (ph.epi == EPI_RESID && !(TP && ph.tp_red)) {  // residual rows, needed only by the epilogue: fetch them now
                const int nvr = rr.v_end - rr.v_begin;
                if (tid < nvr && tid < SK_RPRE) cp_async4(rpre + tid, g.resid + rr.v_begin + tid);
                cp_async_commit();
            }
            if (ph.embed) {
                // hidden = dequant(token_embd[token]) (gemv_q8_0.cuh:24-36) into shared memory after
                // the x records; CTA 0 also stores it as the residual stream
                const int K = g.I * 64;
                float* ebuf = reinterpret_cast<float*>(scratch + A.scratch_bytes) - K;
                const uint8_t* row = ph.embd + (size_t)A.state->token * (K / 32) * 34;
                for (int i = tid; i < K; i += NT) {
                    const uint8_t* blk = row + (i / 32) * 34;
                    const float v = half_bits_to_float(blk[0] | (blk[1] << 8)) * (float)(int8_t)blk[2 + (i & 31)];
                    ebuf[i] = v;
                    if (c == 0) ph.hidden_out[i] = v;
                }
                named_bar_sync(1, NT);
                xsrc = ebuf;
            }
            if (TP && ph.tp_sum) {
                // x = hin + every rank's partial of reduction red_idx, in rank order; a partial is
                // used once its tag matches (bounded spin per element)
                const int H = A.tp_h;
                float* hbuf = reinterpret_cast<float*>(scratch + A.scratch_bytes) - H;
                const unsigned long long* parts = sk_xpart(A, A.tp_rank, ph.red_idx & 1);
                const unsigned tag = sk_red_tag(A, launch0, ph.red_idx);
                const int h0 = (int)((long long)H * c / G), h1 = (int)((long long)H * (c + 1) / G);
                bool ok;
                switch (A.tp_n) {
                    case 2: ok = sk_tp_gather<2>(ph.hin, ph.hout, parts, tag, hbuf, H, h0, h1); break;
                    case 4: ok = sk_tp_gather<4>(ph.hin, ph.hout, parts, tag, hbuf, H, h0, h1); break;
                    default: ok = sk_tp_gather<8>(ph.hin, ph.hout, parts, tag, hbuf, H, h0, h1); break;
                }
                if (!ok) {
                    set_device_error(SK_WAIT_ERR);
                    *abort_flag = 1;
                }
                named_bar_sync(1, NT);
                xsrc = hbuf;
            }
            if (!ph.moe_reuse_x) {
                if (g.wt == WT_Q6K) sk_quantise_xm<WT_Q6K>(ph.xm, xsrc, g.norm_w, g.eps, g.I, xq_sa, misc);
                else sk_quantise_xm<WT_Q80>(ph.xm, xsrc, g.norm_w, g.eps, g.I, xq_sa, misc);
            }
            if (ph.moe == SK_MOE_GU && ph.moe_slot == 0)
                sk_route(static_cast<const float*>(xsrc), g.norm_w, g.eps, ph.route_w, ph.n_exp, ph.n_used, g.I * 64,
                         acc, misc, ph.moe_seq);
            bool moe_owned = true;
            float moe_w = 1.f;
            if (ph.moe) {
                const int e = reinterpret_cast<const int*>(misc + SK_MISC_ROUTE)[ph.moe_slot] - ph.e_lo;
                moe_owned = e >= 0 && e < ph.e_n;
                moe_w = misc[SK_MISC_ROUTE + 2 + ph.moe_slot];
            }
            if (A.trace && tid == 0) A.trace[((size_t)c * NPH + k) * SK_TRACE + 1] = sk_ns();
            if (!moe_owned) {
                // expert parallel: another rank's expert, nothing streamed for this slot
            } else if (g.wt == WT_Q6K)
                use = sk_stages<WT_Q6K>(g, rr, use, ring, A.slot_bytes, smem_sa, xq_sa, acc, full, empty, abort_flag);
            else
                use = sk_stages<WT_Q80>(g, rr, use, ring, A.slot_bytes, smem_sa, xq_sa, acc, full, empty, abort_flag);
            named_bar_sync(1, NT);  // every piece of every row is in shared memory
            if (A.trace && tid == 0) A.trace[((size_t)c * NPH + k) * SK_TRACE + 2] = sk_ns();
            if (ph.epi == EPI_RESID) {
                cp_async_wait_all();
                named_bar_sync(1, NT);
            }
            if (!*abort_flag && (moe_owned || ph.moe == SK_MOE_DN))
                sk_epilogues<TP>(g, ph.epi, rr, acc, rpre, best_v, best_i, A, ph,
                                 TP && ph.tp_red ? sk_red_tag(A, launch0, ph.red_idx) : 0u, moe_owned, moe_w);
            // attention next: this CTA's first unit's K tiles load across the phase change (the x
            // records are dead; the next descriptor was fetched at this phase's start); not after a
            // prefetch that no unit consumed, nor in a step that gave up
            if (k + 1 < NPH && tid < ATTN_THREADS && attn_pre == 0 && !*abort_flag &&
                mbar_wait(&dbar[(k + 1) & 1], (uint32_t)((k + 1) >> 1) & 1u)) {
                const SPhase& nx = *reinterpret_cast<const SPhase*>(desc + ((k + 1) & 1) * SK_DESC);
                if (nx.kind == SP_ATTN) {
                    const int seq = pos + 1;
                    const int clen = sk_attn_clen(seq, nx.at.nchunk, G, nx.at.n_kv_heads, A.attn_solo);
                    const int nch = (seq + clen - 1) / clen;
                    if (nch <= nx.at.nchunk && nx.at.stride_t == SK_ATT_RSTR && c < nx.at.n_kv_heads * nch) {
                        attn_pre = sk_attn_issue_early<KVT>(nx.at, c / nch, c % nch, clen, pos, scratch, abar);
                    }
                }
            }
        } else if (!*abort_flag) {
            const AttnArgs& at = ph.at;
            const int seq = pos + 1;
            const int clen = sk_attn_clen(seq, at.nchunk, G, at.n_kv_heads, A.attn_solo);
            const int nch = (seq + clen - 1) / clen;
            // the partials hold at.nchunk chunks per KV head (the engine sizes them for max_ctx)
            const bool fits = nch <= at.nchunk && at.stride_t == SK_ATT_RSTR;  // the engine's KV layout
            const int units = fits ? at.n_kv_heads * nch : 0;
            if (!fits && tid == 0) {
                set_device_error(SK_WAIT_ERR);
                *abort_flag = 1;
            }
            for (int u = c; u < units; u += G) {
                // the first unit's tile 0 may have been issued at the end of the previous phase
                if (tid < ATTN_THREADS)
                    sk_attn_unit<KVT>(at, u / nch, u % nch, clen, nch, pos, scratch, attn_pre > 0, abar, apar,
                                      abort_flag, (A.trace && u == c) ? A.trace + ((size_t)c * NPH + k) * SK_TRACE : nullptr);
                attn_pre = 0;
                named_bar_sync(1, NT);  // the next unit reuses the scratch
                if (A.trace && tid == 0 && u == c) A.trace[((size_t)c * NPH + k) * SK_TRACE + 1] = sk_ns();
            }
        }
        // ---- this CTA is done with phase k
        named_bar_sync(1, NT);
        if (tid == 0) {
            if (A.trace) {
                A.trace[((size_t)c * NPH + k) * SK_TRACE + 3] = sk_ns();
                if (ph.kind == SP_GEMV) A.trace[((size_t)c * NPH + k) * SK_TRACE + 4] = wcyc;
            }
            // release (cumulative): every consumer write of this CTA, ordered before by the CTA
            // barrier, is visible before the count
            asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(A.bar), "l"(1ull) : "memory");
        }
    }

    cp_async_wait_all();
    if (attn_pre > 0 && tid == 0) {  // tiles issued for a unit that did not run (a step that gave up):
        uint32_t bufs = (1u << attn_pre) - 1u;  // let the copies land (bounded) before the CTA exits
        if (attn_pre <= SK_ATT_TILES / 2) bufs |= bufs << (SK_ATT_TILES / 2);
        for (int b = 0; b < SK_ATT_TILES; ++b)
            if ((bufs >> b) & 1u)
                for (uint32_t it = 0; it < FENCE_WAIT_ROUNDS; ++it)
                    if (mbar_try_wait(&abar[b], (apar >> b) & 1u)) break;
    }
    // ---- argmax of the LM head: thread -> warp -> CTA -> (last CTA of the step) global
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
        for (int w = 0; w < SK_NW; ++w)
            if (warp_best_i[w] >= 0 && argmax_better(warp_best_v[w], warp_best_i[w], bv, bi)) {
                bv = warp_best_v[w];
                bi = warp_best_i[w];
            }
        A.cta_val[c] = bv;
        A.cta_idx[c] = bi;
        __threadfence();
        const unsigned long long prev = atomicAdd(A.bar, 1ull);
        if (prev == base + per_step - 1ull) {  // the last CTA: every CTA's best is visible
            __threadfence();
            float gv = 0.f;
            int gi = -1;
            for (int kk = 0; kk < G; ++kk) {
                const int ik = ((volatile int*)A.cta_idx)[kk];
                const float vk = ((volatile float*)A.cta_val)[kk];
                if (ik >= 0 && argmax_better(vk, ik, gv, gi)) {
                    gv = vk;
                    gi = ik;
                }
            }
            if (gi < 0) gi = 0;
            if (TP) {
                // every rank's shard best (value, global vocabulary index) to every rank, then the
                // best of them (greater value, then smaller index): the same id on every rank
                gi += A.vocab0;
                const unsigned long long pair = ((unsigned long long)(unsigned)gi << 32) | __float_as_uint(gv);
                for (int p = 0; p < A.tp_n; ++p) {
                    *reinterpret_cast<volatile unsigned long long*>(A.xb[p] + SK_XB_ARG + 8 * A.tp_rank) = pair;
                    sk_red_release_sys(reinterpret_cast<unsigned long long*>(A.xb[p] + SK_XB_ACNT), 1ull);
                }
                const unsigned long long* acnt = reinterpret_cast<const unsigned long long*>(A.xb[A.tp_rank] + SK_XB_ACNT);
                bool ok = false;
                for (uint32_t it = 0; it < SK_BAR_SPINS; ++it)
                    if (sk_ld_acquire_sys(acnt) >= (launch0 + 1ull) * (unsigned long long)A.tp_n) { ok = true; break; }
                if (!ok) set_device_error(SK_WAIT_ERR);
                for (int p = 0; p < A.tp_n; ++p) {
                    const unsigned long long q =
                        *reinterpret_cast<volatile const unsigned long long*>(A.xb[A.tp_rank] + SK_XB_ARG + 8 * p);
                    const float qv = __uint_as_float((unsigned)q);
                    const int qi = (int)(q >> 32);
                    if (p == 0 || qv > gv || (qv == gv && qi < gi)) {
                        gv = qv;
                        gi = qi;
                    }
                }
                *reinterpret_cast<volatile unsigned long long*>(A.launch) = launch0 + 1ull;
            }
            DecodeState* st = A.state;
            st->token = gi;
            st->pos = st->pos + 1;
            if (A.token_log && st->step < A.token_log_cap) A.token_log[st->step] = gi;
            st->step = st->step + 1;
            st->err = *reinterpret_cast<volatile int*>(&g_device_error);
        }
    }
}

}  // namespace fence
