// gemv.cu — launch planning for the streaming GEMV, the simple fallback kernels, and the drop-in
// GEMV / embedding entry points of the C-ABI (reference: src/kernels/gemv_q6k.cuh,
// src/kernels/gemv_q8_0.cuh).
#include "gemv.cuh"
#include "host.h"

#include <algorithm>

namespace fence {

// ------------------------------------------------------------------ fallback kernels
// One warp per row; lane t covers elements 8t..8t+7 of every super-block (the reference's
// q6k_dot_f16_warp_partial split, src/kernels/q6k_dot.cuh:199-238), fp32 FMAs, shuffle reduction.
__global__ void gemv_q6k_simple_kernel(const uint8_t* __restrict__ W, const uint16_t* __restrict__ x,
                                       const float* __restrict__ bias, float* __restrict__ y, int M,
                                       int K) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const int nb = K / 256;
    const uint8_t* rb = W + (size_t)row * nb * 210;
    float acc = 0.f;
    for (int b = 0; b < nb; ++b) {
        const uint8_t* blk = rb + (size_t)b * 210;
        const float d = half_bits_to_float(blk[208] | (blk[209] << 8));
        const int base = lane * 8;
        float part = 0.f;
        for (int e = base; e < base + 8; ++e) {
            const int h = e >> 7, rem = e & 127, col = rem >> 5, l = rem & 31;
            const int qlb = blk[64 * h + l + ((col & 1) ? 32 : 0)];
            const int lo = (col >= 2) ? (qlb >> 4) : (qlb & 15);
            const int hi = (blk[128 + 32 * h + l] >> (2 * col)) & 3;
            part = fmaf((float)((lo | (hi << 4)) - 32), half_bits_to_float(x[b * 256 + e]), part);
        }
        const float sc = (float)(int8_t)blk[192 + base / 16];
        acc += d * sc * part;
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = bias ? acc + bias[row] : acc;
}

__global__ void gemv_q8_0_simple_kernel(const uint8_t* __restrict__ W, const float* __restrict__ x,
                                        float* __restrict__ y, int M, int K) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const int nb = K / 32;
    const uint8_t* rb = W + (size_t)row * nb * 34;
    float acc = 0.f;
    for (int b = lane; b < nb; b += 32) {
        const uint8_t* blk = rb + (size_t)b * 34;
        const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
        float s = 0.f;
        for (int i = 0; i < 32; ++i) s += (float)(int8_t)blk[2 + i] * x[b * 32 + i];
        acc += d * s;
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

__global__ void embed_q8_0_kernel(float* __restrict__ out, const uint8_t* __restrict__ W,
                                  const int* __restrict__ token_dev, int token, int dim) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    const int t = token_dev ? *token_dev : token;
    const uint8_t* blk = W + ((size_t)t * (dim / 32) + i / 32) * 34;
    out[i] = half_bits_to_float(blk[0] | (blk[1] << 8)) * (float)(int8_t)blk[2 + (i & 31)];
}

// ------------------------------------------------------------------ planning
static int device_sms(int dev) {
    static int cached[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = v > 0 ? v : 148;
    }
    return cached[dev];
}
static int device_smem_optin(int dev) {
    static int cached[64] = {0};
    if (dev < 0 || dev >= 64) return 232448;
    if (!cached[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cached[dev] = v > 0 ? v : 232448;
    }
    return cached[dev];
}

// Launch plan of the warp-autonomous streaming GEMV:
//  * lanes per row (lpr): the width in {32, 16, 8, 4} that wastes the fewest lanes on the row's
//    items, subject to one warp batch of rows fitting a stage of <= 32 KB;
//  * stage = the largest multiple of the warp batch within 32 KB;
//  * 148 CTAs (one per SM, so the kernel launched next can sit beside it and prefetch) unless the
//    matrix is long enough to want more warps streaming per SM, then 2 per SM.
GemvPlan plan_gemv(int wt, int K, int Mv, int dual, int max_ctas) {
    GemvPlan pl{};
    const int blk_elems = (wt == WT_Q6K) ? 256 : 32;
    const int blk_bytes = (wt == WT_Q6K) ? 210 : 34;
    if (K <= 0 || Mv <= 0 || K % 64 != 0 || K % blk_elems != 0) return pl;
    const int I = K / 64;
    const int rowB = (K / blk_elems) * blk_bytes;
    const int RB = gemv_rows_per_group(dual);
    const int rows_per_unit = dual ? 2 : 1;
    const int stage_cap = 32768;
    int best_lpr = 0;
    double best_eff = -1.0;
    for (int lpr = 32; lpr >= 4; lpr >>= 1) {
        const int BR = (32 / lpr) * RB;
        if ((long long)BR * rows_per_unit * rowB > stage_cap && lpr != 32) continue;
        const int passes = (I + lpr - 1) / lpr;
        const double eff = (double)I / (double)(passes * lpr);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best_lpr = lpr;
        }
    }
    if (!best_lpr) return pl;
    const int BR = (32 / best_lpr) * RB;
    int mult = stage_cap / (BR * rows_per_unit * rowB);
    if (mult < 1) mult = 1;
    int S = BR * mult;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sms(dev);
    int G = max_ctas > 0 ? max_ctas : sms;
    if (max_ctas <= 0) {
        const int stages_one = ((Mv + sms - 1) / sms + S - 1) / S;
        if (stages_one > 8) G = 2 * sms;
    }
    if (G > Mv) G = Mv;
    const int rows_cta = (Mv + G - 1) / G;
    if (S > rows_cta) S = ((rows_cta + BR - 1) / BR) * BR;
    const int stages_cta = (rows_cta + S - 1) / S;
    const int SR = S * rows_per_unit;
    const int stage_bytes = ((SR * rowB + GEMV_STAGE_SLACK + 127) / 128) * 128;
    const int budget = std::min(device_smem_optin(dev) - 1024, 112 * 1024);
    int ring = 8;
    if (ring > stages_cta) ring = stages_cta;
    while (ring > 1 && (int)gemv_smem_layout(ring, stage_bytes, SR, I).total > budget) --ring;
    if ((int)gemv_smem_layout(ring, stage_bytes, SR, I).total > budget) return pl;
    pl.ok = 1;
    pl.I = I;
    pl.rowB = rowB;
    pl.S = S;
    pl.lpr = best_lpr;
    pl.ring = ring;
    pl.stage_bytes = stage_bytes;
    pl.block = GEMV_MAX_NT;
    pl.grid = G;
    pl.smem = (int)gemv_smem_layout(ring, stage_bytes, SR, I).total;
    return pl;
}

void fill_plan(GemvArgs& a, const GemvPlan& pl) {
    a.I = pl.I;
    a.rowB = pl.rowB;
    a.S = pl.S;
    a.lpr = pl.lpr;
    a.ring = pl.ring;
    a.stage_bytes = pl.stage_bytes;
}

template <int WT, int XM, int EPI>
cudaError_t launch_gemv(const GemvArgs& a, const GemvPlan& pl, cudaStream_t st, bool pdl) {
    auto kern = gemv_stream_kernel<WT, XM, EPI>;
    static int attr_set_dev_mask = 0;  // per-instantiation, per device (bit = device ordinal)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_set_dev_mask & (1 << (dev & 31)))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             device_smem_optin(dev));
        if (e != cudaSuccess) return e;
        attr_set_dev_mask |= 1 << (dev & 31);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(pl.block);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// explicit instantiations used by the drop-in entries and the engine
#define FENCE_GEMV_INST(WT, XM, EPI) \
    template cudaError_t launch_gemv<WT, XM, EPI>(const GemvArgs&, const GemvPlan&, cudaStream_t, bool);
FENCE_GEMV_INST(WT_Q6K, X_F16, EPI_STORE)
FENCE_GEMV_INST(WT_Q80, X_F32, EPI_STORE)
FENCE_GEMV_INST(WT_Q6K, X_NORM_R16, EPI_STORE)
FENCE_GEMV_INST(WT_Q80, X_NORM, EPI_STORE)
FENCE_GEMV_INST(WT_Q6K, X_F32_R16, EPI_RESID)
FENCE_GEMV_INST(WT_Q80, X_F32, EPI_RESID)
FENCE_GEMV_INST(WT_Q6K, X_NORM_R16, EPI_SWIGLU)
FENCE_GEMV_INST(WT_Q80, X_NORM, EPI_SWIGLU)
FENCE_GEMV_INST(WT_Q6K, X_F16, EPI_RESID)
FENCE_GEMV_INST(WT_Q80, X_NORM, EPI_LMHEAD)
FENCE_GEMV_INST(WT_Q6K, X_NORM, EPI_LMHEAD)
#undef FENCE_GEMV_INST

}  // namespace fence

using namespace fence;

// Process-wide launch flags of the drop-in GEMVs (fence_set_launch_flags).
static int g_launch_flags = 0;

extern "C" int fence_set_launch_flags(int flags) {
    const int old = g_launch_flags;
    g_launch_flags = flags;
    return old;
}

// Plan of the register-resident Q6_K GEMV (gemv_q6k_reg_kernel): rows of 16-byte multiple length
// (K % 2048 == 0), K <= 4096 (one 64-element item per lane), rows split over one CTA per SM. A chunk
// holds one row per row group of the consumers (GQ_NW warps, one or two per row), so each chunk is
// one item dot per lane with no group idle; chunk slots fill half an SM's shared memory at most
// (every chunk of a config-0 CTA in flight at once); ok = 0 otherwise.
struct GQPlan {
    int ok = 0, grid = 0, rows_cta = 0, RC = 0, slots = 0, slot_bytes = 0, smem = 0;
};
static GQPlan plan_q6k_reg(int M, int K) {
    GQPlan p;
    if (K <= 0 || K > 4096 || K % 2048 || M <= 0) return p;
    const int I = K / 64, rowB = K / 256 * 210;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sms(dev);
    p.rows_cta = (M + sms - 1) / sms;
    p.grid = (M + p.rows_cta - 1) / p.rows_cta;
    const int budget = device_smem_optin(dev) - 1024;
    const int fixed = I * XQ_WORDS * 4 + (2 * p.rows_cta + 2) * 4 + 8 + 2 * GQ_MAX_SLOTS * 8 + 16 + 64;
    const int avail = budget - fixed;
    const int NG = GQ_NW / (I > 32 ? 2 : 1);  // row groups working at once
    p.RC = std::min(NG, p.rows_cta);
    if (avail < 2 * p.RC * rowB) return p;
    p.slots = std::min(std::min(GQ_MAX_SLOTS, (p.rows_cta + p.RC - 1) / p.RC), avail / (p.RC * rowB));
    p.slot_bytes = (p.RC * rowB + 127) / 128 * 128;
    p.smem = p.slots * p.slot_bytes + fixed;
    if (p.smem > budget) return p;
    p.ok = 1;
    return p;
}

static cudaError_t launch_q6k_reg(const GQArgs& a, const GQPlan& pl, cudaStream_t st, bool pdl) {
    static int attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(gemv_q6k_reg_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, device_smem_optin(dev));
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(GQ_NT);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_q6k_reg_kernel, a);
}

// ------------------------------------------------------------------ drop-in entries
static int gemv_q6k_common(const block_q6_K* W, const uint16_t* x, const float* bias, float* y,
                           int M, int K, cudaStream_t st) {
    if (!W || !x || !y || M <= 0 || K <= 0 || K % 256 != 0)
        return set_error(FENCE_E_ARG, "gemv_q6k: need non-null pointers, M > 0, K %% 256 == 0 (M=%d K=%d)", M, K);
    const bool aligned = (reinterpret_cast<uintptr_t>(W) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    // Stream-ordered launches take the register-resident kernel (config 0, 4096 x 4096, back to back
    // in a CUDA graph on a B200: 6.7 us per launch against the streaming kernel's 10.0); launches
    // chained by programmatic dependent launch take the streaming kernel, whose two CTAs per SM let
    // the next launch stream its weights beside the previous one (8.2 us).
    const bool pdl = (g_launch_flags & FENCE_LAUNCH_PDL) != 0;
    const GQPlan gq = pdl ? GQPlan{} : plan_q6k_reg(M, K);
    if (aligned && gq.ok) {
        GQArgs a{};
        a.W = reinterpret_cast<const uint8_t*>(W);
        a.x = x;
        a.bias = bias;
        a.y = y;
        a.M = M;
        a.K = K;
        a.I = K / 64;
        a.rowB = K / 256 * 210;
        a.rows_cta = gq.rows_cta;
        a.RC = gq.RC;
        a.slots = gq.slots;
        a.slot_bytes = gq.slot_bytes;
        return cuda_status(launch_q6k_reg(a, gq, st, false), "gemv_q6k launch");
    }
    GemvPlan pl = plan_gemv(WT_Q6K, K, M, 0, 0);
    cudaError_t e;
    if (aligned && pl.ok) {
        GemvArgs a{};
        a.seg[0] = GemvSeg{reinterpret_cast<const uint8_t*>(W), M, y, bias};
        a.nseg = 1;
        a.Mv = M;
        a.K = K;
        a.x = x;
        fill_plan(a, pl);
        e = launch_gemv<WT_Q6K, X_F16, EPI_STORE>(a, pl, st, pdl);
    } else {
        const int threads = 128;
        gemv_q6k_simple_kernel<<<(M + 3) / 4, threads, 0, st>>>(reinterpret_cast<const uint8_t*>(W), x,
                                                                bias, y, M, K);
        e = cudaGetLastError();
    }
    return cuda_status(e, "gemv_q6k launch");
}

extern "C" int fence_gemv_q6k(const block_q6_K* W, const uint16_t* x, float* y, int M, int K,
                              fence_stream_t stream) {
    return gemv_q6k_common(W, x, nullptr, y, M, K, (cudaStream_t)stream);
}

extern "C" int fence_gemv_q6k_bias(const block_q6_K* W, const uint16_t* x, const float* bias,
                                   float* y, int M, int K, fence_stream_t stream) {
    if (!bias) return set_error(FENCE_E_ARG, "gemv_q6k_bias: bias is null");
    return gemv_q6k_common(W, x, bias, y, M, K, (cudaStream_t)stream);
}

extern "C" int fence_gemv_q8_0(const block_q8_0* W, const float* x, float* y, int M, int K,
                               fence_stream_t stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (!W || !x || !y || M <= 0 || K <= 0 || K % 32 != 0)
        return set_error(FENCE_E_ARG, "gemv_q8_0: need non-null pointers, M > 0, K %% 32 == 0 (M=%d K=%d)", M, K);
    const bool aligned = (reinterpret_cast<uintptr_t>(W) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    GemvPlan pl = plan_gemv(WT_Q80, K, M, 0, 0);
    cudaError_t e;
    if (aligned && pl.ok) {
        GemvArgs a{};
        a.seg[0] = GemvSeg{reinterpret_cast<const uint8_t*>(W), M, y, nullptr};
        a.nseg = 1;
        a.Mv = M;
        a.K = K;
        a.x = x;
        fill_plan(a, pl);
        e = launch_gemv<WT_Q80, X_F32, EPI_STORE>(a, pl, st, (g_launch_flags & FENCE_LAUNCH_PDL) != 0);
    } else {
        gemv_q8_0_simple_kernel<<<(M + 3) / 4, 128, 0, st>>>(reinterpret_cast<const uint8_t*>(W), x, y, M, K);
        e = cudaGetLastError();
    }
    return cuda_status(e, "gemv_q8_0 launch");
}

extern "C" int fence_embed_q8_0(float* out, const block_q8_0* weight, int token_id, int dim,
                                fence_stream_t stream) {
    if (!out || !weight || dim <= 0 || dim % 32 != 0 || token_id < 0)
        return set_error(FENCE_E_ARG, "embed_q8_0: bad arguments (dim=%d token=%d)", dim, token_id);
    embed_q8_0_kernel<<<(dim + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
        out, reinterpret_cast<const uint8_t*>(weight), nullptr, token_id, dim);
    return cuda_status(cudaGetLastError(), "embed_q8_0 launch");
}
