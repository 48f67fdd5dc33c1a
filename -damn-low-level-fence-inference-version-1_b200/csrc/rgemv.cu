// rgemv.cu — load-time repacking of the engine's linears and launch planning for rgemv_kernel
// (layouts and kernel in rgemv.cuh).
#include "host.h"
#include "rgemv.cuh"

#include <algorithm>

namespace fence {

// ------------------------------------------------------------------ repack kernels (load time)
// GGUF Q6_K rows (block_q6_K, src/kernels/q6k_types.h:27-32) -> q/s/d arrays; row r of the source
// becomes row dst_row0 + r * dst_stride of the destination (fused QKV, interleaved gate/up). The
// source rows are src_nsb blocks apart; items item0 .. item0 + I - 1 of each are taken (a column
// slice, a tensor-parallel shard of a row-parallel matrix, when I < 4 src_nsb; it may start and
// end inside a super-block, whose d is then repeated in each neighbour's rows).
__global__ void repack_q6k_kernel(const uint8_t* __restrict__ src, long long rows, int I, int src_nsb, int item0,
                                  uint8_t* __restrict__ q, uint8_t* __restrict__ s, uint8_t* __restrict__ d,
                                  long long dst_row0, int dst_stride) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * I) return;
    const long long r = idx / I;
    const int it = (int)(idx - r * I);
    const int gi = item0 + it;  // item index in the source row
    const int j = gi >> 2, h = (gi >> 1) & 1, l16 = gi & 1;
    const int nsb = (I + (item0 & 3) + 3) >> 2;  // d entries per destination row
    const uint8_t* blk = src + ((size_t)r * src_nsb + j) * 210;
    const long long dr = dst_row0 + r * dst_stride;
    uint8_t* qd = q + ((size_t)dr * I + it) * 48;
    for (int e = 0; e < 16; ++e) {
        qd[e] = blk[64 * h + 16 * l16 + e];
        qd[16 + e] = blk[64 * h + 32 + 16 * l16 + e];
        qd[32 + e] = blk[128 + 32 * h + 16 * l16 + e];
    }
    uint8_t* sd = s + (size_t)dr * rg_sbytes_row(WT_Q6K, I) + (size_t)it * 4;
    for (int c = 0; c < 4; ++c) sd[c] = blk[192 + 8 * h + 2 * c + l16];
    if ((gi & 3) == 0 || it == 0) {  // the first item of each super-block this row holds
        uint8_t* dd = d + ((size_t)dr * nsb + (j - (item0 >> 2))) * 2;
        dd[0] = blk[208];
        dd[1] = blk[209];
    }
}

// GGUF Q8_0 rows (block_q8_0, src/kernels/q8_0_types.h:11-14) -> swizzled q / d arrays; source
// rows src_nb blocks apart, items item0 .. item0 + I - 1 (blocks 2 item0 ..) of each taken.
__global__ void repack_q80_kernel(const uint8_t* __restrict__ src, long long rows, int I, int src_nb, int item0,
                                  uint8_t* __restrict__ q, uint8_t* __restrict__ d, long long dst_row0,
                                  int dst_stride) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * I) return;
    const long long r = idx / I;
    const int it = (int)(idx - r * I);
    const uint8_t* b0 = src + ((size_t)r * src_nb + 2 * (item0 + it)) * 34;
    const uint8_t* b1 = b0 + 34;
    const long long dr = dst_row0 + r * dst_stride;
    uint8_t* qd = q + ((size_t)dr * I + it) * 64;
    const int f = (it >> 1) & 3;
    for (int p = 0; p < 4; ++p) {
        const int k = p ^ f;  // chunk k: elements 16k .. 16k+15 of the item
        const uint8_t* blk = (k >> 1) ? b1 : b0;
        for (int e = 0; e < 16; ++e) qd[16 * p + e] = blk[2 + 16 * (k & 1) + e];
    }
    uint8_t* dd = d + ((size_t)dr * I + it) * 4;
    dd[0] = b0[0];
    dd[1] = b0[1];
    dd[2] = b1[0];
    dd[3] = b1[1];
}

// Row-major repacked matrix -> the step kernel's tiles (sk_tile_bytes): CTA c of G holds the
// virtual rows [Mv c / G, Mv (c + 1) / G) (dual: both rows of each gate/up pair), cut into row blocks
// of RB rows and K-slices of CI items, tiles in (block, slice) order from byte tcta[c]. One thread
// per (row, item) record; Q8_0 chunk positions re-swizzled by the item's slot in its slice; the
// thread of slot 0 also writes the row's Q6_K d entries of the slice. dst must be zeroed.
__device__ __forceinline__ int rt_vbegin(long long Mv, int c, int G) { return (int)((Mv * c) / G); }
__global__ void retile_kernel(int wt, RMat m, int I, int Mv, int dual, int G, int RB, int CI,
                              const unsigned long long* __restrict__ tcta, uint8_t* __restrict__ dst) {
    const long long rows = (long long)Mv * (dual ? 2 : 1);
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * I) return;
    const long long r = idx / I;
    const int it = (int)(idx - r * I);
    const int v = (int)(dual ? r / 2 : r);
    int c = (int)min((long long)G - 1, ((long long)v * G) / Mv);
    while (c > 0 && rt_vbegin(Mv, c, G) > v) --c;
    while (c + 1 < G && rt_vbegin(Mv, c + 1, G) <= v) ++c;
    const int f = dual ? 2 : 1;
    const long long r_begin = (long long)f * rt_vbegin(Mv, c, G);
    const int rows_c = f * (rt_vbegin(Mv, c + 1, G) - rt_vbegin(Mv, c, G));
    const int rl = (int)(r - r_begin), b = rl / RB, rb = rl - b * RB;
    const int rows_b = min(RB, rows_c - b * RB);
    const int ns = (I + CI - 1) / CI, j = it / CI, is = it - j * CI;
    const int items = min(CI, I - j * CI);
    const unsigned long long block_bytes =
        (unsigned long long)(ns - 1) * sk_tile_bytes(wt, RB, CI, CI) + sk_tile_bytes(wt, RB, I - (ns - 1) * CI, CI);
    uint32_t s_off, d_off;
    sk_tile_bytes(wt, rows_b, items, CI, &s_off, &d_off);
    uint8_t* t = dst + tcta[c] + (unsigned long long)b * block_bytes +
                 (unsigned long long)j * sk_tile_bytes(wt, rows_b, CI, CI);
    const uint32_t rec = (uint32_t)(rb * items + is);
    if (wt == WT_Q80) {
        const uint8_t* sq = m.q + ((size_t)r * I + it) * 64;
        const int fs = (it >> 1) & 3, fd = (is >> 1) & 3;
        uint8_t* dq = t + (size_t)rec * 64;
        for (int p = 0; p < 4; ++p) {
            const int k = p ^ fs;  // the chunk at source position p
            for (int e = 0; e < 16; ++e) dq[16 * (k ^ fd) + e] = sq[16 * p + e];
        }
        const uint8_t* sd = m.d + ((size_t)r * I + it) * 4;
        for (int e = 0; e < 4; ++e) t[d_off + rec * 4 + e] = sd[e];
    } else {
        const uint8_t* sq = m.q + ((size_t)r * I + it) * 48;
        for (int e = 0; e < 48; ++e) t[(size_t)rec * 48 + e] = sq[e];
        const uint8_t* ss = m.s + (size_t)r * rg_sbytes_row(WT_Q6K, I) + (size_t)it * 4;
        for (int e = 0; e < 4; ++e) t[s_off + rec * 4 + e] = ss[e];
        if (is == 0) {
            const int ndq = sk_ndq(CI), dbr = rg_dbytes_row(WT_Q6K, I, m.iph), nsb = dbr / 2;
            const int sb0 = (j * CI + m.iph) >> 2;
            for (int e = 0; e < ndq && sb0 + e < nsb; ++e) {
                t[d_off + (rb * ndq + e) * 2] = m.d[(size_t)r * dbr + (sb0 + e) * 2];
                t[d_off + (rb * ndq + e) * 2 + 1] = m.d[(size_t)r * dbr + (sb0 + e) * 2 + 1];
            }
        }
    }
}

// Tile offsets of every CTA (host): tcta[c] for c < G and the matrix's tiled bytes (return).
unsigned long long sk_tile_plan(int wt, int I, int Mv, int dual, int G, int RB, int CI, unsigned long long* tcta) {
    const int ns = (I + CI - 1) / CI, f = dual ? 2 : 1;
    unsigned long long off = 0;
    for (int c = 0; c < G; ++c) {
        tcta[c] = off;
        const int rows_c = f * (int)(((long long)Mv * (c + 1)) / G - ((long long)Mv * c) / G);
        for (int r0 = 0; r0 < rows_c; r0 += RB) {
            const int rows_b = std::min(RB, rows_c - r0);
            for (int j = 0; j < ns; ++j) off += sk_tile_bytes(wt, rows_b, std::min(CI, I - j * CI), CI);
        }
    }
    return off;
}

cudaError_t sk_retile(int wt, const RMat& m, int I, int Mv, int dual, int G, int RB, int CI,
                      const unsigned long long* d_tcta, uint8_t* dst, cudaStream_t st) {
    const long long n = (long long)Mv * (dual ? 2 : 1) * I;
    const int threads = 256;
    retile_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(wt, m, I, Mv, dual, G, RB, CI, d_tcta,
                                                                              dst);
    return cudaGetLastError();
}

size_t rmat_bytes(int wt, long long rows, int K, int iph) {
    const int I = K / 64;
    auto pad = [](size_t x) { return (x + 64 + 255) / 256 * 256; };
    size_t n = pad((size_t)rows * I * rg_qbytes(wt)) + pad((size_t)rows * rg_dbytes_row(wt, I, iph));
    if (wt == WT_Q6K) n += pad((size_t)rows * rg_sbytes_row(wt, I));
    return n;
}

// Carves an RMat of `rows` rows of K inputs out of base (rmat_bytes(wt, rows, K, iph) bytes).
RMat rmat_carve(int wt, long long rows, int K, uint8_t* base, int iph) {
    const int I = K / 64;
    auto pad = [](size_t x) { return (x + 64 + 255) / 256 * 256; };
    RMat m{};
    uint8_t* p = base;
    m.q = p;
    p += pad((size_t)rows * I * rg_qbytes(wt));
    if (wt == WT_Q6K) {
        m.s = p;
        p += pad((size_t)rows * rg_sbytes_row(wt, I));
    }
    m.d = p;
    m.rows = (int)rows;
    m.iph = wt == WT_Q6K ? iph : 0;
    return m;
}

// src: the source rows' start; src_K: inputs per source row (0: K); item0: the first 64-input
// item of each source row taken (a column slice when K < src_K).
cudaError_t rmat_fill(int wt, const uint8_t* src, long long rows, int K, const RMat& m, long long dst_row0,
                      int dst_stride, cudaStream_t st, int src_K, int item0) {
    const int I = K / 64;
    const long long n = rows * I;
    const int threads = 256;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    if (src_K <= 0) src_K = K;
    if (wt == WT_Q6K)
        repack_q6k_kernel<<<blocks, threads, 0, st>>>(src, rows, I, src_K / 256, item0, const_cast<uint8_t*>(m.q),
                                                      const_cast<uint8_t*>(m.s), const_cast<uint8_t*>(m.d), dst_row0,
                                                      dst_stride);
    else
        repack_q80_kernel<<<blocks, threads, 0, st>>>(src, rows, I, src_K / 32, item0, const_cast<uint8_t*>(m.q),
                                                      const_cast<uint8_t*>(m.d), dst_row0, dst_stride);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ planning
// Fills a.np / a.R / a.ring / a.slot_bytes for a GEMV of a.Mv virtual rows of K = a.I * 64.
// smem_budget: dynamic shared memory one CTA may use (two CTAs of consecutive phases share an SM).
RGemvPlan plan_rgemv(RGemvArgs& a, int sms, int smem_budget) {
    RGemvPlan P{};
    const int I = a.I;
    if (I <= 0 || a.Mv <= 0) return P;
    int np = (I + RG_NL - 1) / RG_NL;
    while (np <= I && I % np) ++np;  // equal parts
    const int IP = I / np;
    int R = std::min((RG_NL / IP) / np, RG_MAX_R);
    if (a.dual) R &= ~1;
    if (R < (a.dual ? 2 : 1)) return P;
    {  // no stage larger than the CTA's share of rows
        const int g = std::min(sms, a.Mv);
        const int rc = (int)(((long long)a.Mv + g - 1) / g) * (a.dual ? 2 : 1);
        if (R > rc) R = a.dual ? std::max(2, (rc + 1) & ~1) : std::max(1, rc);
    }
    const int slot = (int)((rg_slot(a.wt, I, R, a.w.iph).bytes + 127u) & ~127u);
    const int S = a.dual ? R / 2 : R;
    const int grid = std::min(sms, a.Mv);
    const int vcta = (a.Mv + grid - 1) / grid;  // max virtual rows of one CTA
    const int stages = (vcta + S - 1) / S;
    int mp = 1;
    for (int r = 0; r < R; ++r) mp = std::max(mp, rg_row_pieces(r, np, IP));
    const int rows_cta = vcta * (a.dual ? 2 : 1);
    int ring = std::min(RG_MAX_RING, std::max(stages, 2));
    while (ring > 2 && (int)rg_smem_layout(ring, slot, I, rows_cta, mp).total > smem_budget) --ring;
    if ((int)rg_smem_layout(ring, slot, I, rows_cta, mp).total > smem_budget) return P;
    a.np = np;
    a.R = R;
    a.ring = ring;
    a.slot_bytes = slot;
    a.mp = mp;
    a.rows_cta = rows_cta;
    P.ok = 1;
    P.grid = grid;
    P.block = RG_NT;
    P.smem = (int)rg_smem_layout(ring, slot, I, rows_cta, mp).total;
    return P;
}

template <int WT, int XM, int EPI>
cudaError_t launch_rgemv(const RGemvArgs& a, const RGemvPlan& P, cudaStream_t st) {
    auto kern = rgemv_kernel<WT, XM, EPI>;
    static int smem_set[64] = {};  // per device: largest dynamic smem enabled so far
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem_set[dev] < P.smem) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P.smem);
        if (e != cudaSuccess) return e;
        smem_set[dev] = P.smem;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(P.grid);
    cfg.blockDim = dim3(P.block);
    cfg.dynamicSmemBytes = P.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// The engine's (weight type, x mode, epilogue) combinations.
cudaError_t rgemv_dispatch(int xm, int epi, const RGemvArgs& a, const RGemvPlan& P, cudaStream_t st) {
#define RCASE(WT, XM, EPI) \
    if (a.wt == WT && xm == XM && epi == EPI) return launch_rgemv<WT, XM, EPI>(a, P, st);
    RCASE(WT_Q6K, X_NORM_R16, EPI_STORE)
    RCASE(WT_Q80, X_NORM, EPI_STORE)
    RCASE(WT_Q6K, X_F32_R16, EPI_RESID)
    RCASE(WT_Q80, X_F32, EPI_RESID)
    RCASE(WT_Q6K, X_NORM_R16, EPI_SWIGLU)
    RCASE(WT_Q80, X_NORM, EPI_SWIGLU)
    RCASE(WT_Q6K, X_F16, EPI_RESID)
    RCASE(WT_Q80, X_NORM, EPI_LMHEAD)
#undef RCASE
    return cudaErrorInvalidValue;
}

}  // namespace fence
