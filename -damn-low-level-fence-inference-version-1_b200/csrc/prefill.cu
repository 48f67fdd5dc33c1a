// prefill.cu — batched prefill: the prompt's tokens through every layer at once as dense
// contractions on the 5th-generation tensor cores (tcgen05, accumulators in tensor memory). The
// reference prefills token by token (src/model/qwen3.cu:478-481: one forward per prompt token, each
// a chain of GEMVs); here a chunk of P tokens is one GEMM per linear, so the weights are read once
// per chunk instead of once per token.
//
// Per layer (same op order and numerics points as the decode step; dense models, one rank):
//   RMSNorm rows -> fp16 | QKV GEMM (+bias) | q/k RMSNorm per head, NeoX RoPE, K/V rows into the
//   cache | causal GQA attention over the cache | O GEMM, += residual | RMSNorm rows -> fp16 |
//   gate/up GEMM with the SwiGLU epilogue -> fp16 | down GEMM, += residual.
// The weights are dequantised from the engine's repacked Q6_K / Q8_0 rows into fp16 per layer
// (each row scaled by a power of two that puts its largest weight near 2^14, so the small Q6_K
// weights stay normal fp16 numbers; the GEMM epilogue multiplies the scale back out).
//
// tc_gemm_kernel: C[P x N] = A[P x K] . B[N x K]^T, A and B fp16 row-major (K-major operands), fp32
// accumulation in tensor memory. CTA tile 128 x 256, K steps of 64 through a 4-stage shared-memory
// ring filled by cp.async (16-byte chunks into the no-swizzle canonical layout: 8-row x 16-byte core
// matrices, 128 bytes apart along K and 1024 bytes apart along M/N); one thread issues four
// tcgen05.mma (M128 N256 K16) per stage and commits them to the stage's mbarrier; the loaders wait on
// it before refilling that stage, after the next stage's MMAs are already queued. Epilogue: each warp reads its 32 accumulator lanes (rows)
// with tcgen05.ld, 32 columns at a time.
#include <cuda_fp16.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "host.h"
#include "rgemv.cuh"

namespace fence {

constexpr int TG_BM = 128, TG_BN = 256, TG_BK = 64, TG_STAGES = 4, TG_THREADS = 128;
constexpr int TG_A_BYTES = TG_BM * TG_BK * 2;
constexpr int TG_B_BYTES = TG_BN * TG_BK * 2;
constexpr int TG_STAGE_BYTES = TG_A_BYTES + TG_B_BYTES;
constexpr int TG_SMEM = TG_STAGES * TG_STAGE_BYTES + 128;  // + mbarriers and the tensor-memory address
constexpr uint32_t TG_TMEM_COLS = 256;

enum : int { TG_EPI_STORE = 0, TG_EPI_ADD = 1, TG_EPI_SWIGLU = 2 };

struct TGArgs {
    const __half* A;      // [P][K]
    const __half* B;      // [N][K]
    const float* bscale;  // [N] multiplies column n of the product (undoes the weight row scaling); null = 1
    int P, N, K;
    float* C;             // STORE / ADD: [P][ldc]
    int ldc;
    const float* bias;    // STORE: [N], optional
    __half* H;            // SWIGLU: [P][ldh], column n / 2 = silu(column n) * column n + 1 (n even)
    int ldh;
};

// 64-bit shared-memory matrix descriptor (no swizzle, K-major): start address, leading-dimension
// byte offset (between core matrices along K), stride-dimension byte offset (between 8-row groups),
// descriptor version 1.
__device__ __forceinline__ uint64_t tg_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor, kind::f16: fp32 accumulator, A and B fp16, both K-major, N, M.
__host__ __device__ constexpr uint32_t tg_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// One stage's operand tiles: chunk (row, k8) of an R-row tile goes to core matrix (row / 8, k8) at
// ((row / 8) * 8 + k8) * 128 + (row % 8) * 16. Rows past `rows` are zero-filled.
__device__ __forceinline__ void tg_load_tile(uint32_t sbase, const __half* g, int ld, int row0, int rows, int k0,
                                             int R) {
    const int n = R * 8;
    for (int c = threadIdx.x; c < n; c += TG_THREADS) {
        const int rr = c & 7, kc = (c >> 3) & 7, grp = c >> 6;
        const int row = grp * 8 + rr;
        const uint32_t dst = sbase + (uint32_t)((grp * 8 + kc) * 128 + rr * 16);
        const bool ok = row0 + row < rows;
        const __half* src = ok ? g + (size_t)(row0 + row) * ld + k0 + kc * 8 : g;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
                     : "memory");
    }
}

__device__ __forceinline__ float tg_silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int EPI>
__global__ void __launch_bounds__(TG_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TGArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int p0 = blockIdx.x * TG_BM, n0 = blockIdx.y * TG_BN;
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TG_STAGES * TG_STAGE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + TG_STAGES);
    if (tid == 0) {
        for (int s = 0; s < TG_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TG_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    const int nk = a.K / TG_BK;
    constexpr uint32_t idesc = tg_idesc(TG_BM, TG_BN);
    bool ok = true;
    for (int s = 0; s < TG_STAGES - 1; ++s) {
        if (s < nk) {
            const uint32_t st = sbase + (uint32_t)(s * TG_STAGE_BYTES);
            tg_load_tile(st, a.A, a.K, p0, a.P, s * TG_BK, TG_BM);
            tg_load_tile(st + TG_A_BYTES, a.B, a.K, n0, a.N, s * TG_BK, TG_BN);
        }
        cp_async_commit();
    }
    for (int kt = 0; kt < nk; ++kt) {
        cp_async_wait_group<TG_STAGES - 2>();                      // k-tile kt has landed (this thread's part)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int s = kt % TG_STAGES;
            const uint32_t sa = sbase + (uint32_t)(s * TG_STAGE_BYTES), sb = sa + TG_A_BYTES;
#pragma unroll
            for (int t = 0; t < TG_BK / 16; ++t) {
                const uint64_t da = tg_desc(sa + (uint32_t)t * 256u, 128u, 1024u);
                const uint64_t db = tg_desc(sb + (uint32_t)t * 256u, 128u, 1024u);
                const uint32_t acc = (kt > 0 || t > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                    "l"(da), "l"(db), "r"(idesc), "r"(acc)
                    : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&bars[s]))
                         : "memory");
        }
        // refill the stage of k-tile kt - 1 with k-tile kt + STAGES - 1 once its MMAs are done (they
        // ran while k-tile kt's were queued behind them)
        const int kn = kt + TG_STAGES - 1;
        if (kn < nk) {
            const int sn = kn % TG_STAGES;
            if (kt >= 1 && !mbar_wait(&bars[sn], (uint32_t)((kt - 1) / TG_STAGES) & 1u)) ok = false;
            const uint32_t st = sbase + (uint32_t)(sn * TG_STAGE_BYTES);
            tg_load_tile(st, a.A, a.K, p0, a.P, kn * TG_BK, TG_BM);
            tg_load_tile(st + TG_A_BYTES, a.B, a.K, n0, a.N, kn * TG_BK, TG_BN);
        }
        cp_async_commit();
    }
    cp_async_wait_all();
    // every MMA of the tile is complete once the last stage's commit has arrived
    if (nk > 0 && !mbar_wait(&bars[(nk - 1) % TG_STAGES], (uint32_t)((nk - 1) / TG_STAGES) & 1u)) ok = false;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    // ---- epilogue: warp w holds rows p0 + 32 w + lane, 32 columns per tensor-memory load
    const int p = p0 + warp * 32 + lane;
    for (int c0 = 0; c0 < TG_BN; c0 += 32) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
            "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
              "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr)
            : "memory");
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (!ok || p >= a.P) continue;
        const int nb = n0 + c0;
        if (EPI == TG_EPI_SWIGLU) {
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const int n = nb + j;
                if (n + 1 < a.N) {
                    const float g = __uint_as_float(r[j]) * (a.bscale ? a.bscale[n] : 1.f);
                    const float u = __uint_as_float(r[j + 1]) * (a.bscale ? a.bscale[n + 1] : 1.f);
                    a.H[(size_t)p * a.ldh + n / 2] = __float2half_rn(tg_silu_mul(g, u));
                }
            }
        } else {
            float* crow = a.C + (size_t)p * a.ldc;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int n = nb + j;
                if (n < a.N) {
                    float v = __uint_as_float(r[j]) * (a.bscale ? a.bscale[n] : 1.f);
                    if (EPI == TG_EPI_STORE) {
                        if (a.bias) v += a.bias[n];
                        crow[n] = v;
                    } else {
                        crow[n] += v;
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TG_TMEM_COLS) : "memory");
}

// ------------------------------------------------------------------ weight dequantisation
// Repacked row r of an RMat (rgemv.cuh layouts, one rank: item0 = 0) -> fp16 row r of W[M][K] in the
// natural column order, times 2^e_r with e_r the largest exponent keeping the row's largest |w| at or
// below 2^14; bscale[r] = 2^-e_r. One CTA per row.
//   Q6_K item i of a row: super-block j = i / 4, half h = (i / 2) & 1, l16 = i & 1; its element
//   (c, e) (column run c < 4, e < 16) is column 256 j + 128 h + 32 c + 16 l16 + e, value
//   d_j * scale_c * (q6 - 32) with q6 = low nibble of byte (c & 1) * 16 + e (its high nibble for
//   c >= 2) | crumb c of byte 32 + e << 4 of the item's 48-byte record.
//   Q8_0 item i: chunk k of 16 int8 at record position k ^ ((i >> 1) & 3); block scales d0, d1.
template <int WT>
__device__ __forceinline__ float dq_value(const RMat& m, int I, long long r, int it, int c, int e, int* col) {
    if (WT == WT_Q6K) {
        const uint8_t* q = m.q + ((size_t)r * I + it) * 48;
        const uint8_t lo = q[(c & 1) * 16 + e];
        const int nib = c >= 2 ? lo >> 4 : lo & 15;
        const int q6 = nib | (((q[32 + e] >> (2 * c)) & 3) << 4);
        const int sc = (int8_t)m.s[(size_t)r * rg_sbytes_row(WT_Q6K, I) + (size_t)it * 4 + c];
        const uint8_t* dp = m.d + (size_t)r * rg_dbytes_row(WT_Q6K, I, 0) + (size_t)(it >> 2) * 2;
        const float d = half_bits_to_float((uint32_t)dp[0] | ((uint32_t)dp[1] << 8));
        *col = (it >> 2) * 256 + ((it >> 1) & 1) * 128 + c * 32 + (it & 1) * 16 + e;
        return d * (float)sc * (float)(q6 - 32);
    } else {
        const int k = c;  // chunk (16 elements)
        const uint8_t* q = m.q + ((size_t)r * I + it) * 64;
        const int qv = (int8_t)q[16 * (k ^ ((it >> 1) & 3)) + e];
        const uint8_t* dp = m.d + ((size_t)r * I + it) * 4 + (k >> 1) * 2;
        const float d = half_bits_to_float((uint32_t)dp[0] | ((uint32_t)dp[1] << 8));
        *col = it * 64 + 16 * k + e;
        return d * (float)qv;
    }
}

template <int WT>
__global__ void dequant_rows_kernel(RMat m, int I, __half* __restrict__ W, float* __restrict__ bscale) {
    __shared__ float red[32];
    const long long r = blockIdx.x;
    const int n = I * 64;
    float amax = 0.f;
    for (int x = threadIdx.x; x < n; x += blockDim.x) {
        int col;
        amax = fmaxf(amax, fabsf(dq_value<WT>(m, I, r, x >> 6, (x >> 4) & 3, x & 15, &col)));
    }
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_max(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    amax = red[0];
    int e = 0;
    if (amax > 0.f && isfinite(amax)) {
        int ex;
        frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
        e = 14 - ex;        // amax * 2^e < 2^14
    }
    const float s = ldexpf(1.f, e);
    if (threadIdx.x == 0) bscale[r] = ldexpf(1.f, -e);
    for (int x = threadIdx.x; x < n; x += blockDim.x) {
        int col;
        const float v = dq_value<WT>(m, I, r, x >> 6, (x >> 4) & 3, x & 15, &col);
        W[(size_t)r * n + col] = __float2half_rn(v * s);
    }
}

// ------------------------------------------------------------------ per-token row kernels
// hidden[p] = dequant(token_embd[tok[p]]) (embed_q8_0, src/kernels/gemv_q8_0.cuh:12-29)
__global__ void embed_rows_kernel(const uint8_t* __restrict__ embd, const int* __restrict__ tok, int H,
                                  float* __restrict__ hidden) {
    const int p = blockIdx.x;
    const uint8_t* row = embd + (size_t)tok[p] * (H / 32) * 34;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const uint8_t* blk = row + (i / 32) * 34;
        hidden[(size_t)p * H + i] = half_bits_to_float(blk[0] | (blk[1] << 8)) * (float)(int8_t)blk[2 + (i & 31)];
    }
}

// out[p] = fp16(w * x[p] * rsqrt(mean(x[p]^2) + eps)) (rms_norm, src/kernels/ops.cuh:17-45, then the
// f32_to_f16 before a GEMV, qwen3.cu:278,325)
__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w, int H, float eps,
                                    __half* __restrict__ out) {
    __shared__ float red[32];
    const int p = blockIdx.x;
    const float* xr = x + (size_t)p * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float rms = rsqrtf(red[0] / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[(size_t)p * H + i] = __float2half_rn(w[i] * xr[i] * rms);
}

// fp32 rows -> fp16 (the attention output before the O GEMM)
__global__ void f32_to_f16_rows_kernel(const float* __restrict__ x, long long n, __half* __restrict__ out) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(x[i]);
}

// q/k RMSNorm per head (w * x * rms, ops.cuh:66-95) and NeoX RoPE at the token's position
// (ops.cuh:115-167, the engine's cos/sin table) for every token of the chunk; q to qout (fp32), k and
// v rounded to the cache type into the cache rows (store_kv, ops.cuh:420-443). A warp per head.
template <typename KVT>
__global__ void prefill_qk_kernel(const float* __restrict__ qkv, int ldqkv, int Hq, int Hkv,
                                  const float* __restrict__ qn, const float* __restrict__ kn, float eps,
                                  const float2* __restrict__ rope, int pos0, float* __restrict__ qout,
                                  KVT* __restrict__ kc, KVT* __restrict__ vc, long long stride_h, int stride_t) {
    using C = KVConv<KVT>;
    constexpr int HD = 128;
    const int p = blockIdx.x, pos = pos0 + p, lane = threadIdx.x & 31;
    const float* row = qkv + (size_t)p * ldqkv;
    const float2* cs = rope + (size_t)pos * (HD / 2);
    for (int head = threadIdx.x >> 5; head < Hq + Hkv; head += blockDim.x >> 5) {
        const bool isq = head < Hq;
        const float* src = row + (size_t)head * HD;  // q heads, then k heads
        const float* w = isq ? qn : kn;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = src[lane + 32 * i];
        if (w) {
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) ss += v[i] * v[i];
            ss = warp_sum(ss);
            const float r = rsqrtf(ss / (float)HD + eps);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = w[lane + 32 * i] * v[i] * r;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {  // pairs (d, d + 64): d = lane + 32 i
            const float2 t = cs[lane + 32 * i];
            const float a = v[i], b = v[i + 2];
            v[i] = a * t.x - b * t.y;
            v[i + 2] = a * t.y + b * t.x;
        }
        if (isq) {
#pragma unroll
            for (int i = 0; i < 4; ++i) qout[((size_t)p * Hq + head) * HD + lane + 32 * i] = v[i];
        } else {
            const int h = head - Hq;
            const float* vsrc = row + (size_t)(Hq + Hkv + h) * HD;
            KVT* kd = kc + (size_t)h * stride_h + (size_t)pos * stride_t;
            KVT* vd = vc + (size_t)h * stride_h + (size_t)pos * stride_t;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                kd[lane + 32 * i] = C::from(v[i]);
                vd[lane + 32 * i] = C::from(vsrc[lane + 32 * i]);
            }
        }
    }
}

// Causal GQA attention of the chunk's tokens over the cache (gqa_attention, ops.cuh:320-403): CTA
// (token p, KV head h) computes its G query heads over positions 0 .. pos0 + p in 64-position tiles
// with an online softmax (fp32; K and V as cached).
constexpr int PA_THREADS = 128, PA_TILE = 64;
template <typename KVT>
__global__ void __launch_bounds__(PA_THREADS) prefill_attn_kernel(const float* __restrict__ q, int Hq, int Hkv,
                                                                   const KVT* __restrict__ kc, const KVT* __restrict__ vc,
                                                                   long long stride_h, int stride_t, int pos0,
                                                                   float* __restrict__ out) {
    using C = KVConv<KVT>;
    constexpr int HD = 128;
    __shared__ float sq[8][HD];
    __shared__ float skv[PA_TILE][HD + 1];
    __shared__ float sp[8][PA_TILE];
    __shared__ float sm[8], sl[8], sc[8];
    const int p = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = Hq / Hkv, seq = pos0 + p + 1;
    const float scale = rsqrtf((float)HD);
    for (int i = tid; i < G * HD; i += PA_THREADS) sq[i / HD][i % HD] = q[((size_t)p * Hq + h * G) * HD + i];
    if (tid < G) {
        sm[tid] = -INFINITY;
        sl[tid] = 0.f;
    }
    float acc[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) acc[g] = 0.f;
    const KVT* kb = kc + (size_t)h * stride_h;
    const KVT* vb = vc + (size_t)h * stride_h;
    for (int t0 = 0; t0 < seq; t0 += PA_TILE) {
        const int n = min(PA_TILE, seq - t0);
        __syncthreads();  // q / softmax state ready; the previous tile's V reads are done
        for (int i = tid; i < n * HD; i += PA_THREADS)
            skv[i / HD][i % HD] = C::to(kb[(size_t)(t0 + i / HD) * stride_t + (i % HD)]);
        __syncthreads();
        for (int i = tid; i < G * PA_TILE; i += PA_THREADS) {
            const int g = i / PA_TILE, j = i % PA_TILE;
            float s = -INFINITY;
            if (j < n) {
                float d = 0.f;
#pragma unroll 8
                for (int k = 0; k < HD; ++k) d += sq[g][k] * skv[j][k];
                s = d * scale;
            }
            sp[g][j] = s;
        }
        __syncthreads();
        for (int g = warp; g < G; g += PA_THREADS / 32) {  // online softmax, a warp per head
            const float a = sp[g][lane], b = sp[g][lane + 32];
            const float mt = warp_max(fmaxf(a, b));
            const float mo = sm[g], mn = fmaxf(mo, mt);
            const float ea = expf(a - mn), eb = expf(b - mn);
            sp[g][lane] = ea;
            sp[g][lane + 32] = eb;
            const float sum = warp_sum(ea + eb);
            if (lane == 0) {
                const float corr = mo == -INFINITY ? 0.f : expf(mo - mn);
                sc[g] = corr;
                sl[g] = sl[g] * corr + sum;
                sm[g] = mn;
            }
        }
        for (int i = tid; i < n * HD; i += PA_THREADS)  // V tile over the K tile (scores are done)
            skv[i / HD][i % HD] = C::to(vb[(size_t)(t0 + i / HD) * stride_t + (i % HD)]);
        __syncthreads();
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            if (g < G) {
                float o = acc[g] * sc[g];
                for (int j = 0; j < n; ++j) o += sp[g][j] * skv[j][tid];
                acc[g] = o;
            }
        }
    }
#pragma unroll
    for (int g = 0; g < 8; ++g)
        if (g < G) out[((size_t)p * Hq + h * G + g) * HD + tid] = acc[g] / sl[g];
}

// ------------------------------------------------------------------ launchers
template <int EPI>
cudaError_t launch_tc_gemm(const TGArgs& a, cudaStream_t st) {
    static int attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, TG_SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    const dim3 grid((unsigned)((a.P + TG_BM - 1) / TG_BM), (unsigned)((a.N + TG_BN - 1) / TG_BN));
    tc_gemm_kernel<EPI><<<grid, TG_THREADS, TG_SMEM, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_dequant(int wt, const RMat& m, int rows, int I, __half* W, float* bscale, cudaStream_t st) {
    if (wt == WT_Q6K) dequant_rows_kernel<WT_Q6K><<<rows, 256, 0, st>>>(m, I, W, bscale);
    else dequant_rows_kernel<WT_Q80><<<rows, 256, 0, st>>>(m, I, W, bscale);
    return cudaGetLastError();
}

}  // namespace fence

// C-ABI: the tensor-core GEMM on its own (no reference counterpart; the building block of the
// batched prefill): C[P][N] = A[P][K] . B[N][K]^T, fp16 operands, fp32 result, K % 64 == 0.
extern "C" int fence_gemm_f16(const uint16_t* A, const uint16_t* B, float* C, int P, int N, int K,
                              fence_stream_t stream) {
    using namespace fence;
    if (!A || !B || !C || P <= 0 || N <= 0 || K <= 0 || K % 64)
        return set_error(FENCE_E_ARG, "gemm_f16: need non-null pointers, P, N > 0 and K %% 64 == 0 (P=%d N=%d K=%d)",
                         P, N, K);
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15)
        return set_error(FENCE_E_ALIGN, "gemm_f16: A and B must be 16-byte aligned");
    TGArgs a{};
    a.A = reinterpret_cast<const __half*>(A);
    a.B = reinterpret_cast<const __half*>(B);
    a.P = P;
    a.N = N;
    a.K = K;
    a.C = C;
    a.ldc = N;
    return cuda_status(launch_tc_gemm<TG_EPI_STORE>(a, (cudaStream_t)stream), "gemm_f16 launch");
}
