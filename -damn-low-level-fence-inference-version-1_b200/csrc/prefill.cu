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
// accumulation in tensor memory. CTA tile 128 x 256, K steps of 64 through a 2-stage shared-memory
// ring (97 KB), two CTAs per SM so one CTA's epilogue overlaps the other's MMAs (their two 256-column
// accumulators fill the SM's tensor memory). Warp-specialised: one lane loads each stage's A and B tiles with two TMA tensor copies
// (cp.async.bulk.tensor.2d, 128-byte swizzle, no multicast) completing on the stage's "full"
// mbarrier; one lane issues the stage's four tcgen05.mma (M128 N256 K16, operands described by
// 128-byte-swizzle K-major shared-memory descriptors) and commits them to the stage's "empty"
// mbarrier, which the loading lane waits on before refilling the stage; the last commit signals the
// epilogue. Epilogue: each warp reads its 32 accumulator lanes (rows) with tcgen05.ld, 32 columns at
// a time.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "host.h"
#include "rgemv.cuh"

namespace fence {

constexpr int TG_BM = 128, TG_BN = 256, TG_BK = 64, TG_STAGES = 2, TG_THREADS = 128;
constexpr int TG_A_BYTES = TG_BM * TG_BK * 2;
constexpr int TG_B_BYTES = TG_BN * TG_BK * 2;
constexpr int TG_STAGE_BYTES = TG_A_BYTES + TG_B_BYTES;
constexpr int TG_SMEM = TG_STAGES * TG_STAGE_BYTES + 1024 + 256;  // + 1024-byte alignment slack, barriers
constexpr uint32_t TG_TMEM_COLS = 256;

enum : int { TG_EPI_STORE = 0, TG_EPI_ADD = 1, TG_EPI_SWIGLU = 2 };

struct TGArgs {
    CUtensorMap tmA;      // A [P][K] fp16, box 64 x 128, 128-byte swizzle
    CUtensorMap tmB;      // B [N][K] fp16, box 64 x 256, 128-byte swizzle
    const float* bscale;  // [N] multiplies column n of the product (undoes the weight row scaling); null = 1
    int P, N, K;
    float* C;             // STORE / ADD: [P][ldc]
    int ldc;
    const float* bias;    // STORE: [N], optional
    __half* H;            // SWIGLU: [P][ldh], column n / 2 = silu(column n) * column n + 1 (n even)
    int ldh;
};

// 64-bit shared-memory matrix descriptor, K-major with 128-byte swizzle: start address, leading-
// dimension byte offset (unused for this layout: 16), stride-dimension byte offset 1024 (8 rows of
// 128 bytes), descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t tg_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator, A and B fp16, both K-major, N, M.
__host__ __device__ constexpr uint32_t tg_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tg_tma_load(uint32_t dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float tg_silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int EPI>
__global__ void __launch_bounds__(TG_THREADS, 2) tc_gemm_kernel(const __grid_constant__ TGArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int p0 = blockIdx.x * TG_BM, n0 = blockIdx.y * TG_BN;
    // 1024-byte aligned tiles (the 128-byte swizzle pattern repeats every 8 rows of 128 bytes)
    const uint32_t sraw = smem_u32(smem);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;
    uint8_t* bar_area = smem + (sbase - sraw) + TG_STAGES * TG_STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
    uint64_t* empty = full + TG_STAGES;
    uint64_t* done = empty + TG_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    if (tid == 0) {
        for (int s = 0; s < TG_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.tmB)) : "memory");
    }
    if (warp == 2) {
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
    bool ok = true;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: k-tile kt into stage kt % STAGES once that stage's previous MMAs are done
        for (int kt = 0; kt < nk && ok; ++kt) {
            const int s = kt % TG_STAGES;
            if (kt >= TG_STAGES && !mbar_wait(&empty[s], (uint32_t)((kt / TG_STAGES) - 1) & 1u)) ok = false;
            if (!ok) break;
            const uint32_t st = sbase + (uint32_t)(s * TG_STAGE_BYTES);
            mbar_arrive_expect_tx(&full[s], (uint32_t)TG_STAGE_BYTES);
            tg_tma_load(st, &a.tmA, kt * TG_BK, p0, &full[s]);
            tg_tma_load(st + TG_A_BYTES, &a.tmB, kt * TG_BK, n0, &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = tg_idesc(TG_BM, TG_BN);
        for (int kt = 0; kt < nk && ok; ++kt) {
            const int s = kt % TG_STAGES;
            if (!mbar_wait(&full[s], (uint32_t)(kt / TG_STAGES) & 1u)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = sbase + (uint32_t)(s * TG_STAGE_BYTES), sb = sa + TG_A_BYTES;
#pragma unroll
            for (int t = 0; t < TG_BK / 16; ++t) {  // K = 16 per MMA: 32 bytes further along the swizzled rows
                const uint64_t da = tg_desc(sa + (uint32_t)t * 32u);
                const uint64_t db = tg_desc(sb + (uint32_t)t * 32u);
                const uint32_t acc = (kt > 0 || t > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                    "l"(da), "l"(db), "r"(idesc), "r"(acc)
                    : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&empty[s]))
                         : "memory");
        }
        // every MMA issued so far completes before this arrival
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(done))
                     : "memory");
    }
    __syncwarp();
    if (!mbar_wait(done, 0u)) ok = false;
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
    if (warp == 2)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TG_TMEM_COLS) : "memory");
}

// ------------------------------------------------------------------ weight dequantisation
// Repacked row r of an RMat (rgemv.cuh layouts, one rank: item0 = 0) -> fp16 row r of W[M][K] in the
// natural column order, times 2^e_r with e_r the largest exponent keeping a bound on the row's
// largest |w| below 2^14; bscale[r] = 2^-e_r.
//   Q6_K item i of a row: super-block j = i / 4, half h = (i / 2) & 1, l16 = i & 1; its element
//   (c, e) (column run c < 4, e < 16) is column 256 j + 128 h + 32 c + 16 l16 + e, value
//   d_j * scale_c * (q6 - 32) with q6 = low nibble of byte (c & 1) * 16 + e (its high nibble for
//   c >= 2) | crumb c of byte 32 + e << 4 of the item's 48-byte record.
//   Q8_0 item i: chunk k of 16 int8 at record position k ^ ((i >> 1) & 3); block scales d0, d1.
// One warp per row. The row's scale exponent comes from a bound on its largest |w| taken from the
// block scales alone (Q8_0: max |d| * 127; Q6_K: max over sub-blocks |d * scale| * 32), then every
// lane turns whole items into fp16 with 16-byte loads and stores.
template <int WT>
__global__ void dequant_rows_kernel(RMat m, int I, int rows, __half* __restrict__ W, float* __restrict__ bscale) {
    const int lane = threadIdx.x & 31;
    const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int n = I * 64;
    float bound = 0.f;
    if (WT == WT_Q6K) {
        const uint8_t* dr = m.d + (size_t)r * rg_dbytes_row(WT_Q6K, I, 0);
        const int8_t* sr = reinterpret_cast<const int8_t*>(m.s + (size_t)r * rg_sbytes_row(WT_Q6K, I));
        for (int it = lane; it < I; it += 32) {
            const float d = fabsf(half_bits_to_float((uint32_t)dr[(it >> 2) * 2] | ((uint32_t)dr[(it >> 2) * 2 + 1] << 8)));
            int smax = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) smax = max(smax, abs((int)sr[it * 4 + c]));
            bound = fmaxf(bound, d * (float)smax * 32.f);
        }
    } else {
        const uint16_t* dr = reinterpret_cast<const uint16_t*>(m.d + (size_t)r * I * 4);
        for (int i = lane; i < 2 * I; i += 32) bound = fmaxf(bound, fabsf(half_bits_to_float(dr[i])) * 127.f);
    }
    bound = warp_max(bound);
    int e = 0;
    if (bound > 0.f && isfinite(bound)) {
        int ex;
        frexpf(bound, &ex);  // bound in [2^(ex-1), 2^ex)
        e = 14 - ex;         // every |w| * 2^e < 2^14
    }
    const float sc2 = ldexpf(1.f, e);
    if (lane == 0) bscale[r] = ldexpf(1.f, -e);
    __half* wrow = W + (size_t)r * n;
    for (int it = lane; it < I; it += 32) {
        if (WT == WT_Q6K) {
            // item it: super-block j, half h, l16; run c covers columns 256 j + 128 h + 32 c + 16 l16 + [0, 16)
            const uint4* q = reinterpret_cast<const uint4*>(m.q + ((size_t)r * I + it) * 48);
            const uint4 u0 = q[0], u1 = q[1], u2 = q[2];
            const uint8_t* lo0 = reinterpret_cast<const uint8_t*>(&u0);
            const uint8_t* lo1 = reinterpret_cast<const uint8_t*>(&u1);
            const uint8_t* hi = reinterpret_cast<const uint8_t*>(&u2);
            const uint32_t sw = *reinterpret_cast<const uint32_t*>(m.s + (size_t)r * rg_sbytes_row(WT_Q6K, I) + (size_t)it * 4);
            const uint8_t* dp = m.d + (size_t)r * rg_dbytes_row(WT_Q6K, I, 0) + (size_t)(it >> 2) * 2;
            const float d = half_bits_to_float((uint32_t)dp[0] | ((uint32_t)dp[1] << 8)) * sc2;
            const int col0 = (it >> 2) * 256 + ((it >> 1) & 1) * 128 + (it & 1) * 16;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float ds = d * (float)(int8_t)(sw >> (8 * c));
                const uint8_t* lo = (c & 1) ? lo1 : lo0;
                uint32_t words[8];
#pragma unroll
                for (int e2 = 0; e2 < 16; e2 += 2) {
                    float v[2];
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int nib = c >= 2 ? lo[e2 + k] >> 4 : lo[e2 + k] & 15;
                        const int q6 = nib | (((hi[e2 + k] >> (2 * c)) & 3) << 4);
                        v[k] = ds * (float)(q6 - 32);
                    }
                    const __half2 h2 = __floats2half2_rn(v[0], v[1]);
                    words[e2 / 2] = *reinterpret_cast<const uint32_t*>(&h2);
                }
                uint4* dst = reinterpret_cast<uint4*>(wrow + col0 + c * 32);
                dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
                dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
            }
        } else {
            const uint4* q = reinterpret_cast<const uint4*>(m.q + ((size_t)r * I + it) * 64);
            const uint32_t dw = *reinterpret_cast<const uint32_t*>(m.d + ((size_t)r * I + it) * 4);
            const float d0 = half_bits_to_float(dw & 0xffffu) * sc2, d1 = half_bits_to_float(dw >> 16) * sc2;
            const int f = (it >> 1) & 3;
#pragma unroll
            for (int p2 = 0; p2 < 4; ++p2) {
                const int k = p2 ^ f;  // the chunk stored at record position p2: elements 16 k .. 16 k + 15
                const uint4 u = q[p2];
                const int8_t* b = reinterpret_cast<const int8_t*>(&u);
                const float d = (k >> 1) ? d1 : d0;
                uint32_t words[8];
#pragma unroll
                for (int e2 = 0; e2 < 16; e2 += 2) {
                    const __half2 h2 = __floats2half2_rn(d * (float)b[e2], d * (float)b[e2 + 1]);
                    words[e2 / 2] = *reinterpret_cast<const uint32_t*>(&h2);
                }
                uint4* dst = reinterpret_cast<uint4*>(wrow + it * 64 + 16 * k);
                dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
                dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
            }
        }
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

// Causal GQA attention of the chunk's tokens over the cache (gqa_attention, ops.cuh:320-403) as
// flash-attention tiles on the tensor cores (mma.sync m16n8k16, fp32 accumulators): CTA (block of
// 64 query positions, query head), 4 warps of 16 query rows; 64-key K / V tiles double-buffered in
// shared memory (cp.async, rows padded to 136 elements as in the cache, so fragment loads are
// conflict-free); online softmax per row in registers. Precision: q and the softmax weights P are
// split into a cache-type high part and its remainder, two products summed (~22 bits for fp16,
// ~16 for bf16) while K and V enter exactly as cached — the decode step's attention numerics.
constexpr int FA_BQ = 64, FA_BK = 64, FA_THREADS = 128, FA_RS = 136;

template <typename KVT>
struct FAMma;
template <>
struct FAMma<__half> {
    static __device__ __forceinline__ uint32_t pack(float x, float y) {
        const __half2 h = __floats2half2_rn(x, y);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
    static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <>
struct FAMma<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float x, float y) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
    static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

template <typename KVT>
__global__ void __launch_bounds__(FA_THREADS) prefill_flash_kernel(const float* __restrict__ q, int Hq, int Hkv,
                                                                    const KVT* __restrict__ kc, const KVT* __restrict__ vc,
                                                                    long long stride_h, int stride_t, int pos0, int P,
                                                                    float* __restrict__ out) {
    using MM = FAMma<KVT>;
    constexpr int HD = 128;
    extern __shared__ __align__(128) uint8_t smem[];
    KVT(*sk)[FA_BK * FA_RS] = reinterpret_cast<KVT(*)[FA_BK * FA_RS]>(smem);  // [2] K tiles
    KVT(*sv)[FA_BK * FA_RS] = sk + 2;                                          // [2] V tiles
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int hq = blockIdx.y, h = hq / (Hq / Hkv);
    const int p_lo = blockIdx.x * FA_BQ, r0 = p_lo + warp * 16;
    const int qpos_max = pos0 + min(p_lo + FA_BQ, P) - 1;
    const int nkt = qpos_max / FA_BK + 1;
    const KVT* kb = kc + (size_t)h * stride_h;
    const KVT* vb = vc + (size_t)h * stride_h;
    const float scale = rsqrtf((float)HD);

    // this warp's 16 query rows as A fragments, high part and remainder, 8 steps of 16 dims
    uint32_t qa[8][4], qr[8][4];
    {
        const int ra = min(r0 + g, P - 1), rb = min(r0 + g + 8, P - 1);
        const float* qa_row = q + ((size_t)ra * Hq + hq) * HD;
        const float* qb_row = q + ((size_t)rb * Hq + hq) * HD;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int c0 = ks * 16 + 2 * t;
            const float2 x0 = *reinterpret_cast<const float2*>(qa_row + c0);
            const float2 x1 = *reinterpret_cast<const float2*>(qb_row + c0);
            const float2 x2 = *reinterpret_cast<const float2*>(qa_row + c0 + 8);
            const float2 x3 = *reinterpret_cast<const float2*>(qb_row + c0 + 8);
            const float2 xs[4] = {x0, x1, x2, x3};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                qa[ks][i] = MM::pack(xs[i].x, xs[i].y);
                qr[ks][i] = MM::pack(xs[i].x - MM::round(xs[i].x), xs[i].y - MM::round(xs[i].y));
            }
        }
    }
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    const int qpos[2] = {pos0 + r0 + g, pos0 + r0 + g + 8};

    auto load_tile = [&](int kt, int buf) {  // keys past the block's last query are zero-filled
        for (int c = tid; c < FA_BK * 16; c += FA_THREADS) {
            const int row = c >> 4, ch = c & 15, key = kt * FA_BK + row;
            const bool ok = key <= qpos_max;
            const uint32_t dk = smem_u32(&sk[buf][row * FA_RS + ch * 8]);
            const uint32_t dv = smem_u32(&sv[buf][row * FA_RS + ch * 8]);
            const KVT* srck = ok ? kb + (size_t)key * stride_t + ch * 8 : kb;
            const KVT* srcv = ok ? vb + (size_t)key * stride_t + ch * 8 : vb;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dk), "l"(srck), "r"(ok ? 16 : 0) : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dv), "l"(srcv), "r"(ok ? 16 : 0) : "memory");
        }
        cp_async_commit();
    };
    load_tile(0, 0);
    for (int kt = 0; kt < nkt; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < nkt) load_tile(kt + 1, buf ^ 1);
        else cp_async_commit();
        cp_async_wait_group<1>();
        __syncthreads();
        const KVT* K = sk[buf];
        const KVT* V = sv[buf];
        // ---- scores of 64 keys: 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
            const KVT* krow = K + (nt * 8 + g) * FA_RS + 2 * t;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + ks * 16);
                const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + ks * 16 + 8);
                MM::mma(s[nt], qa[ks], b0, b1);
                MM::mma(s[nt], qr[ks], b0, b1);
            }
        }
        // ---- causal mask, scale, online softmax (rows g and g + 8 of the warp)
        float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int kp = kt * FA_BK + nt * 8 + 2 * t + (e & 1);
                const float v = kp <= qpos[e >> 1] ? s[nt][e] * scale : -INFINITY;
                s[nt][e] = v;
                mt[e >> 1] = fmaxf(mt[e >> 1], v);
            }
        }
        float corr[2], ls[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 1));
            mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 2));
            const float mn = fmaxf(mrow[r], mt[r]);
            corr[r] = mrow[r] == -INFINITY ? 0.f : expf(mrow[r] - mn);
            mrow[r] = mn;
            ls[r] = 0.f;
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float pv = s[nt][e] == -INFINITY ? 0.f : expf(s[nt][e] - mrow[e >> 1]);
                s[nt][e] = pv;
                ls[e >> 1] += pv;
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
            ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
            lrow[r] = lrow[r] * corr[r] + ls[r];
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            o[n][0] *= corr[0];
            o[n][1] *= corr[0];
            o[n][2] *= corr[1];
            o[n][3] *= corr[1];
        }
        // ---- O += P . V: 4 steps of 16 keys, B fragments by ldmatrix.trans from the V tile
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t pa[4], pr[4];
            const float e0[4] = {s[2 * j][0], s[2 * j][2], s[2 * j + 1][0], s[2 * j + 1][2]};
            const float e1[4] = {s[2 * j][1], s[2 * j][3], s[2 * j + 1][1], s[2 * j + 1][3]};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                pa[i] = MM::pack(e0[i], e1[i]);
                pr[i] = MM::pack(e0[i] - MM::round(e0[i]), e1[i] - MM::round(e1[i]));
            }
            const int mi = lane >> 3, ri = lane & 7;
            const KVT* vrow = V + (j * 16 + (mi & 1) * 8 + ri) * FA_RS + (mi >> 1) * 8;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                uint32_t b[4];
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                             : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                             : "r"(smem_u32(vrow + u * 16)));
                MM::mma(o[2 * u], pa, b[0], b[1]);
                MM::mma(o[2 * u], pr, b[0], b[1]);
                MM::mma(o[2 * u + 1], pa, b[2], b[3]);
                MM::mma(o[2 * u + 1], pr, b[2], b[3]);
            }
        }
        __syncthreads();  // this buffer is refilled two tiles later
    }
    // ---- normalised rows out
    const int rows[2] = {r0 + g, r0 + g + 8};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        if (rows[r] >= P) continue;
        const float inv = 1.f / lrow[r];
        float* orow = out + ((size_t)rows[r] * Hq + hq) * HD + 2 * t;
#pragma unroll
        for (int n = 0; n < 16; ++n)
            *reinterpret_cast<float2*>(orow + n * 8) = make_float2(o[n][2 * r] * inv, o[n][2 * r + 1] * inv);
    }
}

// ------------------------------------------------------------------ launchers
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda dependency).
static PFN_cuTensorMapEncodeTiled tg_encode_fn() {
    static PFN_cuTensorMapEncodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
    }
    return fn;
}

// 2-D fp16 row-major [rows][K] (16-byte aligned base, K % 64 == 0), box 64 x box_rows, 128-byte
// swizzle, out-of-range rows read as zero.
static bool tg_tensor_map(CUtensorMap* tm, const __half* base, int rows, int K, int box_rows) {
    PFN_cuTensorMapEncodeTiled enc = tg_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Fills a.tmA / a.tmB from the operand pointers and launches. A, B: 16-byte aligned, K % 64 == 0.
template <int EPI>
cudaError_t launch_tc_gemm(TGArgs& a, const __half* A, const __half* B, cudaStream_t st) {
    static int attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, TG_SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    if (!tg_tensor_map(&a.tmA, A, a.P, a.K, TG_BM) || !tg_tensor_map(&a.tmB, B, a.N, a.K, TG_BN))
        return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((a.P + TG_BM - 1) / TG_BM), (unsigned)((a.N + TG_BN - 1) / TG_BN));
    tc_gemm_kernel<EPI><<<grid, TG_THREADS, TG_SMEM, st>>>(a);
    return cudaGetLastError();
}

constexpr int FA_SMEM = 4 * FA_BK * FA_RS * 2;  // K and V tiles, double-buffered

template <typename KVT>
cudaError_t launch_prefill_attn(const float* q, int Hq, int Hkv, const KVT* kc, const KVT* vc, long long stride_h,
                                int stride_t, int pos0, int P, float* out, cudaStream_t st) {
    static int attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(prefill_flash_kernel<KVT>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    prefill_flash_kernel<KVT><<<dim3((P + FA_BQ - 1) / FA_BQ, Hq), FA_THREADS, FA_SMEM, st>>>(q, Hq, Hkv, kc, vc, stride_h,
                                                                                          stride_t, pos0, P, out);
    return cudaGetLastError();
}

cudaError_t launch_dequant(int wt, const RMat& m, int rows, int I, __half* W, float* bscale, cudaStream_t st) {
    const unsigned blocks = (unsigned)((rows + 7) / 8);  // 8 warps (rows) per CTA
    if (wt == WT_Q6K) dequant_rows_kernel<WT_Q6K><<<blocks, 256, 0, st>>>(m, I, rows, W, bscale);
    else dequant_rows_kernel<WT_Q80><<<blocks, 256, 0, st>>>(m, I, rows, W, bscale);
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
    a.P = P;
    a.N = N;
    a.K = K;
    a.C = C;
    a.ldc = N;
    return cuda_status(launch_tc_gemm<TG_EPI_STORE>(a, reinterpret_cast<const __half*>(A), reinterpret_cast<const __half*>(B),
                                                    (cudaStream_t)stream),
                       "gemm_f16 launch");
}
