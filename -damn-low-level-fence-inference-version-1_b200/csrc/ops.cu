// ops.cu — drop-in replacements for the reference's src/kernels/ops.cuh launchers, plus the
// C-ABI error plumbing. The engine does not call these (it fuses the same math into the GEMV and
// attention kernels); they exist so reference call sites and tests can use the ops one by one.
#include <cmath>
#include <string>

#include "attention.cuh"
#include "host.h"

namespace fence {

static thread_local std::string t_last_error;

int set_error(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return FENCE_OK;
    set_error((int)e, "%s: %s", what, cudaGetErrorString(e));
    return (int)e;
}

// ------------------------------------------------------------------ kernels
// RMSNorm over n values with one CTA (out may alias x: all reads finish before the first write).
__global__ void rms_norm_kernel(float* out, const float* x, const float* __restrict__ w, int n, float eps) {
    __shared__ float red[32];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i] * x[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += red[k];
    const float r = rsqrtf(tot / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = w[i] * x[i] * r;
}

// One warp per head.
__global__ void rms_norm_per_head_kernel(float* x, const float* __restrict__ w, int n_heads, int hd, float eps) {
    const int head = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (head >= n_heads) return;
    float* v = x + (size_t)head * hd;
    float s = 0.f;
    for (int d = lane; d < hd; d += 32) s += v[d] * v[d];
    s = warp_sum(s);
    const float r = rsqrtf(s / (float)hd + eps);
    for (int d = lane; d < hd; d += 32) v[d] = w[d] * v[d] * r;
}

// NeoX rotary embedding; the angle pos * base^(-2i/hd) and its sine/cosine are evaluated in double
// precision and rounded once to float.
__global__ void rope_kernel(float* q, float* k, int hd, int nq, int nkv, int pos, float base) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const int half = hd / 2;
    const int total = (nq + nkv) * half;
    if (tid >= total) return;
    float* v = (tid < nq * half) ? q : k;
    const int t = (tid < nq * half) ? tid : tid - nq * half;
    const int head = t / half, i = t - head * half;
    const double freq = pow((double)base, -2.0 * (double)i / (double)hd);
    double s, c;
    sincos((double)pos * freq, &s, &c);
    const float cf = (float)c, sf = (float)s;
    float* p = v + (size_t)head * hd;
    const float a = p[i], b = p[i + half];
    p[i] = a * cf - b * sf;
    p[i + half] = a * sf + b * cf;
}

__global__ void silu_mul_kernel(float* out, const float* gate, const float* up, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = silu_mul(gate[i], up[i]);
}
__global__ void residual_add_kernel(float* x, const float* __restrict__ r, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += r[i];
}
__global__ void f32_to_f16_kernel(__half* out, const float* __restrict__ in, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(in[i]);
}
__global__ void f16_to_f32_kernel(float* out, const __half* __restrict__ in, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __half2float(in[i]);
}
__global__ void store_kv_kernel(__half* kc, __half* vc, const float* __restrict__ k, const float* __restrict__ v,
                                int pos, int kv_dim) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= kv_dim) return;
    kc[(size_t)pos * kv_dim + i] = __float2half_rn(k[i]);
    vc[(size_t)pos * kv_dim + i] = __float2half_rn(v[i]);
}

// Softmax with one CTA (ops.cuh:207-246): max, exp-sum, normalise.
__global__ void softmax_kernel(float* x, int n) {
    __shared__ float red[32];
    __shared__ float bc;
    float m = -1e30f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = -1e30f;
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t = fmaxf(t, red[k]);
        bc = t;
    }
    __syncthreads();
    const float mx = bc;
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(x[i] - mx);
        x[i] = e;
        s += e;
    }
    s = warp_sum(s);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
        bc = t;
    }
    __syncthreads();
    const float inv = 1.0f / bc;
    for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] *= inv;
}

// argmax with the reference's tie order, one CTA.
__global__ void argmax_kernel(const float* __restrict__ x, int* result, int n) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = 0.f;
    int bi = -1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (argmax_better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && argmax_better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float gv = 0.f;
        int gi = -1;
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k)
            if (si[k] >= 0 && argmax_better(sv[k], si[k], gv, gi)) {
                gv = sv[k];
                gi = si[k];
            }
        *result = gi < 0 ? 0 : gi;
    }
}

template <typename F>
static cudaError_t set_smem(F kern, int bytes) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int HD>
static int launch_dropin_attention(float* out, const float* q, const uint16_t* kc, const uint16_t* vc,
                                   int nq, int nkv, int seq_len, int max_ctx, float* score_buf,
                                   cudaStream_t st) {
    const int G = nq / nkv;
    // split the context so the partials fit the caller's score_buf (nq * max_ctx floats)
    int nchunk = max_ctx / (HD + 2);
    const int want = (seq_len + 63) / 64;
    if (nchunk > want) nchunk = want;
    if (nchunk > 64) nchunk = 64;
    if (nchunk < 1) nchunk = 1;
    const int clen = (seq_len + nchunk - 1) / nchunk;
    const int n_active = (seq_len + clen - 1) / clen;
    AttnArgs a{};
    a.q = q;
    a.kc = kc;
    a.vc = vc;
    a.stride_t = (long long)nkv * HD;
    a.stride_h = HD;
    a.n_q_heads = nq;
    a.n_kv_heads = nkv;
    a.seq_len = seq_len;
    a.nchunk = n_active;
    a.chunk_fixed = clen;
    a.part = score_buf;
    a.out = out;
    auto kern = attn_partial_kernel<__half, HD, false>;
    constexpr int smem = attn_smem_bytes<__half, HD>();
    FENCE_CUDA_TRY(set_smem(kern, smem));
    kern<<<dim3(n_active, nkv), ATTN_THREADS, smem, st>>>(a);
    FENCE_CUDA_TRY(cudaGetLastError());
    if (n_active > 1) {
        attn_merge_kernel<HD><<<nq, HD, 0, st>>>(score_buf, out, nq, nkv, n_active, n_active);
        FENCE_CUDA_TRY(cudaGetLastError());
    }
    (void)G;
    return FENCE_OK;
}

}  // namespace fence

using namespace fence;

// ------------------------------------------------------------------ C-ABI
extern "C" const char* fence_last_error(void) { return t_last_error.c_str(); }

extern "C" int fence_device_error(void) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_status(e, "fence_device_error: synchronize");
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof v);
    if (e != cudaSuccess) return cuda_status(e, "fence_device_error: read");
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero);
    return v;
}

#define ST ((cudaStream_t)stream)
#define LAUNCH_OK(what) return cuda_status(cudaGetLastError(), what)

extern "C" int fence_rms_norm(float* out, const float* x, const float* w, int n, float eps, fence_stream_t stream) {
    if (!out || !x || !w || n <= 0) return set_error(FENCE_E_ARG, "rms_norm: bad arguments (n=%d)", n);
    rms_norm_kernel<<<1, 1024, 0, ST>>>(out, x, w, n, eps);
    LAUNCH_OK("rms_norm");
}
extern "C" int fence_rms_norm_inplace(float* x, const float* w, int n, float eps, fence_stream_t stream) {
    return fence_rms_norm(x, x, w, n, eps, stream);
}
extern "C" int fence_rms_norm_per_head(float* x, const float* w, int n_heads, int head_dim, float eps,
                                       fence_stream_t stream) {
    if (!x || !w || n_heads <= 0 || head_dim <= 0)
        return set_error(FENCE_E_ARG, "rms_norm_per_head: bad arguments");
    rms_norm_per_head_kernel<<<(n_heads + 3) / 4, 128, 0, ST>>>(x, w, n_heads, head_dim, eps);
    LAUNCH_OK("rms_norm_per_head");
}
extern "C" int fence_apply_rope(float* q, float* k, int head_dim, int n_q_heads, int n_kv_heads, int pos,
                                float freq_base, fence_stream_t stream) {
    if (!q || !k || head_dim <= 0 || head_dim % 2 || n_q_heads < 0 || n_kv_heads < 0 || pos < 0)
        return set_error(FENCE_E_ARG, "apply_rope: bad arguments");
    const int total = (n_q_heads + n_kv_heads) * (head_dim / 2);
    if (total == 0) return FENCE_OK;
    rope_kernel<<<(total + 255) / 256, 256, 0, ST>>>(q, k, head_dim, n_q_heads, n_kv_heads, pos, freq_base);
    LAUNCH_OK("apply_rope");
}
extern "C" int fence_silu_elementwise_mul(float* out, const float* gate, const float* up, int n,
                                          fence_stream_t stream) {
    if (!out || !gate || !up || n < 0) return set_error(FENCE_E_ARG, "silu_elementwise_mul: bad arguments");
    if (n == 0) return FENCE_OK;
    silu_mul_kernel<<<(n + 255) / 256, 256, 0, ST>>>(out, gate, up, n);
    LAUNCH_OK("silu_elementwise_mul");
}
extern "C" int fence_residual_add(float* x, const float* residual, int n, fence_stream_t stream) {
    if (!x || !residual || n < 0) return set_error(FENCE_E_ARG, "residual_add: bad arguments");
    if (n == 0) return FENCE_OK;
    residual_add_kernel<<<(n + 255) / 256, 256, 0, ST>>>(x, residual, n);
    LAUNCH_OK("residual_add");
}
extern "C" int fence_softmax(float* x, int n, fence_stream_t stream) {
    if (!x || n <= 0) return set_error(FENCE_E_ARG, "softmax: bad arguments");
    softmax_kernel<<<1, 1024, 0, ST>>>(x, n);
    LAUNCH_OK("softmax");
}
extern "C" int fence_f32_to_f16(uint16_t* out, const float* in, int n, fence_stream_t stream) {
    if (!out || !in || n < 0) return set_error(FENCE_E_ARG, "f32_to_f16: bad arguments");
    if (n == 0) return FENCE_OK;
    f32_to_f16_kernel<<<(n + 255) / 256, 256, 0, ST>>>(reinterpret_cast<__half*>(out), in, n);
    LAUNCH_OK("f32_to_f16");
}
extern "C" int fence_float_to_half(uint16_t* out, const float* in, int n, fence_stream_t stream) {
    return fence_f32_to_f16(out, in, n, stream);
}
extern "C" int fence_half_to_float(float* out, const uint16_t* in, int n, fence_stream_t stream) {
    if (!out || !in || n < 0) return set_error(FENCE_E_ARG, "half_to_float: bad arguments");
    if (n == 0) return FENCE_OK;
    f16_to_f32_kernel<<<(n + 255) / 256, 256, 0, ST>>>(out, reinterpret_cast<const __half*>(in), n);
    LAUNCH_OK("half_to_float");
}
extern "C" int fence_store_kv(uint16_t* k_cache, uint16_t* v_cache, const float* k, const float* v, int pos,
                              int kv_dim, int max_ctx, fence_stream_t stream) {
    if (!k_cache || !v_cache || !k || !v || kv_dim <= 0 || pos < 0 || pos >= max_ctx)
        return set_error(FENCE_E_ARG, "store_kv: bad arguments (pos=%d max_ctx=%d)", pos, max_ctx);
    store_kv_kernel<<<(kv_dim + 255) / 256, 256, 0, ST>>>(reinterpret_cast<__half*>(k_cache),
                                                          reinterpret_cast<__half*>(v_cache), k, v, pos, kv_dim);
    LAUNCH_OK("store_kv");
}
extern "C" int fence_gqa_attention(float* attn_out, const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                   int head_dim, int n_q_heads, int n_kv_heads, int seq_len, int max_ctx,
                                   float* score_buf, fence_stream_t stream) {
    if (!attn_out || !q || !k_cache || !v_cache || !score_buf || n_q_heads <= 0 || n_kv_heads <= 0 ||
        n_q_heads % n_kv_heads || seq_len <= 0 || seq_len > max_ctx)
        return set_error(FENCE_E_ARG, "gqa_attention: bad arguments (seq_len=%d max_ctx=%d)", seq_len, max_ctx);
    if (n_q_heads / n_kv_heads > ATTN_MAX_G)
        return set_error(FENCE_E_UNSUPPORTED, "gqa_attention: more than %d query heads per kv head", ATTN_MAX_G);
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
        return set_error(FENCE_E_ALIGN, "gqa_attention: KV cache must be 16-byte aligned");
    switch (head_dim) {
        case 64: return launch_dropin_attention<64>(attn_out, q, k_cache, v_cache, n_q_heads, n_kv_heads, seq_len, max_ctx, score_buf, ST);
        case 128: return launch_dropin_attention<128>(attn_out, q, k_cache, v_cache, n_q_heads, n_kv_heads, seq_len, max_ctx, score_buf, ST);
        case 256: return launch_dropin_attention<256>(attn_out, q, k_cache, v_cache, n_q_heads, n_kv_heads, seq_len, max_ctx, score_buf, ST);
        default: return set_error(FENCE_E_UNSUPPORTED, "gqa_attention: head_dim %d not in {64,128,256}", head_dim);
    }
}
extern "C" int fence_argmax(const float* x, int* result, int n, fence_stream_t stream) {
    if (!x || !result || n <= 0) return set_error(FENCE_E_ARG, "argmax: bad arguments");
    argmax_kernel<<<1, 1024, 0, ST>>>(x, result, n);
    LAUNCH_OK("argmax");
}
