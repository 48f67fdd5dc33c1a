// attention_static.cu — fence_gqa_attention_static: the drop-in GQA attention without the caller's
// score_buf. It has no counterpart in the reference (gqa_attention, src/kernels/ops.cuh:405-414,
// always takes a caller-allocated score_buf).
//
// Who needs it: callers that hold only the operands of the op and cannot allocate at the call
// site — a foreign-language binding (cgo / JNI / ctypes) that is handed q, the KV cache and the
// output by its runtime and owns no device allocator, or a host loop that must not call
// cudaMalloc per token because cudaMalloc/cudaFree synchronise the device and stall the stream.
// This entry point therefore allocates nothing: the split-context partial results live in a
// fixed file-scope device array.
//
// Contract:
//  * scratch: FENCE_ATTN_STATIC_FLOATS floats (2 MiB) of partials per device. A call needs
//    n_q_heads * chunks * (head_dim + 2) floats when it splits the context into chunks > 1, with
//    chunks = min(max_ctx / (head_dim + 2), ceil(seq_len / 64), 64) — the same split as
//    fence_gqa_attention, so both entry points give identical results. Larger requests are
//    rejected with FENCE_E_SCRATCH before anything is launched (the worst case, 64 chunks, fits
//    up to 63 query heads at head_dim 128 and 31 at head_dim 256).
//  * nothing in the scratch has to start at zero: every partial the merge kernel reads was written
//    by the same call's first kernel, so no clearing is done or needed.
//  * set-up: the first call on each device (with that device current) looks up the array's device
//    address with cudaGetSymbolAddress and caches it per device ordinal; make that first call
//    before any stream capture begins. The cache is not dropped by cudaDeviceReset (after which
//    the module reloads and the array's address may change): a process that resets a device must
//    not call this entry point on that device again.
//  * one scratch per device: calls that overlap in time on the same device (different streams or
//    host threads without ordering) race on the partials. Serialise them on one stream.
#include <mutex>

namespace fence {

static __device__ __align__(256) float g_attn_static_part[FENCE_ATTN_STATIC_FLOATS];

constexpr int ATTN_STATIC_MAX_DEVICES = 64;
static std::mutex g_attn_static_mu;
static float* g_attn_static_ptr[ATTN_STATIC_MAX_DEVICES] = {};

// Device address of this device's scratch (set-up on first use per device).
static int attn_static_scratch(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "gqa_attention_static: cudaGetDevice");
    if (dev < 0 || dev >= ATTN_STATIC_MAX_DEVICES)
        return set_error(FENCE_E_UNSUPPORTED, "gqa_attention_static: device ordinal %d >= %d", dev,
                         ATTN_STATIC_MAX_DEVICES);
    std::lock_guard<std::mutex> lock(g_attn_static_mu);
    if (!g_attn_static_ptr[dev]) {
        float* p = nullptr;
        e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_attn_static_part);
        if (e != cudaSuccess) return cuda_status(e, "gqa_attention_static: cudaGetSymbolAddress");
        if (!p) return set_error(FENCE_E_UNSUPPORTED, "gqa_attention_static: null scratch address");
        g_attn_static_ptr[dev] = p;
    }
    *out = g_attn_static_ptr[dev];
    return FENCE_OK;
}

template <int HD>
static int launch_static_attention(float* out, const float* q, const uint16_t* kc, const uint16_t* vc, int nq,
                                   int nkv, int seq_len, int max_ctx, cudaStream_t st) {
    int nchunk = max_ctx / (HD + 2);
    const int want = (seq_len + 63) / 64;
    if (nchunk > want) nchunk = want;
    if (nchunk > 64) nchunk = 64;
    if (nchunk < 1) nchunk = 1;
    const int clen = (seq_len + nchunk - 1) / nchunk;
    const int n_active = (seq_len + clen - 1) / clen;
    const long long need = (long long)nq * n_active * (HD + 2);
    if (n_active > 1 && need > FENCE_ATTN_STATIC_FLOATS)
        return set_error(FENCE_E_SCRATCH,
                         "gqa_attention_static: %lld floats of partials needed (n_q_heads=%d, %d chunks, "
                         "head_dim=%d), the static scratch holds %d; use fence_gqa_attention with a score_buf",
                         need, nq, n_active, HD, FENCE_ATTN_STATIC_FLOATS);
    float* part = nullptr;
    const int rc = attn_static_scratch(&part);
    if (rc != FENCE_OK) return rc;
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
    a.part = part;
    a.out = out;
    auto kern = attn_partial_kernel<__half, HD, false>;
    constexpr int smem = attn_smem_bytes<__half, HD>();
    FENCE_CUDA_TRY(set_smem(kern, smem));
    kern<<<dim3(n_active, nkv), ATTN_THREADS, smem, st>>>(a);
    FENCE_CUDA_TRY(cudaGetLastError());
    if (n_active > 1) {
        attn_merge_kernel<HD><<<nq, HD, 0, st>>>(part, out, nq, nkv, n_active, n_active);
        FENCE_CUDA_TRY(cudaGetLastError());
    }
    return FENCE_OK;
}

}  // namespace fence

extern "C" int fence_gqa_attention_static(float* attn_out, const float* q, const uint16_t* k_cache,
                                          const uint16_t* v_cache, int head_dim, int n_q_heads, int n_kv_heads,
                                          int seq_len, int max_ctx, fence_stream_t stream) {
    using namespace fence;
    if (!attn_out || !q || !k_cache || !v_cache || n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads ||
        seq_len <= 0 || seq_len > max_ctx)
        return set_error(FENCE_E_ARG, "gqa_attention_static: bad arguments (seq_len=%d max_ctx=%d)", seq_len,
                         max_ctx);
    if (n_q_heads / n_kv_heads > ATTN_MAX_G)
        return set_error(FENCE_E_UNSUPPORTED, "gqa_attention_static: more than %d query heads per kv head",
                         ATTN_MAX_G);
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
        return set_error(FENCE_E_ALIGN, "gqa_attention_static: KV cache must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    switch (head_dim) {
        case 64: return launch_static_attention<64>(attn_out, q, k_cache, v_cache, n_q_heads, n_kv_heads, seq_len, max_ctx, st);
        case 128: return launch_static_attention<128>(attn_out, q, k_cache, v_cache, n_q_heads, n_kv_heads, seq_len, max_ctx, st);
        case 256: return launch_static_attention<256>(attn_out, q, k_cache, v_cache, n_q_heads, n_kv_heads, seq_len, max_ctx, st);
        default:
            return set_error(FENCE_E_UNSUPPORTED, "gqa_attention_static: head_dim %d not in {64,128,256}", head_dim);
    }
}
