// sampler_dev.cu — the reference's nucleus sampler (Qwen3Model::sample_nucleus,
// src/model/qwen3.cu:351-460) on the device. The reference copies the whole logits vector to the
// host every token and sorts all of it; here a few small kernels do the same steps where the
// logits already are and only the chosen id comes back:
//   1. repetition penalty once per occurrence of a token in the history (qwen3.cu:358-369): the
//      first occurrence of each token counts its occurrences and applies them in order, so the
//      float result is the reference's sequence of divisions / multiplications;
//   2. max, min-p cut (qwen3.cu:371-384), entropy of the surviving softmax and the clamped
//      temperature scale (388-412), the softmax at that temperature (414-426): per-CTA partial
//      sums reduced in a fixed order (the reference sums sequentially: the float results differ
//      in the last bits);
//   3. the top_k largest probabilities (428-448 sort the whole vocabulary): each CTA keeps the
//      top_k of its slice (bitonic sorts of 64-bit keys, probability bits above the complemented
//      id, so ties go to the smaller id), one CTA merges the candidates;
//   4. the top-p prefix (sequential float cumulative, as the reference) and the draw
//      (std::discrete_distribution, libstdc++: the kept weights normalised and accumulated in
//      double, the last cumulative set to 1, the first entry whose cumulative is >= u) with the
//      caller's uniform u in [0, 1).
#include "host.h"

namespace fence {

constexpr int SD_NT = 512;
constexpr int SD_MAX_K = 256;    // largest top_k of the device sampler
constexpr int SD_TILE = 2048;    // keys one CTA sorts at a time (its running top_k + new entries)
constexpr int SD_FINAL = 4096;   // candidate keys the merging CTA sorts (CTAs x top_k <= this)
constexpr int SD_MAX_G = 148;

struct SDArgs {
    const float* logits;
    int vocab;
    const int* hist;
    int n_hist;
    float temperature, top_p, min_p, rep_penalty;
    int top_k, dyn;
    double u;
    float* buf;                   // [vocab] penalised logits
    float* part;                  // [4][G] per-CTA partials: max, dyn sum, entropy, softmax sum
    unsigned long long* cand;     // [G][top_k] candidate keys
    int* out;
};

__host__ __device__ inline int sd_ctas(int top_k) {
    int g = SD_FINAL / top_k;
    return g < SD_MAX_G ? (g < 1 ? 1 : g) : SD_MAX_G;
}

// key order = (probability desc, id asc): probabilities are >= 0, so their bits order like them
__device__ __forceinline__ unsigned long long sd_key(float p, int i) {
    return ((unsigned long long)__float_as_uint(p) << 32) | (unsigned)(~(unsigned)i);
}
__device__ __forceinline__ float sd_key_p(unsigned long long k) { return __uint_as_float((unsigned)(k >> 32)); }
__device__ __forceinline__ int sd_key_i(unsigned long long k) { return (int)(~(unsigned)k); }

// descending bitonic sort of n (a power of two) keys in shared memory, by the whole block
__device__ void sd_bitonic_desc(unsigned long long* k, int n) {
    for (int size = 2; size <= n; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int t = threadIdx.x; t < n / 2; t += blockDim.x) {
                const int lo = 2 * stride * (t / stride) + (t % stride), hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long a = k[lo], b = k[hi];
                if ((a < b) == desc) {
                    k[lo] = b;
                    k[hi] = a;
                }
            }
        }
    __syncthreads();
}

__device__ __forceinline__ float sd_block_sum(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    if (threadIdx.x == 0)
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    __syncthreads();
    return t;  // thread 0
}
__device__ __forceinline__ float sd_block_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = -1e30f;
    if (threadIdx.x == 0)
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, red[w]);
    __syncthreads();
    return t;
}
__device__ __forceinline__ void sd_slice(int vocab, int& b, int& e) {
    b = (int)((long long)vocab * blockIdx.x / gridDim.x);
    e = (int)((long long)vocab * (blockIdx.x + 1) / gridDim.x);
}

__global__ void sd_copy_kernel(SDArgs a) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.vocab; i += gridDim.x * blockDim.x)
        a.buf[i] = a.logits[i];
}

// step 1 (one CTA): the first occurrence of each history token applies all of its occurrences
__global__ void sd_penalty_kernel(SDArgs a) {
    if (!(a.rep_penalty > 1.0f)) return;
    for (int h = threadIdx.x; h < a.n_hist; h += blockDim.x) {
        const int t = a.hist[h];
        if (t < 0 || t >= a.vocab) continue;
        bool first = true;
        for (int j = 0; j < h && first; ++j) first = a.hist[j] != t;
        if (!first) continue;
        int m = 0;
        for (int j = h; j < a.n_hist; ++j) m += a.hist[j] == t;
        float v = a.buf[t];
        for (int r = 0; r < m; ++r) v = v > 0 ? v / a.rep_penalty : v * a.rep_penalty;
        a.buf[t] = v;
    }
}

__global__ void sd_max_kernel(SDArgs a) {
    __shared__ float red[32];
    int b, e;
    sd_slice(a.vocab, b, e);
    float m = -1e30f;
    for (int i = b + threadIdx.x; i < e; i += blockDim.x) m = fmaxf(m, a.buf[i]);
    m = sd_block_max(m, red);
    if (threadIdx.x == 0) a.part[blockIdx.x] = m;
}

// every CTA reads the G partials in the same order: identical values everywhere
__device__ __forceinline__ float sd_total_max(const SDArgs& a) {
    float m = -1e30f;
    for (int c = 0; c < (int)gridDim.x; ++c) m = fmaxf(m, a.part[c]);
    return m;
}
__device__ __forceinline__ float sd_total(const float* p, int n) {
    float s = 0.f;
    for (int c = 0; c < n; ++c) s += p[c];
    return s;
}
__device__ __forceinline__ bool sd_survives(float l, float thr, bool cut) { return !(cut && l < thr); }

// step 2a: exp-sum of the min-p survivors (for the entropy)
__global__ void sd_dyn_kernel(SDArgs a) {
    __shared__ float red[32];
    const float mx = sd_total_max(a);
    const bool cut = a.min_p > 0.0f;
    const float thr = mx + logf(a.min_p > 0.0f ? a.min_p : 1.0f);
    int b, e;
    sd_slice(a.vocab, b, e);
    float s = 0.f;
    for (int i = b + threadIdx.x; i < e; i += blockDim.x)
        if (sd_survives(a.buf[i], thr, cut)) s += expf(a.buf[i] - mx);
    s = sd_block_sum(s, red);
    if (threadIdx.x == 0) a.part[gridDim.x + blockIdx.x] = s;
}

// step 2b: entropy of the survivors' softmax (terms with p > 1e-6)
__global__ void sd_entropy_kernel(SDArgs a) {
    __shared__ float red[32];
    const float mx = sd_total_max(a);
    const bool cut = a.min_p > 0.0f;
    const float thr = mx + logf(a.min_p > 0.0f ? a.min_p : 1.0f);
    const float dyn = sd_total(a.part + gridDim.x, gridDim.x);
    int b, e;
    sd_slice(a.vocab, b, e);
    float h = 0.f;
    for (int i = b + threadIdx.x; i < e; i += blockDim.x)
        if (sd_survives(a.buf[i], thr, cut)) {
            const float p = expf(a.buf[i] - mx) / dyn;
            if (p > 1e-6f) h -= p * logf(p);
        }
    h = sd_block_sum(h, red);
    if (threadIdx.x == 0) a.part[2 * gridDim.x + blockIdx.x] = h;
}

// step 2c + 3: softmax numerators at the final temperature, their CTA sum, the CTA's top_k keys
__global__ void __launch_bounds__(SD_NT) sd_prob_kernel(SDArgs a) {
    __shared__ float red[32];
    __shared__ unsigned long long keys[SD_TILE];
    const float mx = sd_total_max(a);
    const bool cut = a.min_p > 0.0f;
    const float thr = mx + logf(a.min_p > 0.0f ? a.min_p : 1.0f);
    float temp = a.temperature;
    if (a.dyn) {
        const float sc = sd_total(a.part + 2 * gridDim.x, gridDim.x) / 2.0f;
        temp *= fminf(fmaxf(sc, 0.5f), 2.0f);
    }
    int b, e;
    sd_slice(a.vocab, b, e);
    const int K = a.top_k;
    float s = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) keys[i] = 0ull;  // below every real key
    for (int t0 = b; t0 < e; t0 += SD_TILE - K) {
        const int n = min(SD_TILE - K, e - t0);
        for (int j = threadIdx.x; j < SD_TILE - K; j += blockDim.x) {
            unsigned long long key = 0ull;
            if (j < n) {
                const int i = t0 + j;
                const float l = a.buf[i];
                const float p = sd_survives(l, thr, cut) ? expf((l - mx) / temp) : 0.0f;
                s += p;
                key = sd_key(p, i);
            }
            keys[K + j] = key;
        }
        sd_bitonic_desc(keys, SD_TILE);  // the first K are the slice's best so far
    }
    s = sd_block_sum(s, red);
    if (threadIdx.x == 0) a.part[3 * gridDim.x + blockIdx.x] = s;
    for (int i = threadIdx.x; i < K; i += blockDim.x) a.cand[(size_t)blockIdx.x * K + i] = keys[i];
}

// step 3 (merge) + 4, one CTA: sort the candidates, top-p prefix, draw
__global__ void __launch_bounds__(1024) sd_final_kernel(SDArgs a, int G) {
    __shared__ unsigned long long keys[SD_FINAL];
    const int K = a.top_k, n = G * K;
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = threadIdx.x; i < np2; i += blockDim.x) keys[i] = i < n ? a.cand[i] : 0ull;
    sd_bitonic_desc(keys, np2);
    if (threadIdx.x != 0) return;
    const float sum = sd_total(a.part + 3 * G, G);
    const int limit = min(K, a.vocab);
    float cum = 0.0f;
    int kept = limit;
    for (int i = 0; i < limit; ++i) {
        cum += sd_key_p(keys[i]) / sum;
        if (cum >= a.top_p) {
            kept = i + 1;
            break;
        }
    }
    int pick = 0;
    if (kept > 1) {
        double w = 0.0;
        for (int i = 0; i < kept; ++i) w += (double)(sd_key_p(keys[i]) / sum);
        double c = 0.0;
        pick = kept - 1;
        for (int i = 0; i < kept - 1; ++i) {
            c += (double)(sd_key_p(keys[i]) / sum) / w;
            if (c >= a.u) {
                pick = i;
                break;
            }
        }
    }
    *a.out = sd_key_i(keys[pick]);
}

}  // namespace fence

using namespace fence;

extern "C" size_t fence_sample_scratch_bytes(int vocab, int top_k) {
    if (vocab <= 0 || top_k < 1 || top_k > SD_MAX_K) return 0;
    const int G = sd_ctas(top_k);
    return ((size_t)vocab * 4 + 255) / 256 * 256 + (size_t)4 * G * 4 + 256 + (size_t)G * top_k * 8;
}

extern "C" int fence_sample_nucleus_dev(const float* logits, int vocab, const int* history, int n_history,
                                        float temperature, float top_p, int top_k, float rep_penalty, float min_p,
                                        int dynamic_temp, double u, void* scratch, size_t scratch_bytes,
                                        int* out_id, fence_stream_t stream) {
    if (!logits || !scratch || !out_id || vocab <= 0 || n_history < 0 || (n_history > 0 && !history))
        return set_error(FENCE_E_ARG, "sample_nucleus_dev: bad arguments");
    if (!(temperature > 0.0f) || top_k < 2 || top_k > SD_MAX_K)
        return set_error(FENCE_E_ARG, "sample_nucleus_dev: temperature must be > 0 and top_k in 2..%d (greedy: "
                         "fence_argmax)", SD_MAX_K);
    if (!(u >= 0.0 && u < 1.0)) return set_error(FENCE_E_ARG, "sample_nucleus_dev: u must be in [0, 1)");
    if (n_history > (1 << 16))  // the penalty step scans the history once per entry
        return set_error(FENCE_E_ARG, "sample_nucleus_dev: more than 65536 history ids");
    const size_t need = fence_sample_scratch_bytes(vocab, top_k);
    if (scratch_bytes < need)
        return set_error(FENCE_E_ARG, "sample_nucleus_dev: scratch of %zu bytes, %zu needed", scratch_bytes, need);
    if (reinterpret_cast<uintptr_t>(scratch) % 256)
        return set_error(FENCE_E_ALIGN, "sample_nucleus_dev: scratch must be 256-byte aligned");
    const int G = sd_ctas(top_k);
    uint8_t* p = static_cast<uint8_t*>(scratch);
    SDArgs a{};
    a.logits = logits;
    a.vocab = vocab;
    a.hist = history;
    a.n_hist = n_history;
    a.temperature = temperature;
    a.top_p = top_p;
    a.min_p = min_p;
    a.rep_penalty = rep_penalty;
    a.top_k = top_k;
    a.dyn = dynamic_temp ? 1 : 0;
    a.u = u;
    a.buf = reinterpret_cast<float*>(p);
    p += ((size_t)vocab * 4 + 255) / 256 * 256;
    a.part = reinterpret_cast<float*>(p);
    p += ((size_t)4 * G * 4 + 255) / 256 * 256;
    a.cand = reinterpret_cast<unsigned long long*>(p);
    a.out = out_id;
    cudaStream_t st = (cudaStream_t)stream;
    sd_copy_kernel<<<G, SD_NT, 0, st>>>(a);
    sd_penalty_kernel<<<1, 1024, 0, st>>>(a);
    sd_max_kernel<<<G, SD_NT, 0, st>>>(a);
    sd_dyn_kernel<<<G, SD_NT, 0, st>>>(a);
    if (a.dyn) sd_entropy_kernel<<<G, SD_NT, 0, st>>>(a);
    sd_prob_kernel<<<G, SD_NT, 0, st>>>(a);
    sd_final_kernel<<<1, 1024, 0, st>>>(a, G);
    return cuda_status(cudaGetLastError(), "sample_nucleus_dev launch");
}
