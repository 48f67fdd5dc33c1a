// engine.cu — the batch-1 decode engine: the reference's Qwen3Model (src/model/qwen3.h:115-155,
// src/model/qwen3.cu:47-519) rebuilt around the fused sm_100a kernels.
//
// Token step (reference order qwen3.cu:241-341, ~16 launches and ~9 device syncs per layer there):
//   embed(token read from device state)
//   per layer:
//     1. QKV GEMV      prologue RMSNorm(attn_norm) [+fp16 rounding for Q6_K]; q, k, v in one launch
//     2. attention     q/k-norm + RoPE + KV-cache store + split-context attention + merge
//     3. O GEMV        prologue fp32 -> [fp16]; epilogue hidden += (residual add)
//     4. gate/up GEMV  prologue RMSNorm(ffn_norm); epilogue SwiGLU -> act (fp16 for a Q6_K down)
//     5. down GEMV     epilogue hidden +=
//   LM head (tied token_embd, Q8_0)  prologue RMSNorm(output_norm); epilogue logits + argmax; the
//   last CTA writes the sampled id and pos+1 into the device decode state.
// Five launches per layer, chained with programmatic dependent launch so each kernel streams its
// weights while the previous one drains, all captured once in a CUDA graph that is replayed per
// token with no host synchronisation.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "attention.cuh"
#include "gemv.cuh"
#include "gguf.h"
#include "rgemv.cuh"
#include "step.cuh"
#include "host.h"

namespace fence {

size_t rmat_bytes(int wt, long long rows, int K, int iph = 0);
RMat rmat_carve(int wt, long long rows, int K, uint8_t* base, int iph = 0);
cudaError_t rmat_fill(int wt, const uint8_t* src, long long rows, int K, const RMat& m, long long dst_row0,
                      int dst_stride, cudaStream_t st, int src_K = 0, int item0 = 0);
RGemvPlan plan_rgemv(RGemvArgs& a, int sms, int smem_budget);
unsigned long long sk_tile_plan(int wt, int I, int Mv, int dual, int G, int RB, int CI, unsigned long long* tcta);
cudaError_t sk_retile(int wt, const RMat& m, int I, int Mv, int dual, int G, int RB, int CI,
                      const unsigned long long* d_tcta, uint8_t* dst, cudaStream_t st);
cudaError_t rgemv_dispatch(int xm, int epi, const RGemvArgs& a, const RGemvPlan& P, cudaStream_t st);

cudaError_t launch_dequant(int wt, const RMat& m, int rows, int I, __half* W, float* bscale, cudaStream_t st);
int host_sample_nucleus(const float* logits, int vocab, const int* history, int n_history, float temperature,
                        float top_p, int top_k, float rep_penalty, float min_p, bool dynamic_temp,
                        std::mt19937& rng);

struct LayerW {
    // linears: the GGUF rows in the host file mapping (streamed to the device per layer at load)
    const uint8_t *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    const uint8_t *gate = nullptr, *up = nullptr, *down = nullptr;
    int t_qkv = 14, t_o = 14, t_gu = 14, t_down = 14;  // GGML type ids
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    const float *q_bias = nullptr, *k_bias = nullptr, *v_bias = nullptr;
    const float* router = nullptr;  // sparse MoE: ffn_gate_inp [n_exp][H] fp32; gate/up/down are then the
                                    // [K, M, n_exp] expert tensors (expert e's rows contiguous)
};

// One GEMV phase of the token step over repacked weights.
struct RPhase {
    RGemvArgs a;
    RGemvPlan p;
    int xm, epi;
};

struct LayerLaunch {
    RPhase qkv, o, gu, down;  // QKV fused into one matrix, gate/up rows interleaved
    AttnArgs attn;
};

}  // namespace fence

using namespace fence;

struct fence_model {
    fence_config cfg{};
    fence_load_opts opts{};
    int dev = 0;
    cudaStream_t stream = nullptr;
    GGUFFile gguf;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    std::vector<LayerW> layers;
    const uint8_t* tok_embd = nullptr;
    const float* out_norm = nullptr;
    void* kcache = nullptr;
    void* vcache = nullptr;
    float *hidden = nullptr, *qkv = nullptr, *attn_out = nullptr, *logits = nullptr, *attn_part = nullptr;
    void* act = nullptr;
    unsigned int* counters = nullptr;  // [Hkv] attention + [1] LM head
    float* lm_val = nullptr;
    int* lm_idx = nullptr;
    DecodeState* state = nullptr;
    int* token_log = nullptr;
    int token_log_cap = 0;
    float2* rope = nullptr;
    DecodeState* h_state = nullptr;  // pinned staging ring
    int h_state_n = 0;
    int* h_token = nullptr;          // pinned
    DecodeState* h_out = nullptr;    // pinned: the device state after the last fence_forward
    int fwd_valid = 0;               // h_out holds the state of the step that produced m->logits
    std::vector<LayerLaunch> launches;
    RPhase lm{};
    uint8_t* rarena = nullptr;      // repacked linears (rgemv.cuh layouts; freed once the step kernel's tiles exist)
    uint8_t* tarena = nullptr;      // the step kernel's tiled linears
    unsigned long long* d_tcta = nullptr;  // per GEMV phase, per CTA: first tile offset
    // persistent token-step kernel (step.cuh)
    int use_step = 0;
    std::vector<SPhase> h_phases;
    SPhase* d_phases = nullptr;
    unsigned long long* d_bar = nullptr;
    StepArgs sargs{};
    StepPlan splan{};
    float* qkv_bias = nullptr;      // fused q|k|v bias when the model has any
    int attn_nchunk = 0;            // per-phase attention kernel: chunks per KV head
    int step_nchunk = 0;            // step kernel: chunks per KV head its partials hold
    // tensor parallel (tp_n > 1): this rank's shard; the exchange buffer is shared with the peers
    int tp_n = 1, tp_rank = 0, vocab0 = 0, vocab_n = 0;
    float* hidden_b = nullptr;      // residual stream after the odd reductions
    uint8_t* xbuf = nullptr;        // this rank's exchange buffer (sk_xb_bytes)
    uint8_t* xpeer[SK_TP_MAX] = {};  // every rank's exchange buffer as mapped here (own = xbuf)
    unsigned long long* tp_launch = nullptr;
    int tp_connected = 0;
    // sparse MoE FFN: local experts [e_lo, e_lo + e_n) (all of them unless expert parallel), each
    // with its repacked gate/up and down matrices ([layer][local expert])
    int moe = 0, moe_ep = 0, e_lo = 0, e_n = 0;
    std::vector<RMat> moe_gu, moe_dn;
    float* moe_acc = nullptr;       // tensor parallel: the expert slots' partial rows before the last slot
    // batched prefill (prefill.cu): the repacked row-major weights are kept for it (one rank, dense
    // FFN, opts.prefill); its scratch is allocated on the first call for pf_cap tokens per chunk
    int prefill_ok = 0;
    int pf_cap = 0;
    int* pf_tok = nullptr;
    float *pf_hidden = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_attn = nullptr, *pf_bscale = nullptr;
    __half *pf_x16 = nullptr, *pf_act = nullptr, *pf_w = nullptr;
    // device nucleus sampler (allocated on its first use)
    void* samp_scratch = nullptr;
    size_t samp_bytes = 0;
    int* samp_hist = nullptr;
    int samp_hist_cap = 0;
    int* samp_out = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t gexec = nullptr;
    std::mt19937 rng{0x5eed};
    std::vector<float> h_logits;
};

namespace {

// Streaming host -> device upload of GGUF data (the reference copies tensor by tensor with
// synchronous pageable cudaMemcpy, qwen3.cu:104-111). A ring of pinned staging buffers: worker
// threads copy the next chunk out of the file mapping (taking the page faults of a cold file in
// parallel) while the DMA engine moves the previous chunks; each buffer is reused once its copy has
// completed (an event per buffer). A piece is `rows` rows of `width` bytes, `pitch` bytes apart in
// the file, packed row after row at the destination: a whole tensor, a rank's rows of it, or a
// rank's column slice of every row. Copies are ordered on the stream, so kernels enqueued after them
// on that stream read the data.
struct Uploader {
    static constexpr int NB = 4;
    static constexpr size_t CHUNK = 32u << 20;
    cudaStream_t st = nullptr;
    uint8_t* pin[NB] = {};
    cudaEvent_t ev[NB] = {};
    bool busy[NB] = {};
    int cur = 0;
    int threads = 1;
    size_t bytes = 0;

    int init(cudaStream_t s) {
        st = s;
        threads = (int)std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
        for (int i = 0; i < NB; ++i) {
            if (cudaMallocHost(&pin[i], CHUNK) != cudaSuccess || cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess)
                return set_error(FENCE_E_NOMEM, "upload: pinned staging allocation failed");
        }
        return FENCE_OK;
    }
    ~Uploader() {
        for (int i = 0; i < NB; ++i) {
            if (ev[i]) {
                cudaEventSynchronize(ev[i]);
                cudaEventDestroy(ev[i]);
            }
            if (pin[i]) cudaFreeHost(pin[i]);
        }
    }
    // host side of one chunk: rows [r0, r1) of the piece, or bytes [b0, b1) of a single-row piece
    void pack(uint8_t* dst, const uint8_t* src, size_t pitch, size_t width, size_t r0, size_t r1) const {
        const size_t n = r1 - r0;
        auto work = [&](size_t a, size_t b) {
            if (width == pitch) {
                std::memcpy(dst + a * width, src + (r0 + a) * pitch, (b - a) * width);
            } else {
                for (size_t r = a; r < b; ++r) std::memcpy(dst + r * width, src + (r0 + r) * pitch, width);
            }
        };
        const int nt = (int)std::min<size_t>((size_t)threads, (n * width) >> 22 ? n : 1);  // threads for >= 4 MB
        if (nt <= 1) {
            work(0, n);
            return;
        }
        std::vector<std::thread> th;
        for (int t = 0; t < nt; ++t) th.emplace_back(work, n * t / nt, n * (t + 1) / nt);
        for (auto& x : th) x.join();
    }
    int put(uint8_t* dst, const uint8_t* src, size_t pitch, size_t width, size_t rows) {
        if (rows == 1) {  // one contiguous range: chunk it as rows of 64 KB (and a remainder)
            const size_t unit = 65536, full = width / unit, tail = width - full * unit;
            if (full) {
                const int rc = put_rows(dst, src, unit, unit, full);
                if (rc) return rc;
            }
            return tail ? put_rows(dst + full * unit, src + full * unit, tail, tail, 1) : FENCE_OK;
        }
        return put_rows(dst, src, pitch, width, rows);
    }
    int put_rows(uint8_t* dst, const uint8_t* src, size_t pitch, size_t width, size_t rows) {
        if (width > CHUNK) return set_error(FENCE_E_UNSUPPORTED, "upload: a row of %zu bytes exceeds the staging chunk", width);
        const size_t per = CHUNK / width;
        for (size_t r0 = 0; r0 < rows; r0 += per) {
            const size_t r1 = std::min(rows, r0 + per);
            if (busy[cur] && cudaEventSynchronize(ev[cur]) != cudaSuccess)
                return set_error(FENCE_E_NOMEM, "upload: staging copy failed");
            pack(pin[cur], src, pitch, width, r0, r1);
            if (cudaMemcpyAsync(dst + r0 * width, pin[cur], (r1 - r0) * width, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaEventRecord(ev[cur], st) != cudaSuccess)
                return set_error(FENCE_E_NOMEM, "upload: host to device copy failed");
            busy[cur] = true;
            cur = (cur + 1) % NB;
            bytes += (r1 - r0) * width;
        }
        return FENCE_OK;
    }
};

// Bytes of the blocks covering input columns [c0, c1) of a row of a Q6_K (super-blocks of 256) or
// Q8_0 (blocks of 32) matrix, and the first covering block.
struct ColCover {
    size_t b0, nb, bytes;
};
ColCover col_cover(int ggml_type, uint64_t c0, uint64_t c1) {
    const uint64_t bs = ggml_type == 14 ? 256 : 32, ts = ggml_type == 14 ? 210 : 34;
    ColCover cc;
    cc.b0 = c0 / bs;
    cc.nb = (c1 + bs - 1) / bs - cc.b0;
    cc.bytes = cc.nb * ts;
    return cc;
}

int step_attn_solo() {
#ifdef FENCE_TUNE_ENV
    if (const char* e = getenv("FENCE_ATTN_SOLO")) return atoi(e);
#endif
    return kStepAttnSolo;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int wtype_id(GGMLType t) { return (int)t; }

__global__ void embed_state_kernel(float* __restrict__ out, const uint8_t* __restrict__ W,
                                   const DecodeState* __restrict__ st, int dim) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    const int t = st->token;
    const uint8_t* blk = W + ((size_t)t * (dim / 32) + i / 32) * 34;
    out[i] = half_bits_to_float(blk[0] | (blk[1] << 8)) * (float)(int8_t)blk[2 + (i & 31)];
}

template <typename KVT>
cudaError_t launch_attn(const AttnArgs& a, int nchunk, int nkv, cudaStream_t st) {
    auto kern = attn_partial_kernel<KVT, 128, true>;
    constexpr int smem = attn_smem_bytes<KVT, 128>();
    static int set_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(set_mask & (1 << (dev & 31)))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        set_mask |= 1 << (dev & 31);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(nchunk, nkv);
    cfg.blockDim = dim3(ATTN_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// Enqueue one token step on m->stream.
int enqueue_step(fence_model* m) {
    const fence_config& c = m->cfg;
    cudaStream_t st = m->stream;
    if (m->use_step) {
        if (c.kv_dtype == FENCE_KV_F16) FENCE_CUDA_TRY(launch_step<__half>(m->sargs, m->splan, st));
        else FENCE_CUDA_TRY(launch_step<__nv_bfloat16>(m->sargs, m->splan, st));
        return FENCE_OK;
    }
    embed_state_kernel<<<(c.embed_dim + 255) / 256, 256, 0, st>>>(m->hidden, m->tok_embd, m->state, c.embed_dim);
    FENCE_CUDA_TRY(cudaGetLastError());
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerW& w = m->layers[l];
        const LayerLaunch& L = m->launches[l];
        FENCE_CUDA_TRY(rgemv_dispatch(L.qkv.xm, L.qkv.epi, L.qkv.a, L.qkv.p, st));
        if (c.kv_dtype == FENCE_KV_F16) FENCE_CUDA_TRY(launch_attn<__half>(L.attn, m->attn_nchunk, c.n_kv_heads, st));
        else FENCE_CUDA_TRY(launch_attn<__nv_bfloat16>(L.attn, m->attn_nchunk, c.n_kv_heads, st));
        FENCE_CUDA_TRY(rgemv_dispatch(L.o.xm, L.o.epi, L.o.a, L.o.p, st));
        FENCE_CUDA_TRY(rgemv_dispatch(L.gu.xm, L.gu.epi, L.gu.a, L.gu.p, st));
        FENCE_CUDA_TRY(rgemv_dispatch(L.down.xm, L.down.epi, L.down.a, L.down.p, st));
    }
    FENCE_CUDA_TRY(rgemv_dispatch(m->lm.xm, m->lm.epi, m->lm.a, m->lm.p, st));
    return FENCE_OK;
}

int run_step(fence_model* m) {
    if (m->tp_n > 1 && !m->tp_connected)
        return set_error(FENCE_E_ARG, "tensor-parallel model: call fence_tp_connect on every rank first");
    if (m->gexec) return cuda_status(cudaGraphLaunch(m->gexec, m->stream), "graph launch");
    return enqueue_step(m);
}

int capture_graph(fence_model* m) {
    FENCE_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(m);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc != FENCE_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    FENCE_CUDA_TRY(e);
    m->graph = g;
    FENCE_CUDA_TRY(cudaGraphInstantiate(&m->gexec, g, 0));
    return FENCE_OK;
}

// Sets the device decode state from the host (pinned ring slot; async, ordered on the stream).
int set_state(fence_model* m, int token, int pos, int step) {
    static thread_local int slot = 0;
    slot = (slot + 1) % m->h_state_n;
    DecodeState* hs = m->h_state + slot;
    // the slot was used h_state_n launches ago; make sure that copy has executed
    if (slot == 0) FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    hs->token = token;
    hs->pos = pos;
    hs->step = step;
    hs->err = 0;
    FENCE_CUDA_TRY(cudaMemcpyAsync(m->state, hs, sizeof(DecodeState), cudaMemcpyHostToDevice, m->stream));
    return FENCE_OK;
}

// Enqueues the copy of the device decode state into m->h_out (pinned), to be read after the next
// stream synchronisation.
int fetch_state(fence_model* m) {
    FENCE_CUDA_TRY(cudaMemcpyAsync(m->h_out, m->state, sizeof(DecodeState), cudaMemcpyDeviceToHost, m->stream));
    return FENCE_OK;
}

// After a synchronisation that followed fetch_state: FENCE_E_DEVICE_WAIT if a step gave up on a
// bounded wait (its results are invalid).
int state_status(fence_model* m, const char* what) {
    if (m->h_out->err)
        return set_error(FENCE_E_DEVICE_WAIT, "%s: a device-side bounded wait expired (device error %d); the step's "
                         "results are invalid", what, m->h_out->err);
    return FENCE_OK;
}

const GGUFTensorInfo* need(fence_model* m, const std::string& name, std::string& err) {
    const GGUFTensorInfo* t = m->gguf.find_tensor(name);
    if (!t && err.empty()) err = "missing tensor " + name;
    return t;
}

bool check_linear(const GGUFTensorInfo* t, uint64_t K, uint64_t M, std::string& err) {
    if (!t) return false;
    if (t->type != GGMLType::Q6_K && t->type != GGMLType::Q8_0) {
        err = "tensor " + t->name + " has type " + ggml_type_name(t->type) + " (engine streams Q6_K and Q8_0)";
        return false;
    }
    if (t->n_dims != 2 || t->dims[0] != K || t->dims[1] != M) {
        err = "tensor " + t->name + " has dims [" + std::to_string(t->dims[0]) + ", " + std::to_string(t->dims[1]) +
              "], expected [" + std::to_string(K) + ", " + std::to_string(M) + "]";
        return false;
    }
    return true;
}
// A sparse-MoE expert tensor: n_exp matrices [K, M] stacked as dims [K, M, n_exp].
bool check_experts(const GGUFTensorInfo* t, uint64_t K, uint64_t M, uint64_t E, std::string& err) {
    if (!t) return false;
    if (t->type != GGMLType::Q6_K && t->type != GGMLType::Q8_0) {
        err = "tensor " + t->name + " has type " + ggml_type_name(t->type) + " (engine streams Q6_K and Q8_0)";
        return false;
    }
    if (t->n_dims != 3 || t->dims[0] != K || t->dims[1] != M || t->dims[2] != E) {
        err = "tensor " + t->name + " must have dims [" + std::to_string(K) + ", " + std::to_string(M) + ", " +
              std::to_string(E) + "]";
        return false;
    }
    return true;
}
bool check_vec(const GGUFTensorInfo* t, uint64_t n, std::string& err) {
    if (!t) return true;  // optional vectors are checked by the caller
    if (t->type != GGMLType::F32 || t->n_elements() != n) {
        err = "tensor " + t->name + " must be F32 with " + std::to_string(n) + " elements";
        return false;
    }
    return true;
}

// The token step as the persistent kernel's phase list, from the per-phase launch arguments.
int build_step_phases(fence_model* m) {
    const fence_config& c = m->cfg;
    std::vector<SPhase>& ph = m->h_phases;
    ph.clear();
    auto gemv = [&](const RPhase& r) {
        SPhase p{};
        p.kind = SP_GEMV;
        p.g = r.a;
        p.xm = r.xm;
        p.epi = r.epi;
        return p;
    };
    // tensor parallel: reduction 2l after o_proj, 2l+1 after down; the residual stream alternates
    // between hidden (read by even reductions) and hidden_b (odd)
    const bool tp = m->tp_n > 1;
    auto tp_sum = [&](SPhase& p, int red) {
        if (!tp || red < 0) return;
        p.tp_sum = 1;
        p.red_idx = red;
        p.hin = (red & 1) ? m->hidden_b : m->hidden;
        p.hout = (red & 1) ? m->hidden : m->hidden_b;
    };
    auto tp_red = [&](SPhase& p, int red) {
        if (!tp) return;
        p.tp_red = 1;
        p.red_idx = red;
    };
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerLaunch& L = m->launches[l];
        SPhase q = gemv(L.qkv);
        if (l == 0) {  // the token embedding is folded into the first phase's prologue
            q.embed = 1;
            q.embd = m->tok_embd;
            q.hidden_out = m->hidden;
        }
        tp_sum(q, 2 * l - 1);
        ph.push_back(q);
        SPhase at{};
        at.kind = SP_ATTN;
        at.at = L.attn;
        at.at.nchunk = m->step_nchunk;
        ph.push_back(at);
        SPhase o = gemv(L.o), gu = gemv(L.gu), dn = gemv(L.down);
        tp_red(o, 2 * l);
        tp_sum(gu, 2 * l);
        ph.push_back(o);
        if (!m->moe) {
            tp_red(dn, 2 * l + 1);
            ph.push_back(gu);
            ph.push_back(dn);
            continue;
        }
        // sparse MoE: gate/up of every routed slot (slot 0 routes; later slots reuse its x records and
        // need no grid wait), then down of every slot (slot 0 waits for every CTA's gate/up; later
        // slots write the same rows of the same CTA and need none)
        const int K = c.n_experts_used;
        const size_t act_el = L.gu.a.act_f16 ? 2 : 4;
        auto moe = [&](SPhase& p, int kind, int slot) {
            p.moe = kind;
            p.moe_slot = slot;
            p.moe_seq = l + 1;
            p.n_exp = c.n_experts;
            p.n_used = K;
            p.e_lo = m->e_lo;
            p.e_n = m->e_n;
            p.route_w = m->layers[l].router;
            p.moe_acc = m->moe_acc;
            p.moe_chain = slot > 0;
        };
        for (int s = 0; s < K; ++s) {
            SPhase p = gu;
            moe(p, SK_MOE_GU, s);
            if (s > 0) {
                p.moe_reuse_x = 1;
                p.tp_sum = 0;
            }
            p.g.act = static_cast<uint8_t*>(m->act) + (size_t)s * L.gu.a.Mv * act_el;
            ph.push_back(p);
        }
        for (int s = 0; s < K; ++s) {
            SPhase p = dn;
            moe(p, SK_MOE_DN, s);
            p.g.x = static_cast<uint8_t*>(m->act) + (size_t)s * L.gu.a.Mv * act_el;
            p.moe_last = s == K - 1;
            if (p.moe_last) tp_red(p, 2 * l + 1);
            ph.push_back(p);
        }
    }
    SPhase lm = gemv(m->lm);
    tp_sum(lm, 2 * c.n_layers - 1);
    ph.push_back(lm);
    std::string err;
    m->splan = plan_step(ph, m->dev, err);
    if (!m->splan.ok) return set_error(FENCE_E_UNSUPPORTED, "%s", err.c_str());
    if (m->splan.grid > 4096) return set_error(FENCE_E_UNSUPPORTED, "step kernel: more than 4096 SMs");
    // re-tile every GEMV phase's matrix for the step kernel (per-CTA row blocks x K-slices, one bulk
    // copy per tile), then drop the row-major copy
    {
        const int G = m->splan.grid;
        size_t ngemv = 0;
        for (const SPhase& p : ph) ngemv += p.kind == SP_GEMV;
        std::vector<unsigned long long> tc(ngemv * G);
        std::vector<unsigned long long> base(ngemv);
        unsigned long long total = 0;
        size_t gi = 0;
        for (SPhase& p : ph) {
            if (p.kind != SP_GEMV) continue;
            const RGemvArgs& g = p.g;
            base[gi] = total;
            const unsigned long long tb = (sk_tile_plan(g.wt, g.I, g.Mv, g.dual, G, g.RB, g.CI, &tc[gi * G]) + 255) / 256 * 256;
            if (!p.moe) {
                total += tb;
            } else if (p.moe_slot == 0) {  // one tile set per local expert; later slots share them
                p.estride = (long long)tb;
                total += tb * (unsigned long long)m->e_n;
            }
            ++gi;
        }
        FENCE_CUDA_TRY(cudaMalloc(&m->tarena, total + 256));
        FENCE_CUDA_TRY(cudaMemset(m->tarena, 0, total + 256));
        FENCE_CUDA_TRY(cudaMalloc(&m->d_tcta, tc.size() * sizeof(unsigned long long)));
        FENCE_CUDA_TRY(cudaMemcpy(m->d_tcta, tc.data(), tc.size() * sizeof(unsigned long long), cudaMemcpyHostToDevice));
        gi = 0;
        for (size_t i = 0; i < ph.size(); ++i) {
            SPhase& p = ph[i];
            if (p.kind != SP_GEMV) continue;
            RGemvArgs& g = p.g;
            g.tb = m->tarena + base[gi];
            g.tcta = m->d_tcta + gi * G;
            if (!p.moe) {
                FENCE_CUDA_TRY(sk_retile(g.wt, g.w, g.I, g.Mv, g.dual, G, g.RB, g.CI, g.tcta, const_cast<uint8_t*>(g.tb),
                                         m->stream));
            } else if (p.moe_slot == 0) {
                const std::vector<RMat>& mats = p.moe == SK_MOE_GU ? m->moe_gu : m->moe_dn;
                for (int e = 0; e < m->e_n; ++e)
                    FENCE_CUDA_TRY(sk_retile(g.wt, mats[(size_t)(p.moe_seq - 1) * m->e_n + e], g.I, g.Mv, g.dual, G,
                                             g.RB, g.CI, g.tcta, const_cast<uint8_t*>(g.tb) + (size_t)e * p.estride,
                                             m->stream));
            } else {  // the tiles of this layer's slot-0 phase of the same kind (same shape, same CTA split)
                for (size_t j = 0; j < i; ++j)
                    if (ph[j].moe == p.moe && ph[j].moe_seq == p.moe_seq && ph[j].moe_slot == 0) {
                        g.tb = ph[j].g.tb;
                        p.estride = ph[j].estride;
                    }
            }
            ++gi;
        }
        FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
        if (!m->prefill_ok) {  // the per-phase path and the batched prefill are the readers of the row-major copy
            cudaFree(m->rarena);
            m->rarena = nullptr;
        }
    }
    FENCE_CUDA_TRY(cudaMalloc(&m->d_phases, ph.size() * sizeof(SPhase)));
    FENCE_CUDA_TRY(cudaMemcpy(m->d_phases, ph.data(), ph.size() * sizeof(SPhase), cudaMemcpyHostToDevice));
    FENCE_CUDA_TRY(cudaMalloc(&m->d_bar, sizeof(unsigned long long)));
    FENCE_CUDA_TRY(cudaMemset(m->d_bar, 0, sizeof(unsigned long long)));
    StepArgs& A = m->sargs;
    A = StepArgs{};
    A.ph = m->d_phases;
    A.nph = (int)ph.size();
    A.ring = m->splan.ring;
    A.attn_solo = step_attn_solo();
    A.slot_bytes = m->splan.slot_bytes;
    A.scratch_bytes = m->splan.scratch_bytes;
    A.acc_floats = m->splan.acc_floats;
    A.bar = m->d_bar;
    A.state = m->state;
    A.cta_val = m->lm_val;
    A.cta_idx = m->lm_idx;
    A.token_log = m->token_log;
    A.token_log_cap = m->token_log_cap;
    A.stall_phase = (m->opts.wait_test_phase >= 0 && m->opts.wait_test_phase < A.nph) ? m->opts.wait_test_phase : -1;
    if (tp) {
        A.tp_n = m->tp_n;
        A.tp_rank = m->tp_rank;
        A.tp_h = c.embed_dim;
        A.n_red = 2 * c.n_layers;
        A.vocab0 = m->vocab0;
        for (int p = 0; p < m->tp_n; ++p) A.xb[p] = m->xpeer[p];
        A.launch = m->tp_launch;
    } else {
        A.tp_n = 1;
    }
    m->use_step = 1;
    return FENCE_OK;
}

void free_model(fence_model* m) {
    if (!m) return;
    if (!m->stream) {  // failed before any device work
        m->gguf.close();
        delete m;
        return;
    }
    if (m->dev >= 0) cudaSetDevice(m->dev);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->gexec) cudaGraphExecDestroy(m->gexec);
    if (m->graph) cudaGraphDestroy(m->graph);
    cudaFree(m->arena);
    cudaFree(m->kcache);
    cudaFree(m->vcache);
    cudaFree(m->hidden);
    cudaFree(m->qkv);
    cudaFree(m->attn_out);
    cudaFree(m->logits);
    cudaFree(m->attn_part);
    cudaFree(m->act);
    cudaFree(m->counters);
    cudaFree(m->lm_val);
    cudaFree(m->lm_idx);
    cudaFree(m->state);
    cudaFree(m->token_log);
    cudaFree(m->rope);
    cudaFree(m->rarena);
    cudaFree(m->tarena);
    cudaFree(m->d_tcta);
    cudaFree(m->qkv_bias);
    cudaFree(m->d_phases);
    cudaFree(m->d_bar);
    for (int p = 0; p < m->tp_n; ++p)
        if (p != m->tp_rank && m->xpeer[p]) cudaIpcCloseMemHandle(m->xpeer[p]);
    cudaFree(m->xbuf);
    cudaFree(m->hidden_b);
    cudaFree(m->tp_launch);
    cudaFree(m->moe_acc);
    cudaFree(m->pf_tok);
    cudaFree(m->pf_hidden);
    cudaFree(m->pf_qkv);
    cudaFree(m->pf_q);
    cudaFree(m->pf_attn);
    cudaFree(m->pf_bscale);
    cudaFree(m->pf_x16);
    cudaFree(m->pf_act);
    cudaFree(m->pf_w);
    cudaFree(m->samp_scratch);
    cudaFree(m->samp_hist);
    cudaFree(m->samp_out);
    if (m->h_state) cudaFreeHost(m->h_state);
    if (m->h_token) cudaFreeHost(m->h_token);
    if (m->h_out) cudaFreeHost(m->h_out);
    if (m->stream) cudaStreamDestroy(m->stream);
    m->gguf.close();
    delete m;
}

}  // namespace

// =============================================================================================
extern "C" void fence_load_opts_default(fence_load_opts* o) {
    std::memset(o, 0, sizeof *o);
    o->max_ctx = 4096;
    o->kv_dtype = FENCE_KV_F16;
    o->device = 0;
    o->use_graph = 1;
    o->verbose = 0;
    o->tp_rank = 0;
    o->tp_size = 1;
    o->step_kernel = 1;
    o->wait_test_phase = -1;
    o->moe_ep = 0;
    o->prefill = 1;
}

extern "C" fence_model* fence_model_load(const char* path, const fence_load_opts* opts_in) {
    fence_load_opts opts;
    if (opts_in) opts = *opts_in;
    else fence_load_opts_default(&opts);
    if (!path) {
        set_error(FENCE_E_ARG, "model_load: null path");
        return nullptr;
    }
    if (opts.tp_size > 1 && ((opts.tp_size != 2 && opts.tp_size != 4 && opts.tp_size != 8) || opts.tp_rank < 0 ||
                             opts.tp_rank >= opts.tp_size)) {
        set_error(FENCE_E_ARG, "model_load: tp_rank %d / tp_size %d (tp_size 2, 4 or 8)", opts.tp_rank, opts.tp_size);
        return nullptr;
    }
    if (opts.tp_size > 1 && !opts.step_kernel) {
        set_error(FENCE_E_UNSUPPORTED, "model_load: tensor parallel decode runs in the step kernel (step_kernel = 1)");
        return nullptr;
    }
    fence_model* m = new fence_model();
    m->opts = opts;
    m->dev = opts.device;
    auto bail = [&](int code, const std::string& msg) -> fence_model* {
        set_error(code, "%s", msg.c_str());
        free_model(m);
        return nullptr;
    };
    if (opts.verbose) printf("Loading GGUF: %s\n", path);
    if (!m->gguf.open(path)) return bail(FENCE_E_FORMAT, "model_load: " + m->gguf.last_error());

    // ---- config from metadata, with the reference's keys, types and fallbacks (qwen3.cu:116-160)
    fence_config& c = m->cfg;
    std::string arch = "qwen2";
    try {
        arch = m->gguf.get_string("general.architecture");
    } catch (...) {
    }
    try {
        c.n_layers = (int)m->gguf.get_u32(arch + ".block_count");
        c.embed_dim = (int)m->gguf.get_u32(arch + ".embedding_length");
        c.ff_dim = (int)m->gguf.get_u32(arch + ".feed_forward_length");
        c.n_heads = (int)m->gguf.get_u32(arch + ".attention.head_count");
        c.n_kv_heads = (int)m->gguf.get_u32(arch + ".attention.head_count_kv");
    } catch (const std::exception& ex) {
        return bail(FENCE_E_FORMAT, std::string("model_load: ") + ex.what());
    }
    try {
        c.head_dim = (int)m->gguf.get_u32(arch + ".attention.key_length");
    } catch (...) {
        c.head_dim = c.n_heads ? c.embed_dim / c.n_heads : 0;
        if (opts.verbose) printf("Config: head_dim not in metadata, inferred %d\n", c.head_dim);
    }
    try {
        c.rope_freq_base = m->gguf.get_f32(arch + ".rope.freq_base");
    } catch (...) {
        c.rope_freq_base = 10000.0f;
        if (opts.verbose) printf("Config: rope.freq_base not in metadata, using default %.0f\n", c.rope_freq_base);
    }
    try {
        c.rms_eps = m->gguf.get_f32(arch + ".attention.layer_norm_rms_epsilon");
    } catch (...) {
        c.rms_eps = 1e-5f;
        if (opts.verbose) printf("Config: rms_epsilon not in metadata, using default %.0e\n", c.rms_eps);
    }
    try {
        c.n_experts = (int)m->gguf.get_u32(arch + ".expert_count");
        c.n_experts_used = (int)m->gguf.get_u32(arch + ".expert_used_count");
    } catch (...) {
        c.n_experts = c.n_experts_used = 0;
    }
    const GGUFTensorInfo* embd = m->gguf.find_tensor("token_embd.weight");
    if (!embd) return bail(FENCE_E_FORMAT, "model_load: missing token_embd.weight");
    c.vocab_size = (int)embd->dims[1];
    c.max_ctx = opts.max_ctx > 0 ? opts.max_ctx : 4096;
    c.temperature = 0.7f;
    c.top_p = 0.8f;
    c.top_k = 50;
    c.repetition_penalty = 1.15f;
    c.min_p = 0.05f;
    c.dynamic_temp = 1;
    c.kv_dtype = opts.kv_dtype;
    c.tp_rank = opts.tp_size > 1 ? opts.tp_rank : 0;
    c.tp_size = opts.tp_size > 1 ? opts.tp_size : 1;
    c.embd_type = (int)embd->type;

    if (c.n_layers <= 0 || c.embed_dim <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads)
        return bail(FENCE_E_FORMAT, "model_load: inconsistent head counts / dimensions in metadata");
    if (c.head_dim != 128)
        return bail(FENCE_E_UNSUPPORTED, "model_load: head_dim " + std::to_string(c.head_dim) + " (engine kernels are built for 128)");
    if (c.n_heads / c.n_kv_heads > ATTN_MAX_G)
        return bail(FENCE_E_UNSUPPORTED, "model_load: more than 8 query heads per KV head");
    const bool moe = c.n_experts > 0;
    if (moe) {
        if (c.n_experts > SK_MOE_EMAX || c.n_experts_used < 1 || c.n_experts_used > 2 || c.n_experts_used > c.n_experts)
            return bail(FENCE_E_UNSUPPORTED, "model_load: sparse MoE needs at most " + std::to_string(SK_MOE_EMAX) +
                                                 " experts and 1 or 2 routed per token");
        if (!opts.step_kernel)
            return bail(FENCE_E_UNSUPPORTED, "model_load: sparse MoE runs in the step kernel (step_kernel = 1)");
        if (opts.moe_ep && opts.tp_size > 1 && c.n_experts % opts.tp_size)
            return bail(FENCE_E_UNSUPPORTED, "model_load: expert parallel needs the experts to split evenly over the ranks");
    }
    if (embd->type != GGMLType::Q8_0 || embd->dims[0] != (uint64_t)c.embed_dim)
        return bail(FENCE_E_UNSUPPORTED, "model_load: token_embd.weight must be Q8_0 [embed_dim, vocab]");
    if (c.embed_dim % 64)
        return bail(FENCE_E_UNSUPPORTED, "model_load: embed_dim must be a multiple of 64");

    const uint64_t H = c.embed_dim, F = c.ff_dim, qd = (uint64_t)c.n_heads * c.head_dim,
                   kvd = (uint64_t)c.n_kv_heads * c.head_dim;
    // ---- this rank's shard (Megatron split, tp_size ranks): q/k/v rows by heads and gate/up rows by
    // FFN rows (column-parallel, no exchange), o_proj and down by input columns (row-parallel: each
    // rank's partial rows are summed over the ranks), the tied LM head by vocabulary rows
    const int TPN = c.tp_size, TPR = c.tp_rank;
    // expert parallel (MoE, tp_size > 1, opts.moe_ep): each rank holds n_experts / tp_size whole
    // experts; otherwise every rank holds a 1/tp_size slice of every expert (as a dense FFN)
    const bool ep = moe && opts.moe_ep && TPN > 1;
    if (TPN > 1 && (c.n_heads % TPN || c.n_kv_heads % TPN || (!ep && c.ff_dim % TPN)))
        return bail(FENCE_E_UNSUPPORTED, "model_load: heads / FFN rows do not split evenly over tp_size ranks");
    const uint64_t qdl = qd / TPN, kvdl = kvd / TPN, Fl = ep ? F : F / TPN;
    const int FTPR = ep ? 0 : TPR;  // this rank's FFN row slice (expert parallel: whole experts)
    m->moe = moe ? 1 : 0;
    m->moe_ep = ep ? 1 : 0;
    m->e_lo = ep ? TPR * (c.n_experts / TPN) : 0;
    m->e_n = moe ? (ep ? c.n_experts / TPN : c.n_experts) : 0;
    const int Hq_l = c.n_heads / TPN, Hkv_l = c.n_kv_heads / TPN;
    const int Vl = (c.vocab_size + TPN - 1) / TPN, v0 = TPR * Vl, vn = std::min(c.vocab_size, v0 + Vl) - v0;
    m->tp_n = TPN;
    m->tp_rank = TPR;
    m->vocab0 = v0;
    m->vocab_n = vn;

    // ---- collect and validate tensors; lay out the device arena of the tensors kept as they are in
    // the file (embedding, norms, biases, router); the linears stay in the file mapping until the
    // per-layer streaming upload below
    struct Up {
        const GGUFTensorInfo* t;
        size_t off;
    };
    std::vector<Up> ups;
    size_t total = 0;
    auto place = [&](const GGUFTensorInfo* t) -> size_t {
        const size_t off = total;
        ups.push_back({t, off});
        total = align_up(total + t->data_size_bytes, 256);
        return off;
    };
    std::string err;
    const GGUFTensorInfo* onorm = need(m, "output_norm.weight", err);
    if (!err.empty() || !check_vec(onorm, H, err)) return bail(FENCE_E_FORMAT, "model_load: " + err);
    std::vector<std::vector<std::pair<const GGUFTensorInfo*, size_t>>> lt(c.n_layers);
    const size_t off_embd = place(embd);
    const size_t off_onorm = place(onorm);
    struct LOff {
        size_t q, k, v, o, g, u, d, an, fn, qn, kn, qb, kb, vb, rt;
        bool has_qn, has_kn, has_qb, has_kb, has_vb;
    };
    std::vector<LOff> lo(c.n_layers);
    m->layers.resize(c.n_layers);
    size_t bytes_per_token = embd->data_size_bytes;
    c.linear_type = 0;
    for (int l = 0; l < c.n_layers; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        const GGUFTensorInfo *an = need(m, p + "attn_norm.weight", err), *q = need(m, p + "attn_q.weight", err),
                             *k = need(m, p + "attn_k.weight", err), *v = need(m, p + "attn_v.weight", err),
                             *o = need(m, p + "attn_output.weight", err), *fn = need(m, p + "ffn_norm.weight", err),
                             *g = need(m, p + (moe ? "ffn_gate_exps.weight" : "ffn_gate.weight"), err),
                             *u = need(m, p + (moe ? "ffn_up_exps.weight" : "ffn_up.weight"), err),
                             *d = need(m, p + (moe ? "ffn_down_exps.weight" : "ffn_down.weight"), err),
                             *rt = moe ? need(m, p + "ffn_gate_inp.weight", err) : nullptr;
        if (!err.empty()) return bail(FENCE_E_FORMAT, "model_load: " + err);
        const GGUFTensorInfo *qn = m->gguf.find_tensor(p + "attn_q_norm.weight"),
                             *kn = m->gguf.find_tensor(p + "attn_k_norm.weight"),
                             *qb = m->gguf.find_tensor(p + "attn_q.bias"), *kb = m->gguf.find_tensor(p + "attn_k.bias"),
                             *vb = m->gguf.find_tensor(p + "attn_v.bias");
        const uint64_t E = (uint64_t)c.n_experts;
        auto lin = [&](const GGUFTensorInfo* t, uint64_t K, uint64_t M) {
            return moe ? check_experts(t, K, M, E, err) : check_linear(t, K, M, err);
        };
        if (moe && (rt->type != GGMLType::F32 || rt->n_dims != 2 || rt->dims[0] != H || rt->dims[1] != E)) {
            err = "tensor " + rt->name + " must be F32 [" + std::to_string(H) + ", " + std::to_string(E) + "]";
            return bail(FENCE_E_FORMAT, "model_load: " + err);
        }
        if (!check_linear(q, H, qd, err) || !check_linear(k, H, kvd, err) || !check_linear(v, H, kvd, err) ||
            !check_linear(o, qd, H, err) || !lin(g, H, F) || !lin(u, H, F) ||
            !lin(d, F, H) || !check_vec(an, H, err) || !check_vec(fn, H, err) ||
            !check_vec(qn, c.head_dim, err) || !check_vec(kn, c.head_dim, err) || !check_vec(qb, qd, err) ||
            !check_vec(kb, kvd, err) || !check_vec(vb, kvd, err))
            return bail(FENCE_E_FORMAT, "model_load: " + err);
        if (q->type != k->type || q->type != v->type || g->type != u->type)
            return bail(FENCE_E_UNSUPPORTED, "model_load: q/k/v (and gate/up) must share one quant type in a layer");
        LayerW& w = m->layers[l];
        w.t_qkv = (int)q->type;
        w.t_o = (int)o->type;
        w.t_gu = (int)g->type;
        w.t_down = (int)d->type;
        if (c.linear_type == 0) c.linear_type = (int)q->type;
        LOff& L = lo[l];
        L.an = place(an);
        L.fn = place(fn);
        w.q = static_cast<const uint8_t*>(q->data);
        w.k = static_cast<const uint8_t*>(k->data);
        w.v = static_cast<const uint8_t*>(v->data);
        w.o = static_cast<const uint8_t*>(o->data);
        w.gate = static_cast<const uint8_t*>(g->data);
        w.up = static_cast<const uint8_t*>(u->data);
        w.down = static_cast<const uint8_t*>(d->data);
        L.has_qn = qn && kn;  // the reference applies q/k-norm only when both exist (qwen3.cu:292)
        L.has_kn = L.has_qn;
        if (L.has_qn) {
            L.qn = place(qn);
            L.kn = place(kn);
        }
        L.has_qb = qb != nullptr;
        L.has_kb = kb != nullptr;
        L.has_vb = vb != nullptr;
        if (qb) L.qb = place(qb);
        if (kb) L.kb = place(kb);
        if (vb) L.vb = place(vb);
        if (rt) L.rt = place(rt);
        // MoE: the routed experts' share of the expert tensors and the router are streamed per token
        const uint64_t ffn = g->data_size_bytes + u->data_size_bytes + d->data_size_bytes;
        bytes_per_token += q->data_size_bytes + k->data_size_bytes + v->data_size_bytes + o->data_size_bytes +
                           (moe ? ffn / E * (uint64_t)c.n_experts_used + rt->data_size_bytes : ffn);
    }
    c.has_qk_norm = lo[0].has_qn ? 1 : 0;
    c.weight_bytes = bytes_per_token;
    m->arena_bytes = total;
    if (opts.verbose) {
        printf("Config: layers=%d embed=%d ff=%d heads=%d/%d head_dim=%d vocab=%d\n", c.n_layers, c.embed_dim,
               c.ff_dim, c.n_heads, c.n_kv_heads, c.head_dim, c.vocab_size);
        printf("Copying embedding and norms to GPU (%.2f GB); linears stream per layer...\n", total / 1e9);
    }

    // ---- device allocations (everything above is host-side parsing and validation)
    if (cudaSetDevice(m->dev) != cudaSuccess) return bail(FENCE_E_ARG, "model_load: cannot select CUDA device");
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(FENCE_E_NOMEM, "model_load: stream creation failed");
    if (cudaMalloc(&m->arena, total) != cudaSuccess) return bail(FENCE_E_NOMEM, "model_load: weight arena allocation failed");
    const auto t0 = std::chrono::steady_clock::now();
    Uploader up;
    if (up.init(m->stream) != FENCE_OK) return bail(FENCE_E_NOMEM, fence_last_error());
    for (const Up& u : ups)
        if (up.put(m->arena + u.off, static_cast<const uint8_t*>(u.t->data), u.t->data_size_bytes, u.t->data_size_bytes, 1))
            return bail(FENCE_E_NOMEM, std::string("model_load: upload of ") + u.t->name + ": " + fence_last_error());
    m->tok_embd = m->arena + off_embd;
    m->out_norm = reinterpret_cast<const float*>(m->arena + off_onorm);
    for (int l = 0; l < c.n_layers; ++l) {
        LayerW& w = m->layers[l];
        const LOff& L = lo[l];
        auto PF = [&](size_t off) { return reinterpret_cast<const float*>(m->arena + off); };
        w.attn_norm = PF(L.an);
        w.ffn_norm = PF(L.fn);
        if (L.has_qn) {
            w.q_norm = PF(L.qn);
            w.k_norm = PF(L.kn);
        }
        if (L.has_qb) w.q_bias = PF(L.qb);
        if (L.has_kb) w.k_bias = PF(L.kb);
        if (L.has_vb) w.v_bias = PF(L.vb);
        if (moe) w.router = PF(L.rt);
    }

    const int HD = c.head_dim, G = c.n_heads / c.n_kv_heads;
    // KV cache [layer][kv_head][max_ctx][SK_ATT_RSTR]: rows padded from 128 to 136 elements, so that
    // one bulk copy moves a whole 64-position tile into the bank-conflict-free layout the step
    // kernel's attention reads (the 8 padding elements of a row are never read as data)
    const size_t kv_elems = (size_t)c.n_layers * Hkv_l * c.max_ctx * SK_ATT_RSTR;
    // chunks per KV head: 64-position chunks up to 120 (the merge keeps G x chunks scale factors in
    // the CTA's score buffer); longer contexts get longer chunks
    m->attn_nchunk = std::min(120, std::max(32, (c.max_ctx + ATTN_CHUNK - 1) / ATTN_CHUNK));
    // the step kernel's attention units span at most SK_ATT_MAXLEN positions: enough chunks to cover max_ctx
    m->step_nchunk = std::max(m->attn_nchunk, (c.max_ctx + SK_ATT_MAXLEN - 1) / SK_ATT_MAXLEN);
    const int part_chunks = std::max(m->attn_nchunk, m->step_nchunk);
    bool ok = cudaMalloc(&m->kcache, kv_elems * 2) == cudaSuccess && cudaMalloc(&m->vcache, kv_elems * 2) == cudaSuccess &&
              cudaMemset(m->kcache, 0, kv_elems * 2) == cudaSuccess && cudaMemset(m->vcache, 0, kv_elems * 2) == cudaSuccess &&
              cudaMalloc(&m->hidden, H * 4) == cudaSuccess && cudaMalloc(&m->qkv, (qdl + 2 * kvdl) * 4) == cudaSuccess &&
              cudaMalloc(&m->attn_out, qdl * 4) == cudaSuccess && cudaMalloc(&m->logits, (size_t)vn * 4) == cudaSuccess &&
              cudaMalloc(&m->attn_part, (size_t)Hkv_l * part_chunks * G * SK_PART_STRIDE * 4) == cudaSuccess &&
              cudaMalloc(&m->act, Fl * 4 * (moe ? 2 : 1)) == cudaSuccess &&
              cudaMalloc(&m->counters, (Hkv_l + 1) * sizeof(unsigned)) == cudaSuccess &&
              cudaMemset(m->counters, 0, (Hkv_l + 1) * sizeof(unsigned)) == cudaSuccess &&
              cudaMalloc(&m->lm_val, 4096 * 4) == cudaSuccess && cudaMalloc(&m->lm_idx, 4096 * 4) == cudaSuccess &&
              cudaMalloc(&m->state, sizeof(DecodeState)) == cudaSuccess &&
              cudaMemset(m->state, 0, sizeof(DecodeState)) == cudaSuccess &&
              cudaMalloc(&m->rope, (size_t)c.max_ctx * (HD / 2) * sizeof(float2)) == cudaSuccess &&
              cudaMallocHost(&m->h_state, 64 * sizeof(DecodeState)) == cudaSuccess &&
              cudaMallocHost(&m->h_token, 64 * sizeof(int)) == cudaSuccess &&
              cudaMallocHost(&m->h_out, sizeof(DecodeState)) == cudaSuccess;
    if (!ok) return bail(FENCE_E_NOMEM, "model_load: device allocation failed");
    if (moe && TPN > 1 && cudaMalloc(&m->moe_acc, H * 4) != cudaSuccess)
        return bail(FENCE_E_NOMEM, "model_load: device allocation failed");
    if (TPN > 1) {
        const size_t xb = sk_xb_bytes(TPN, (int)H);
        if (cudaMalloc(&m->hidden_b, H * 4) != cudaSuccess || cudaMalloc(&m->xbuf, xb) != cudaSuccess ||
            cudaMemset(m->xbuf, 0, xb) != cudaSuccess || cudaMalloc(&m->tp_launch, 8) != cudaSuccess ||
            cudaMemset(m->tp_launch, 0, 8) != cudaSuccess)
            return bail(FENCE_E_NOMEM, "model_load: exchange buffer allocation failed");
    }
    m->h_state_n = 64;
    m->token_log_cap = std::max(c.max_ctx, 4096);
    if (cudaMalloc(&m->token_log, m->token_log_cap * sizeof(int)) != cudaSuccess)
        return bail(FENCE_E_NOMEM, "model_load: device allocation failed");

    // RoPE table: angle pos * base^(-2i/HD) and its cos/sin in double, rounded once to float.
    {
        std::vector<float2> tab((size_t)c.max_ctx * (HD / 2));
        for (int pos = 0; pos < c.max_ctx; ++pos)
            for (int i = 0; i < HD / 2; ++i) {
                const double ang = (double)pos * std::pow((double)c.rope_freq_base, -2.0 * i / (double)HD);
                tab[(size_t)pos * (HD / 2) + i] = make_float2((float)std::cos(ang), (float)std::sin(ang));
            }
        if (cudaMemcpy(m->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(FENCE_E_NOMEM, "model_load: rope table upload failed");
    }

    // ---- repacked linears (rgemv.cuh): one fused QKV matrix and one gate/up-interleaved matrix per
    // layer, O, down and the tied LM head, rewritten once on the device from the uploaded blocks
    auto wt_of = [](int t) { return t == 14 ? WT_Q6K : WT_Q80; };
    const long long QKVR = (long long)(qdl + 2 * kvdl);
    size_t rbytes = rmat_bytes(WT_Q80, vn, (int)H);
    size_t shard_bytes = (size_t)vn * (H / 32) * 34;  // LM-head shard (+ the layers' shards below)
    auto raw_row = [](int t, uint64_t K) { return t == 14 ? (K * 210 + 255) / 256 : K / 32 * 34; };
    // FFN matrices per layer: one (dense), one per local expert (MoE); streamed per token: one, or the
    // routed experts' (tensor parallel: every rank streams its slice of each; expert parallel: on
    // average n_used / tp_size whole experts per rank)
    const int n_ffn = moe ? m->e_n : 1;
    const double ffn_streamed = moe ? (ep ? (double)c.n_experts_used / TPN : (double)c.n_experts_used) : 1.0;
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerW& w = m->layers[l];
        rbytes += rmat_bytes(wt_of(w.t_qkv), QKVR, (int)H) +
                  rmat_bytes(wt_of(w.t_o), (long long)H, (int)qdl, (int)((TPR * qdl / 64) & 3)) +
                  (size_t)n_ffn * (rmat_bytes(wt_of(w.t_gu), 2 * (long long)Fl, (int)H) +
                                   rmat_bytes(wt_of(w.t_down), (long long)H, (int)Fl, (int)((FTPR * Fl / 64) & 3)));
        shard_bytes += QKVR * raw_row(w.t_qkv, H) + H * raw_row(w.t_o, qdl) +
                       (size_t)(ffn_streamed * (double)(2 * Fl * raw_row(w.t_gu, H) + H * raw_row(w.t_down, Fl))) +
                       (moe ? (size_t)c.n_experts * H * 4 : 0);
    }
    if (moe) m->moe_gu.resize((size_t)c.n_layers * m->e_n), m->moe_dn.resize((size_t)c.n_layers * m->e_n);
    // Q8_0 rows only need 64-element items; Q6_K super-blocks need 256 (a rank's column slice too)
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerW& w = m->layers[l];
        // (a rank's o_proj / down column slice needs whole 64-input items only: a Q6_K super-block
        // cut between two ranks has its d in both ranks' rows)
        if ((w.t_qkv == 14 && H % 256) || (w.t_o == 14 && qd % 256) || (w.t_gu == 14 && H % 256) ||
            (w.t_down == 14 && F % 256) || qdl % 64 || Fl % 64 || H % 64)
            return bail(FENCE_E_UNSUPPORTED, TPN > 1 ? "model_load: a rank's o_proj / down column slice is not a whole "
                                                       "number of 64-input items (choose another tp_size)"
                                                     : "model_load: linear input width not a multiple of the block size");
    }
    if (TPN > 1) c.weight_bytes = shard_bytes;
    if (cudaMalloc(&m->rarena, rbytes) != cudaSuccess) return bail(FENCE_E_NOMEM, "model_load: repacked arena allocation failed");
    int sms = 0, smem_sm = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, m->dev);
    // two CTAs share an SM (a phase and the next, under programmatic dependent launch)
    const int smem_budget = smem_sm / 2 - 2048;
    uint8_t* rp = m->rarena;
    auto carve = [&](int wt, long long rows, int K, int iph) {
        RMat r = rmat_carve(wt, rows, K, rp, iph);
        rp += rmat_bytes(wt, rows, K, iph);
        return r;
    };
    bool any_bias = false;
    for (const LayerW& w : m->layers) any_bias = any_bias || w.q_bias || w.k_bias || w.v_bias;
    if (any_bias) {
        if (cudaMalloc(&m->qkv_bias, (size_t)c.n_layers * QKVR * 4) != cudaSuccess ||
            cudaMemsetAsync(m->qkv_bias, 0, (size_t)c.n_layers * QKVR * 4, m->stream) != cudaSuccess)
            return bail(FENCE_E_NOMEM, "model_load: bias allocation failed");
    }
    cudaStream_t st = m->stream;
    auto fill = [&](int wt, const uint8_t* src, long long rows, int K, const RMat& r, long long row0, int stride) {
        return rmat_fill(wt, src, rows, K, r, row0, stride, st) == cudaSuccess;
    };
    auto phase = [&](RPhase& ph, const RMat& r, int wt, int K, int Mv, int dual, int xm, int epi) -> bool {
        ph = RPhase{};
        ph.a.w = r;
        ph.a.wt = wt;
        ph.a.I = K / 64;
        ph.a.Mv = Mv;
        ph.a.dual = dual;
        ph.xm = xm;
        ph.epi = epi;
        ph.p = plan_rgemv(ph.a, sms, smem_budget);
        // the per-phase kernel's plan (its own 224-lane geometry) matters only without the step
        // kernel, which plans every phase itself (plan_step)
        return ph.p.ok != 0 || opts.step_kernel != 0;
    };

    m->launches.resize(c.n_layers);
    const size_t kv_layer = (size_t)Hkv_l * c.max_ctx * SK_ATT_RSTR;
    // Streaming upload of the linears, one layer at a time: this rank's pieces only (its q/k/v and
    // FFN rows, the blocks covering its o_proj / down input columns, its experts) go through the
    // pinned staging ring into one device staging buffer and are repacked from there on the same
    // stream, so the next layer's copies overwrite the buffer only after the repack has read it.
    const uint64_t q_c0 = (uint64_t)TPR * qdl, f_c0 = (uint64_t)FTPR * Fl;
    auto a256 = [](size_t x) { return align_up(x, 256); };
    size_t stage_bytes = 0;
    for (const LayerW& w : m->layers) {
        // exactly the pieces `take` carves below, each rounded to 256 bytes
        const size_t b = a256(qdl * raw_row(w.t_qkv, H)) + 2 * a256(kvdl * raw_row(w.t_qkv, H)) +
                         a256(H * col_cover(w.t_o, q_c0, q_c0 + qdl).bytes) +
                         (size_t)n_ffn * (2 * a256(Fl * raw_row(w.t_gu, H)) + a256(H * col_cover(w.t_down, f_c0, f_c0 + Fl).bytes));
        stage_bytes = std::max(stage_bytes, b);
    }
    uint8_t* stage = nullptr;
    if (cudaMalloc(&stage, stage_bytes) != cudaSuccess) return bail(FENCE_E_NOMEM, "model_load: staging allocation failed");
    struct StageFree {
        uint8_t* p;
        cudaStream_t s;
        ~StageFree() {
            if (p) cudaStreamSynchronize(s), cudaFree(p);
        }
    } stage_free{stage, st};
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerW& w = m->layers[l];
        LayerLaunch& L = m->launches[l];
        const int wq = wt_of(w.t_qkv), wo = wt_of(w.t_o), wg = wt_of(w.t_gu), wd = wt_of(w.t_down);
        const int o_item0 = (int)(TPR * qdl / 64), d_item0 = (int)(FTPR * Fl / 64);
        const RMat rq = carve(wq, QKVR, (int)H, 0), ro = carve(wo, (long long)H, (int)qdl, o_item0 & 3);
        // this rank's rows (q/k/v heads, FFN rows) and input columns (o_proj, down)
        const uint64_t rq_b = raw_row(w.t_qkv, H), rg_b = raw_row(w.t_gu, H), rd_b = raw_row(w.t_down, F);
        const ColCover oc = col_cover(w.t_o, q_c0, q_c0 + qdl), dc = col_cover(w.t_down, f_c0, f_c0 + Fl);
        const uint64_t obs = w.t_o == 14 ? 256 : 32, dbs = w.t_down == 14 ? 256 : 32;
        uint8_t* sp = stage;
        auto take = [&](size_t bytes) {
            uint8_t* p = sp;
            sp += a256(bytes);
            return p;
        };
        bool over = false;  // set if a piece would pass the staging buffer's end (checked before any copy)
        auto room = [&]() { over = over || sp > stage + stage_bytes; };
        uint8_t *sq = take(qdl * rq_b), *sk = take(kvdl * rq_b), *sv = take(kvdl * rq_b), *so = take(H * oc.bytes);
        room();
        if (over) return bail(FENCE_E_NOMEM, "model_load: staging plan too small");
        if (up.put(sq, w.q + TPR * qdl * rq_b, qdl * rq_b, qdl * rq_b, 1) ||
            up.put(sk, w.k + TPR * kvdl * rq_b, kvdl * rq_b, kvdl * rq_b, 1) ||
            up.put(sv, w.v + TPR * kvdl * rq_b, kvdl * rq_b, kvdl * rq_b, 1) ||
            up.put(so, w.o + oc.b0 * (oc.bytes / oc.nb), raw_row(w.t_o, qd), oc.bytes, H))
            return bail(FENCE_E_NOMEM, std::string("model_load: ") + fence_last_error());
        if (!fill(wq, sq, (long long)qdl, (int)H, rq, 0, 1) ||
            !fill(wq, sk, (long long)kvdl, (int)H, rq, (long long)qdl, 1) ||
            !fill(wq, sv, (long long)kvdl, (int)H, rq, (long long)(qdl + kvdl), 1) ||
            rmat_fill(wo, so, (long long)H, (int)qdl, ro, 0, 1, st, (int)(oc.nb * obs), (int)((q_c0 - oc.b0 * obs) / 64)) !=
                cudaSuccess)
            return bail(FENCE_E_NOMEM, "model_load: repacking failed");
        // FFN: the dense matrices, or every local expert's (expert e's rows start at e * F (gate/up)
        // and e * H (down) in the stacked tensors)
        RMat rg{}, rd{};
        for (int e = 0; e < n_ffn; ++e) {
            const uint64_t ge = moe ? (uint64_t)(m->e_lo + e) : 0;
            const RMat eg = carve(wg, 2 * (long long)Fl, (int)H, 0), ed = carve(wd, (long long)H, (int)Fl, d_item0 & 3);
            uint8_t *sg = take(Fl * rg_b), *su = take(Fl * rg_b), *sd = take(H * dc.bytes);
            room();
            if (over) return bail(FENCE_E_NOMEM, "model_load: staging plan too small");
            if (up.put(sg, w.gate + (ge * F + f_c0) * rg_b, Fl * rg_b, Fl * rg_b, 1) ||
                up.put(su, w.up + (ge * F + f_c0) * rg_b, Fl * rg_b, Fl * rg_b, 1) ||
                up.put(sd, w.down + ge * H * rd_b + dc.b0 * (dc.bytes / dc.nb), rd_b, dc.bytes, H))
                return bail(FENCE_E_NOMEM, std::string("model_load: ") + fence_last_error());
            if (!fill(wg, sg, (long long)Fl, (int)H, eg, 0, 2) || !fill(wg, su, (long long)Fl, (int)H, eg, 1, 2) ||
                rmat_fill(wd, sd, (long long)H, (int)Fl, ed, 0, 1, st, (int)(dc.nb * dbs),
                          (int)((f_c0 - dc.b0 * dbs) / 64)) != cudaSuccess)
                return bail(FENCE_E_NOMEM, "model_load: repacking failed");
            if (e == 0) rg = eg, rd = ed;
            if (moe) m->moe_gu[(size_t)l * m->e_n + e] = eg, m->moe_dn[(size_t)l * m->e_n + e] = ed;
        }
        float* bias = nullptr;
        if (any_bias) {
            bias = m->qkv_bias + (size_t)l * QKVR;
            if ((w.q_bias && cudaMemcpyAsync(bias, w.q_bias + TPR * qdl, qdl * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess) ||
                (w.k_bias && cudaMemcpyAsync(bias + qdl, w.k_bias + TPR * kvdl, kvdl * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess) ||
                (w.v_bias && cudaMemcpyAsync(bias + qdl + kvdl, w.v_bias + TPR * kvdl, kvdl * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess))
                return bail(FENCE_E_NOMEM, "model_load: bias upload failed");
        }
        if (!phase(L.qkv, rq, wq, (int)H, (int)QKVR, 0, wq == WT_Q6K ? X_NORM_R16 : X_NORM, EPI_STORE) ||
            !phase(L.o, ro, wo, (int)qdl, (int)H, 0, wo == WT_Q6K ? X_F32_R16 : X_F32, EPI_RESID) ||
            !phase(L.gu, rg, wg, (int)H, (int)Fl, 1, wg == WT_Q6K ? X_NORM_R16 : X_NORM, EPI_SWIGLU) ||
            !phase(L.down, rd, wd, (int)Fl, (int)H, 0, wd == WT_Q6K ? X_F16 : X_F32, EPI_RESID))
            return bail(FENCE_E_UNSUPPORTED, "model_load: a layer shape does not fit the streaming GEMV");
        L.qkv.a.x = m->hidden;
        L.qkv.a.norm_w = w.attn_norm;
        L.qkv.a.eps = c.rms_eps;
        L.qkv.a.y = m->qkv;  // [q | k | v], the fused matrix's row order
        L.qkv.a.bias = bias;
        L.o.a.x = m->attn_out;
        L.o.a.resid = m->hidden;
        L.gu.a.x = m->hidden;
        L.gu.a.norm_w = w.ffn_norm;
        L.gu.a.eps = c.rms_eps;
        L.gu.a.act = m->act;
        L.gu.a.act_f16 = (w.t_down == 14) ? 1 : 0;  // the reference rounds the down input to fp16
        L.down.a.x = m->act;
        L.down.a.resid = m->hidden;
        // attention
        AttnArgs at{};
        at.q = m->qkv;
        at.kc = static_cast<uint8_t*>(m->kcache) + l * kv_layer * 2;
        at.vc = static_cast<uint8_t*>(m->vcache) + l * kv_layer * 2;
        at.kc_w = const_cast<void*>(at.kc);
        at.vc_w = const_cast<void*>(at.vc);
        at.stride_t = SK_ATT_RSTR;
        at.stride_h = (long long)c.max_ctx * SK_ATT_RSTR;
        at.n_q_heads = Hq_l;
        at.n_kv_heads = Hkv_l;
        at.nchunk = m->attn_nchunk;
        at.part = m->attn_part;
        at.state = m->state;
        at.k_new = m->qkv + qdl;
        at.v_new = m->qkv + qdl + kvdl;
        at.q_norm_w = w.q_norm;
        at.k_norm_w = w.k_norm;
        at.eps = c.rms_eps;
        at.rope = m->rope;
        at.out = m->attn_out;
        at.counter = m->counters;
        L.attn = at;
    }
    // every layer's pieces are repacked: the staging buffer goes before the step kernel's tiles are built
    if (cudaStreamSynchronize(st) != cudaSuccess) return bail(FENCE_E_NOMEM, "model_load: upload / repack failed");
    cudaFree(stage);
    stage_free.p = nullptr;
    if (opts.verbose)
        printf("Weights streamed: %.2f GB in %.1f s\n", up.bytes / 1e9,
               std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
    // LM head: tied token_embd (the reference ignores output.weight, qwen3.cu:180-212,261)
    {
        const RMat rl = carve(WT_Q80, vn, (int)H, 0);
        if (!fill(WT_Q80, m->tok_embd + (size_t)v0 * (H / 32) * 34, vn, (int)H, rl, 0, 1))
            return bail(FENCE_E_NOMEM, "model_load: repacking failed");
        if (!phase(m->lm, rl, WT_Q80, (int)H, vn, 0, X_NORM, EPI_LMHEAD) || m->lm.p.grid > 4096)
            return bail(FENCE_E_UNSUPPORTED, "model_load: LM head shape not supported");
        RGemvArgs& a = m->lm.a;
        a.x = m->hidden;
        a.norm_w = m->out_norm;
        a.eps = c.rms_eps;
        a.logits = m->logits;
        a.cta_val = m->lm_val;
        a.cta_idx = m->lm_idx;
        a.counter = m->counters + Hkv_l;
        a.state = m->state;
        a.token_log = m->token_log;
        a.token_log_cap = m->token_log_cap;
    }
    m->prefill_ok = (opts.prefill && TPN == 1 && !moe) ? 1 : 0;
    if (opts.step_kernel && TPN == 1) {  // tensor parallel: once the ranks are connected (fence_tp_connect)
        const int rc = build_step_phases(m);
        if (rc != FENCE_OK) return bail(rc, std::string("model_load: ") + fence_last_error());
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(FENCE_E_NOMEM, "model_load: device error during setup");
    if (opts.use_graph && TPN == 1) {
        const int rc = capture_graph(m);
        if (rc != FENCE_OK) return bail(rc, std::string("model_load: graph capture failed: ") + fence_last_error());
    }
    m->h_logits.resize(c.vocab_size);
    if (opts.verbose) printf("Model ready!\n\n");
    return m;
}

extern "C" void fence_model_free(fence_model* m) { free_model(m); }

extern "C" int fence_step_trace(fence_model* m, int token, int pos, unsigned long long* host_out, int cap,
                                int* n_phases, int* n_ctas) {
    if (!m || !host_out) return set_error(FENCE_E_ARG, "step_trace: null argument");
    if (!m->use_step) return set_error(FENCE_E_UNSUPPORTED, "step_trace: the model was loaded without the step kernel");
    if (token < 0 || token >= m->cfg.vocab_size || pos < 0 || pos >= m->cfg.max_ctx)
        return set_error(FENCE_E_ARG, "step_trace: token %d / pos %d out of range", token, pos);
    const int NPH = m->sargs.nph, G = m->splan.grid;
    if (n_phases) *n_phases = NPH;
    if (n_ctas) *n_ctas = G;
    const size_t n = (size_t)G * NPH * SK_TRACE;
    if ((size_t)cap < n) return set_error(FENCE_E_ARG, "step_trace: needs %zu entries, got %d", n, cap);
    cudaSetDevice(m->dev);
    unsigned long long* d = nullptr;
    FENCE_CUDA_TRY(cudaMalloc(&d, n * sizeof(unsigned long long)));
    int rc = cuda_status(cudaMemsetAsync(d, 0, n * sizeof(unsigned long long), m->stream), "step_trace: clear");
    if (rc == FENCE_OK) rc = set_state(m, token, pos, 0);
    if (rc == FENCE_OK) {
        StepArgs a = m->sargs;
        a.trace = d;
        const cudaError_t e = (m->cfg.kv_dtype == FENCE_KV_F16) ? launch_step<__half>(a, m->splan, m->stream)
                                                                : launch_step<__nv_bfloat16>(a, m->splan, m->stream);
        rc = cuda_status(e, "step_trace: launch");
    }
    m->fwd_valid = 0;
    if (rc == FENCE_OK) rc = cuda_status(cudaStreamSynchronize(m->stream), "step_trace");
    if (rc == FENCE_OK)
        rc = cuda_status(cudaMemcpy(host_out, d, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost),
                         "step_trace: copy");
    cudaFree(d);
    return rc;
}

extern "C" int fence_model_config(const fence_model* m, fence_config* out) {
    if (!m || !out) return set_error(FENCE_E_ARG, "model_config: null argument");
    *out = m->cfg;
    return FENCE_OK;
}

extern "C" int fence_set_sampling(fence_model* m, float temperature, float top_p, int top_k, float rep) {
    if (!m) return set_error(FENCE_E_ARG, "set_sampling: null model");
    m->cfg.temperature = temperature;
    m->cfg.top_p = top_p;
    m->cfg.top_k = top_k;
    m->cfg.repetition_penalty = rep;
    return FENCE_OK;
}

extern "C" int fence_set_seed(fence_model* m, uint64_t seed) {
    if (!m) return set_error(FENCE_E_ARG, "set_seed: null model");
    m->rng.seed((std::mt19937::result_type)(seed ^ (seed >> 32)));
    return FENCE_OK;
}

extern "C" int fence_sample_nucleus_device(fence_model* m, const float* d_logits, const int* history, int n_history) {
    if (!m || !d_logits || n_history < 0 || (n_history > 0 && !history))
        return set_error(FENCE_E_ARG, "sample_nucleus_device: bad arguments");
    const fence_config& c = m->cfg;
    if (c.temperature <= 0.0f || c.top_k <= 1) return fence_sample_greedy(m, d_logits);
    if (m->tp_n > 1) return set_error(FENCE_E_UNSUPPORTED, "sample_nucleus_device: a tensor-parallel rank holds a vocabulary shard");
    cudaSetDevice(m->dev);
    const size_t need = fence_sample_scratch_bytes(c.vocab_size, c.top_k);
    if (!need) return set_error(FENCE_E_UNSUPPORTED, "sample_nucleus_device: top_k %d (the device sampler takes 2..256)", c.top_k);
    if (m->samp_bytes < need) {
        cudaFree(m->samp_scratch);
        m->samp_scratch = nullptr;
        m->samp_bytes = 0;
        FENCE_CUDA_TRY(cudaMalloc(&m->samp_scratch, need));
        m->samp_bytes = need;
    }
    if (!m->samp_out) FENCE_CUDA_TRY(cudaMalloc(&m->samp_out, sizeof(int)));
    if (n_history > m->samp_hist_cap) {
        cudaFree(m->samp_hist);
        m->samp_hist = nullptr;
        m->samp_hist_cap = 0;
        FENCE_CUDA_TRY(cudaMalloc(&m->samp_hist, (size_t)n_history * sizeof(int)));
        m->samp_hist_cap = n_history;
    }
    if (n_history > 0)
        FENCE_CUDA_TRY(cudaMemcpyAsync(m->samp_hist, history, (size_t)n_history * sizeof(int), cudaMemcpyHostToDevice,
                                       m->stream));
    // the one draw std::discrete_distribution makes (libstdc++: generate_canonical<double, 53>)
    const double u = std::generate_canonical<double, 53>(m->rng);
    int rc = fence_sample_nucleus_dev(d_logits, c.vocab_size, m->samp_hist, n_history, c.temperature, c.top_p, c.top_k,
                                      c.repetition_penalty, c.min_p, c.dynamic_temp, u, m->samp_scratch, m->samp_bytes,
                                      m->samp_out, m->stream);
    if (rc) return rc;
    FENCE_CUDA_TRY(cudaMemcpyAsync(m->h_token, m->samp_out, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return *m->h_token;
}

extern "C" const float* fence_forward(fence_model* m, int token_id, int pos) {
    if (!m) {
        set_error(FENCE_E_ARG, "forward: null model");
        return nullptr;
    }
    if (token_id < 0 || token_id >= m->cfg.vocab_size || pos < 0 || pos >= m->cfg.max_ctx) {
        set_error(FENCE_E_ARG, "forward: token %d / pos %d out of range", token_id, pos);
        return nullptr;
    }
    cudaSetDevice(m->dev);
    m->fwd_valid = 0;
    if (set_state(m, token_id, pos, 0) != FENCE_OK) return nullptr;
    if (run_step(m) != FENCE_OK) return nullptr;
    if (fetch_state(m) != FENCE_OK) return nullptr;
    if (cuda_status(cudaStreamSynchronize(m->stream), "forward") != FENCE_OK) return nullptr;
    if (state_status(m, "forward") != FENCE_OK) return nullptr;
    m->fwd_valid = 1;  // h_out->token is the greedy id of these logits
    return m->logits;
}

namespace {

// Scratch of the batched prefill for chunks of up to `cap` tokens (allocated once, on first use).
int prefill_scratch(fence_model* m, int cap) {
    if (m->pf_cap >= cap) return FENCE_OK;
    const fence_config& c = m->cfg;
    const size_t H = c.embed_dim, F = c.ff_dim, qd = (size_t)c.n_heads * c.head_dim,
                 QKVR = qd + 2 * (size_t)c.n_kv_heads * c.head_dim;
    size_t wmax = 0, rmax = 0;
    auto see = [&](const RPhase& r) {
        wmax = std::max(wmax, (size_t)r.a.Mv * (r.a.dual ? 2 : 1) * (size_t)r.a.I * 64);
        rmax = std::max(rmax, (size_t)r.a.Mv * (r.a.dual ? 2 : 1));
    };
    for (const LayerLaunch& L : m->launches) {
        see(L.qkv);
        see(L.o);
        see(L.gu);
        see(L.down);
    }
    cudaFree(m->pf_tok), cudaFree(m->pf_hidden), cudaFree(m->pf_qkv), cudaFree(m->pf_q), cudaFree(m->pf_attn);
    cudaFree(m->pf_bscale), cudaFree(m->pf_x16), cudaFree(m->pf_act), cudaFree(m->pf_w);
    m->pf_cap = 0;
    const size_t P = (size_t)cap;
    if (cudaMalloc(&m->pf_tok, P * 4) != cudaSuccess || cudaMalloc(&m->pf_hidden, P * H * 4) != cudaSuccess ||
        cudaMalloc(&m->pf_qkv, P * QKVR * 4) != cudaSuccess || cudaMalloc(&m->pf_q, P * qd * 4) != cudaSuccess ||
        cudaMalloc(&m->pf_attn, P * qd * 4) != cudaSuccess || cudaMalloc(&m->pf_bscale, rmax * 4) != cudaSuccess ||
        cudaMalloc(&m->pf_x16, P * std::max(H, qd) * 2) != cudaSuccess || cudaMalloc(&m->pf_act, P * F * 2) != cudaSuccess ||
        cudaMalloc(&m->pf_w, wmax * 2) != cudaSuccess)
        return set_error(FENCE_E_NOMEM, "prefill: scratch allocation failed");
    m->pf_cap = cap;
    return FENCE_OK;
}

// One linear of the chunk: its repacked weights dequantised to fp16 rows, then the tensor-core GEMM
// with the given epilogue.
template <int EPI>
int prefill_linear(fence_model* m, const RPhase& r, const __half* A, int P, TGArgs a) {
    const int rows = r.a.Mv * (r.a.dual ? 2 : 1);
    FENCE_CUDA_TRY(launch_dequant(r.a.wt, r.a.w, rows, r.a.I, m->pf_w, m->pf_bscale, m->stream));
    a.bscale = m->pf_bscale;
    a.P = P;
    a.N = rows;
    a.K = r.a.I * 64;
    FENCE_CUDA_TRY(launch_tc_gemm<EPI>(a, A, m->pf_w, m->stream));
    return FENCE_OK;
}

// tokens[0 .. n) at positions pos0 .. pos0 + n - 1 through every layer in chunks: the K/V cache rows
// of those positions are written (the residual stream of the chunk is not needed afterwards).
int prefill_batched(fence_model* m, const int* tokens, int n, int pos0) {
    const fence_config& c = m->cfg;
    const int H = c.embed_dim, HD = c.head_dim, Hq = c.n_heads, Hkv = c.n_kv_heads, qd = Hq * HD,
              QKVR = qd + 2 * Hkv * HD, F = c.ff_dim;
    const int cap = std::min(n, 2048);
    if (const int rc = prefill_scratch(m, std::max(cap, m->pf_cap))) return rc;
    cudaStream_t st = m->stream;
    const size_t kv_layer = (size_t)Hkv * c.max_ctx * SK_ATT_RSTR;
    const long long stride_h = (long long)c.max_ctx * SK_ATT_RSTR;
    for (int c0 = 0; c0 < n; c0 += cap) {
        const int P = std::min(cap, n - c0), p0 = pos0 + c0;
        FENCE_CUDA_TRY(cudaMemcpyAsync(m->pf_tok, tokens + c0, (size_t)P * 4, cudaMemcpyHostToDevice, st));
        FENCE_CUDA_TRY(cudaStreamSynchronize(st));  // the host ids may be reused by the caller
        embed_rows_kernel<<<P, 256, 0, st>>>(m->tok_embd, m->pf_tok, H, m->pf_hidden);
        for (int l = 0; l < c.n_layers; ++l) {
            const LayerLaunch& L = m->launches[l];
            const LayerW& w = m->layers[l];
            rmsnorm_rows_kernel<<<P, 256, 0, st>>>(m->pf_hidden, w.attn_norm, H, c.rms_eps, m->pf_x16);
            TGArgs a{};
            a.C = m->pf_qkv;
            a.ldc = QKVR;
            a.bias = L.qkv.a.bias;
            if (const int rc = prefill_linear<TG_EPI_STORE>(m, L.qkv, m->pf_x16, P, a)) return rc;
            uint8_t* kc = static_cast<uint8_t*>(m->kcache) + (size_t)l * kv_layer * 2;
            uint8_t* vc = static_cast<uint8_t*>(m->vcache) + (size_t)l * kv_layer * 2;
            if (c.kv_dtype == FENCE_KV_BF16) {
                auto* k16 = reinterpret_cast<__nv_bfloat16*>(kc);
                auto* v16 = reinterpret_cast<__nv_bfloat16*>(vc);
                prefill_qk_kernel<__nv_bfloat16><<<P, 128, 0, st>>>(m->pf_qkv, QKVR, Hq, Hkv, w.q_norm, w.k_norm,
                                                                    c.rms_eps, m->rope, p0, m->pf_q, k16, v16, stride_h,
                                                                    SK_ATT_RSTR);
                FENCE_CUDA_TRY(launch_prefill_attn<__nv_bfloat16>(m->pf_q, Hq, Hkv, k16, v16, stride_h, SK_ATT_RSTR, p0, P,
                                                                  m->pf_attn, st));
            } else {
                auto* k16 = reinterpret_cast<__half*>(kc);
                auto* v16 = reinterpret_cast<__half*>(vc);
                prefill_qk_kernel<__half><<<P, 128, 0, st>>>(m->pf_qkv, QKVR, Hq, Hkv, w.q_norm, w.k_norm, c.rms_eps,
                                                             m->rope, p0, m->pf_q, k16, v16, stride_h, SK_ATT_RSTR);
                FENCE_CUDA_TRY(launch_prefill_attn<__half>(m->pf_q, Hq, Hkv, k16, v16, stride_h, SK_ATT_RSTR, p0, P,
                                                           m->pf_attn, st));
            }
            f32_to_f16_rows_kernel<<<592, 256, 0, st>>>(m->pf_attn, (long long)P * qd, m->pf_x16);
            a = TGArgs{};
            a.C = m->pf_hidden;
            a.ldc = H;
            if (const int rc = prefill_linear<TG_EPI_ADD>(m, L.o, m->pf_x16, P, a)) return rc;
            rmsnorm_rows_kernel<<<P, 256, 0, st>>>(m->pf_hidden, w.ffn_norm, H, c.rms_eps, m->pf_x16);
            a = TGArgs{};
            a.H = m->pf_act;
            a.ldh = F;
            if (const int rc = prefill_linear<TG_EPI_SWIGLU>(m, L.gu, m->pf_x16, P, a)) return rc;
            a = TGArgs{};
            a.C = m->pf_hidden;
            a.ldc = H;
            if (const int rc = prefill_linear<TG_EPI_ADD>(m, L.down, m->pf_act, P, a)) return rc;
        }
        FENCE_CUDA_TRY(cudaGetLastError());
    }
    return FENCE_OK;
}

}  // namespace

extern "C" const float* fence_prefill(fence_model* m, const int* tokens, int n, int pos0) {
    if (!m || !tokens || n <= 0 || pos0 < 0 || pos0 + n > (m ? m->cfg.max_ctx : 0)) {
        set_error(FENCE_E_ARG, "prefill: bad arguments (n=%d pos0=%d)", n, pos0);
        return nullptr;
    }
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab_size) {
            set_error(FENCE_E_ARG, "prefill: token %d out of range", tokens[i]);
            return nullptr;
        }
    cudaSetDevice(m->dev);
    if (m->prefill_ok && n > 1) {
        if (prefill_batched(m, tokens, n - 1, pos0) != FENCE_OK) return nullptr;
    } else {
        for (int i = 0; i + 1 < n; ++i)
            if (!fence_forward(m, tokens[i], pos0 + i)) return nullptr;
    }
    return fence_forward(m, tokens[n - 1], pos0 + n - 1);  // the last token through the decode step: its logits
}

extern "C" int fence_sample_greedy(fence_model* m, const float* d_logits) {
    if (!m || !d_logits) return set_error(FENCE_E_ARG, "sample_greedy: null argument");
    cudaSetDevice(m->dev);
    if (d_logits == m->logits && m->fwd_valid) return m->h_out->token;  // read back by fence_forward
    if (d_logits == m->logits) {
        // the LM head already reduced the argmax (reference tie order) into the decode state
        FENCE_CUDA_TRY(cudaMemcpyAsync(m->h_token, &m->state->token, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    } else {
        const int rc = fence_argmax(d_logits, m->lm_idx, m->cfg.vocab_size, m->stream);
        if (rc) return rc;
        FENCE_CUDA_TRY(cudaMemcpyAsync(m->h_token, m->lm_idx, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    }
    FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return *m->h_token;
}

extern "C" int fence_sample_nucleus(fence_model* m, const float* d_logits, const int* history, int n_history) {
    if (!m || !d_logits) return set_error(FENCE_E_ARG, "sample_nucleus: null argument");
    const fence_config& c = m->cfg;
    if (c.temperature <= 0.0f || c.top_k <= 1) return fence_sample_greedy(m, d_logits);
    if (m->tp_n > 1) return set_error(FENCE_E_UNSUPPORTED, "sample_nucleus: a tensor-parallel rank holds a vocabulary shard");
    cudaSetDevice(m->dev);
    FENCE_CUDA_TRY(cudaMemcpyAsync(m->h_logits.data(), d_logits, (size_t)c.vocab_size * 4, cudaMemcpyDeviceToHost, m->stream));
    FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return host_sample_nucleus(m->h_logits.data(), c.vocab_size, history, n_history, c.temperature, c.top_p, c.top_k,
                               c.repetition_penalty, c.min_p, c.dynamic_temp != 0, m->rng);
}

extern "C" int fence_generate(fence_model* m, const int* prompt, int n_prompt, int max_new, int eos_id, int* out,
                              int out_cap, int* n_out) {
    if (!m || !prompt || n_prompt <= 0 || !out || !n_out) return set_error(FENCE_E_ARG, "generate: bad arguments");
    if (n_prompt > m->cfg.max_ctx) return set_error(FENCE_E_ARG, "generate: prompt longer than max_ctx");
    cudaSetDevice(m->dev);
    m->fwd_valid = 0;
    std::vector<int> output(prompt, prompt + n_prompt);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->cfg.vocab_size) return set_error(FENCE_E_ARG, "generate: prompt id out of range");
    // prefill: all but the last prompt token batched on the tensor cores where the model allows it,
    // else token by token as in the reference (qwen3.cu:478-481); the last one through the decode
    // step, which leaves its logits; no host sync between tokens
    int first = 0;
    if (m->prefill_ok && n_prompt > 1) {
        if (const int rc = prefill_batched(m, prompt, n_prompt - 1, 0)) return rc;
        first = n_prompt - 1;
    }
    for (int i = first; i < n_prompt; ++i) {
        int rc = set_state(m, prompt[i], i, 0);
        if (!rc) rc = run_step(m);
        if (rc) return rc;
    }
    FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    int pos = n_prompt;
    for (int i = 0; i < max_new && pos < m->cfg.max_ctx; ++i) {
        const int next = fence_sample_nucleus(m, m->logits, output.data(), (int)output.size());
        if (next < 0) return next;
        if (next == eos_id) break;
        output.push_back(next);
        int rc = set_state(m, next, pos, 0);
        if (!rc) rc = run_step(m);
        if (rc) return rc;
        ++pos;
    }
    if (const int fr = fetch_state(m)) return fr;
    FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    if (const int st = state_status(m, "generate")) return st;
    const int n = (int)std::min<size_t>(output.size(), (size_t)out_cap);
    std::copy(output.begin(), output.begin() + n, out);
    *n_out = (int)output.size();
    return FENCE_OK;
}

extern "C" int fence_decode_greedy(fence_model* m, int token, int pos, int n_steps, int* out_tokens) {
    if (!m || n_steps < 0 || !out_tokens) return set_error(FENCE_E_ARG, "decode_greedy: bad arguments");
    if (pos < 0 || pos + n_steps > m->cfg.max_ctx || n_steps > m->token_log_cap)
        return set_error(FENCE_E_ARG, "decode_greedy: positions [%d, %d) exceed max_ctx", pos, pos + n_steps);
    cudaSetDevice(m->dev);
    m->fwd_valid = 0;
    int rc = set_state(m, token, pos, 0);
    if (rc) return rc;
    for (int s = 0; s < n_steps; ++s)
        if ((rc = run_step(m))) return rc;
    FENCE_CUDA_TRY(cudaMemcpyAsync(out_tokens, m->token_log, (size_t)n_steps * sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    if ((rc = fetch_state(m))) return rc;
    FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return state_status(m, "decode_greedy");
}

extern "C" int fence_time_decode(fence_model* m, int token, int pos, int n_steps, float* ms) {
    if (!m || !ms || n_steps <= 0) return set_error(FENCE_E_ARG, "time_decode: bad arguments");
    if (pos < 0 || pos + n_steps > m->cfg.max_ctx) return set_error(FENCE_E_ARG, "time_decode: positions exceed max_ctx");
    cudaSetDevice(m->dev);
    m->fwd_valid = 0;
    cudaEvent_t e0, e1;
    FENCE_CUDA_TRY(cudaEventCreate(&e0));
    FENCE_CUDA_TRY(cudaEventCreate(&e1));
    int rc = set_state(m, token, pos, 0);
    if (!rc) rc = cuda_status(cudaEventRecord(e0, m->stream), "event record");
    for (int s = 0; s < n_steps && !rc; ++s) rc = run_step(m);
    if (!rc) rc = cuda_status(cudaEventRecord(e1, m->stream), "event record");
    if (!rc) rc = cuda_status(cudaEventSynchronize(e1), "event sync");
    if (!rc) rc = cuda_status(cudaEventElapsedTime(ms, e0, e1), "elapsed");
    if (!rc) rc = fetch_state(m);
    if (!rc) rc = cuda_status(cudaStreamSynchronize(m->stream), "time_decode");
    if (!rc) rc = state_status(m, "time_decode");
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return rc;
}

extern "C" int fence_tp_handle(fence_model* m, void* out, int cap) {
    if (!m || !out || cap < FENCE_TP_HANDLE_BYTES) return set_error(FENCE_E_ARG, "tp_handle: bad arguments");
    if (m->tp_n < 2) return set_error(FENCE_E_ARG, "tp_handle: the model was loaded with tp_size 1");
    static_assert(sizeof(cudaIpcMemHandle_t) <= FENCE_TP_HANDLE_BYTES, "handle size");
    cudaSetDevice(m->dev);
    cudaIpcMemHandle_t h;
    FENCE_CUDA_TRY(cudaIpcGetMemHandle(&h, m->xbuf));
    std::memset(out, 0, FENCE_TP_HANDLE_BYTES);
    std::memcpy(out, &h, sizeof h);
    return FENCE_OK;
}

extern "C" int fence_tp_connect(fence_model* m, const void* handles, int n_ranks) {
    if (!m || !handles) return set_error(FENCE_E_ARG, "tp_connect: null argument");
    if (m->tp_n < 2 || n_ranks != m->tp_n)
        return set_error(FENCE_E_ARG, "tp_connect: %d handles for a model of tp_size %d", n_ranks, m->tp_n);
    if (m->tp_connected) return set_error(FENCE_E_ARG, "tp_connect: already connected");
    cudaSetDevice(m->dev);
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int p = 0; p < n_ranks; ++p) {
        if (p == m->tp_rank) {
            m->xpeer[p] = m->xbuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)p * FENCE_TP_HANDLE_BYTES, sizeof h);
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error((int)e, "tp_connect: rank %d's exchange buffer: %s", p, cudaGetErrorString(e));
        m->xpeer[p] = static_cast<uint8_t*>(ptr);
    }
    int rc = build_step_phases(m);
    if (rc != FENCE_OK) return rc;
    FENCE_CUDA_TRY(cudaDeviceSynchronize());
    if (m->opts.use_graph) {
        rc = capture_graph(m);
        if (rc != FENCE_OK) return rc;
    }
    m->tp_connected = 1;
    return FENCE_OK;
}

extern "C" int fence_copy_logits(fence_model* m, float* host_out) {
    if (!m || !host_out) return set_error(FENCE_E_ARG, "copy_logits: null argument");
    cudaSetDevice(m->dev);
    FENCE_CUDA_TRY(cudaMemcpyAsync(host_out, m->logits, (size_t)m->vocab_n * 4, cudaMemcpyDeviceToHost, m->stream));
    FENCE_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return FENCE_OK;
}
