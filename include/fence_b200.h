/*
 * fence_b200.h — C-ABI of the B200 (sm_100a) decode engine for Fence's GGUF token loop.
 *
 * Two layers live behind this header, both exported from libfence_b200.so with C linkage:
 *
 *  1. Drop-in kernel launchers. Each `fence_<name>` replaces the inline host launcher of the same
 *     name in the reference's header-only kernels (src/kernels/gemv_q6k.cuh, gemv_q8_0.cuh, ops.cuh):
 *     same argument order, same meaning, caller-owned device pointers, asynchronous on `stream`,
 *     never allocate. They return a status (0 = ok, else a cudaError_t value or a FENCE_E_* code),
 *     where the reference returned void and left errors to the caller's next CUDA_CHECK.
 *     Under C++ the header also defines `inline` wrappers with the reference's exact names, void
 *     return and `cudaStream_t stream = 0` default, so reference call sites compile unchanged.
 *
 *  2. The engine: the reference's Qwen3Model (src/model/qwen3.h:115-155) — load / forward /
 *     sample_greedy / sample_nucleus / generate — as opaque-handle C functions, plus the
 *     synthetic-GGUF writer used by the tests and the benchmark.
 *
 * Layout contracts (identical to the reference):
 *   block_q6_K  src/kernels/q6k_types.h:27-32   210 B / 256 weights: ql[128] qh[64] int8 scales[16] fp16 d
 *   block_q8_0  src/kernels/q8_0_types.h:11-14   34 B / 32 weights: fp16 d, int8 qs[32]
 *   Weight matrix W[M x K]: M rows, each row K/256 (Q6_K) or K/32 (Q8_0) consecutive blocks;
 *   the GGUF dims of such a tensor are [K, M] (ne0 = input, ne1 = output).
 *   KV cache (drop-in store_kv / gqa_attention): [max_ctx][n_kv_heads * head_dim] fp16 per layer.
 *
 * Preconditions beyond the reference's: weight pointers handed to the GEMV launchers must be
 * 16-byte aligned (cudaMalloc and GGUF's 32-byte tensor alignment both give that); violations
 * return FENCE_E_ALIGN instead of launching.
 */
#ifndef FENCE_B200_H
#define FENCE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st; /* cudaStream_t is `struct CUstream_st*`; pass one directly (NULL = legacy stream). */
typedef struct CUstream_st* fence_stream_t;

/* ---- status codes (negative: library codes; positive: cudaError_t values) ---- */
#define FENCE_OK              0
#define FENCE_E_ARG         (-1)  /* bad shape / null pointer / unsupported size              */
#define FENCE_E_ALIGN       (-2)  /* pointer alignment precondition violated                  */
#define FENCE_E_FORMAT      (-3)  /* GGUF file malformed or missing tensors / metadata        */
#define FENCE_E_UNSUPPORTED (-4)  /* a tensor type or shape the engine does not handle        */
#define FENCE_E_DEVICE_WAIT (-5)  /* a device-side bounded wait expired (kernel gave up)       */
#define FENCE_E_IO          (-6)  /* file could not be opened / written                       */
#define FENCE_E_NOMEM       (-7)  /* device or host allocation failed                         */
#define FENCE_E_SCRATCH     (-8)  /* request exceeds a fixed static scratch (see *_static)    */

/* Thread-local text of the last error raised by any fence_* call on this thread ("" if none). */
const char* fence_last_error(void);
/* Returns and clears the device-side error word that kernels set when a bounded wait expires
 * (0 if none). Synchronises the device. */
int fence_device_error(void);

/* ---- quant block types (byte-identical to the reference) ---- */
#pragma pack(push, 1)
typedef struct block_q6_K {
    uint8_t ql[128];     /* low 4 bits of each 6-bit quant, 2 per byte          */
    uint8_t qh[64];      /* high 2 bits, 4 per byte                              */
    int8_t  scales[16];  /* signed scale per 16-element sub-block               */
#if defined(__cplusplus) && defined(__CUDA_FP16_TYPES_EXIST__) && !defined(FENCE_BUILDING_LIBRARY)
    __half  d;           /* fp16 super-block scale                               */
#else
    uint16_t d;          /* fp16 super-block scale (IEEE binary16 bits)          */
#endif
} block_q6_K;
typedef struct block_q8_0 {
#if defined(__cplusplus) && defined(__CUDA_FP16_TYPES_EXIST__) && !defined(FENCE_BUILDING_LIBRARY)
    __half  d;
#else
    uint16_t d;
#endif
    int8_t  qs[32];
} block_q8_0;
#pragma pack(pop)

/* =====================================================================================
 * 1. Drop-in kernel launchers. All pointers are device pointers owned by the caller.
 *    fp16 buffers are passed as uint16_t* (IEEE binary16 bit patterns, i.e. __half*).
 * ===================================================================================== */

/* Launch flags of the drop-in GEMVs (process-wide; returns the previous flags).
 * FENCE_LAUNCH_PDL: launch with programmatic dependent launch, so a GEMV starts streaming its
 * weights while the preceding kernel in the stream is still running (its reads of x wait for that
 * kernel to finish). Set it only when no earlier work in the stream writes the weight matrices.
 * No counterpart in the reference (its launchers take only the stream). */
#define FENCE_LAUNCH_PDL 1
int fence_set_launch_flags(int flags);

/* y[M] = W_q6k[M x K] . x[K]; x fp16, y fp32, K % 256 == 0.
 * Replaces gemv_q6k, src/kernels/gemv_q6k.cuh:89-102. */
int fence_gemv_q6k(const block_q6_K* W, const uint16_t* x, float* y, int M, int K,
                   fence_stream_t stream);
/* y = W.x + bias. Replaces gemv_q6k_bias, src/kernels/gemv_q6k.cuh:140-151. */
int fence_gemv_q6k_bias(const block_q6_K* W, const uint16_t* x, const float* bias, float* y,
                        int M, int K, fence_stream_t stream);
/* y[M] = W_q8_0[M x K] . x[K]; x fp32, y fp32, K % 32 == 0.
 * Replaces gemv_q8_0, src/kernels/gemv_q8_0.cuh:99-104. */
int fence_gemv_q8_0(const block_q8_0* W, const float* x, float* y, int M, int K,
                    fence_stream_t stream);
/* out[0..dim) = dequant(row token_id of a Q8_0 matrix with `dim` columns).
 * Replaces embed_q8_0, src/kernels/gemv_q8_0.cuh:31-36. */
int fence_embed_q8_0(float* out, const block_q8_0* weight, int token_id, int dim,
                     fence_stream_t stream);

/* out[i] = w[i] * x[i] * rsqrt(mean(x^2) + eps). Replaces rms_norm, src/kernels/ops.cuh:47-51. */
int fence_rms_norm(float* out, const float* x, const float* w, int n, float eps,
                   fence_stream_t stream);
/* In-place form. Replaces rms_norm_inplace, src/kernels/ops.cuh:54-60. */
int fence_rms_norm_inplace(float* x, const float* w, int n, float eps, fence_stream_t stream);
/* RMSNorm of each head_dim slice of x (n_heads slices), weight w[head_dim] shared by all heads.
 * Replaces rms_norm_per_head, src/kernels/ops.cuh:97-103. */
int fence_rms_norm_per_head(float* x, const float* w, int n_heads, int head_dim, float eps,
                            fence_stream_t stream);
/* NeoX-pair rotary embedding of q [n_q_heads*head_dim] and k [n_kv_heads*head_dim] in place:
 * pair (i, i+head_dim/2), angle = pos * freq_base^(-2i/head_dim).
 * Replaces apply_rope, src/kernels/ops.cuh:169-177. */
int fence_apply_rope(float* q, float* k, int head_dim, int n_q_heads, int n_kv_heads, int pos,
                     float freq_base, fence_stream_t stream);
/* out[i] = gate[i] / (1 + exp(-gate[i])) * up[i]. Replaces silu_elementwise_mul, ops.cuh:197-202. */
int fence_silu_elementwise_mul(float* out, const float* gate, const float* up, int n,
                               fence_stream_t stream);
/* x[i] += residual[i]. Replaces residual_add, src/kernels/ops.cuh:265-270. */
int fence_residual_add(float* x, const float* residual, int n, fence_stream_t stream);
/* In-place softmax of x[0..n). Replaces softmax, src/kernels/ops.cuh:248-251. */
int fence_softmax(float* x, int n, fence_stream_t stream);
/* fp32 -> fp16 (round to nearest even). Replaces f32_to_f16, ops.cuh:457-462, and
 * float_to_half, ops.cuh:284-289 (same operation). */
int fence_f32_to_f16(uint16_t* out, const float* in, int n, fence_stream_t stream);
int fence_float_to_half(uint16_t* out, const float* in, int n, fence_stream_t stream);
/* fp16 -> fp32. Replaces half_to_float, src/kernels/ops.cuh:303-308. */
int fence_half_to_float(float* out, const uint16_t* in, int n, fence_stream_t stream);
/* k_cache[pos*kv_dim + i] = fp16(k[i]), same for v. Replaces store_kv, ops.cuh:435-443. */
int fence_store_kv(uint16_t* k_cache, uint16_t* v_cache, const float* k, const float* v, int pos,
                   int kv_dim, int max_ctx, fence_stream_t stream);
/* Single-query grouped-query attention over positions [0, seq_len) of an fp16 KV cache laid out
 * [max_ctx][n_kv_heads*head_dim]; q head h reads kv head h / (n_q_heads/n_kv_heads).
 * score_buf: caller scratch of n_q_heads*max_ctx floats, as in the reference; this engine keeps
 * its split-context partial results there. head_dim must be 64, 128 or 256.
 * Replaces gqa_attention, src/kernels/ops.cuh:405-414. */
int fence_gqa_attention(float* attn_out, const float* q, const uint16_t* k_cache,
                        const uint16_t* v_cache, int head_dim, int n_q_heads, int n_kv_heads,
                        int seq_len, int max_ctx, float* score_buf, fence_stream_t stream);
/* *result = index of the largest x[i], with the reference's tie order (256-thread strided scan,
 * then a tree that keeps the lower position on ties): among equal maxima the index whose
 * (i mod 256) has the smallest 8-bit reversal wins, then the smallest index; NaN and values
 * <= -1e30 never win; 0 when nothing qualifies. Replaces argmax, src/kernels/ops.cuh:501-505. */
int fence_argmax(const float* x, int* result, int n, fence_stream_t stream);

/* Qwen3Model::sample_nucleus (src/model/qwen3.cu:351-460) on the device: repetition penalty once
 * per occurrence of a token in `history` (device ids), min-p cut, entropy-scaled temperature,
 * softmax, top_k largest probabilities (ties to the smaller id), the shortest prefix reaching
 * top_p, then the draw std::discrete_distribution makes, with the caller's uniform u in [0, 1)
 * (the kept weights normalised and accumulated in double; the first id whose cumulative is >= u).
 * Only the id (*out_id, device) leaves the device, where the reference copies the whole logits
 * vector to the host and sorts it. top_k in 2..256 and temperature > 0 (greedy decoding is
 * fence_argmax); history up to 65536 ids. Caller-owned scratch of fence_sample_scratch_bytes(vocab,
 * top_k) bytes, 256-byte aligned; logits are not modified. Sums run in a fixed tree order, so a
 * probability differs from the reference's sequential float sum in its last bits. */
size_t fence_sample_scratch_bytes(int vocab, int top_k);
int fence_sample_nucleus_dev(const float* logits, int vocab, const int* history, int n_history, float temperature,
                             float top_p, int top_k, float rep_penalty, float min_p, int dynamic_temp, double u,
                             void* scratch, size_t scratch_bytes, int* out_id, fence_stream_t stream);

/* No counterpart in the reference. fence_gqa_attention without score_buf, for callers that cannot
 * allocate at the call site (a foreign-language binding handed only the operands, or a per-token
 * host loop that must not call the device-synchronising cudaMalloc). Allocates nothing: the
 * split-context partials live in a per-device static array of FENCE_ATTN_STATIC_FLOATS floats
 * (2 MiB). Same split and same results as fence_gqa_attention; a call that needs more than the
 * array (n_q_heads * chunks * (head_dim + 2) floats, chunks as in fence_gqa_attention) returns
 * FENCE_E_SCRATCH without launching. At head_dim 128 and 64 chunks that admits up to 63 query
 * heads, at head_dim 256 up to 31. The first call on each device resolves the array's address
 * (cudaGetSymbolAddress) and caches it per device ordinal; make that first call before any stream
 * capture. The cache does not survive cudaDeviceReset: after a reset of a device the address may
 * change, so do not call this entry point on that device again in the same process. Calls that
 * overlap in time on one device race on the shared array: order them on one stream. */
#define FENCE_ATTN_STATIC_FLOATS 524288
int fence_gqa_attention_static(float* attn_out, const float* q, const uint16_t* k_cache,
                               const uint16_t* v_cache, int head_dim, int n_q_heads, int n_kv_heads,
                               int seq_len, int max_ctx, fence_stream_t stream);

/* =====================================================================================
 * 2. Engine — the reference's Qwen3Model (src/model/qwen3.h:115-155) as a C handle.
 * ===================================================================================== */

typedef struct fence_model fence_model;

typedef struct fence_config {
    int   n_layers, embed_dim, ff_dim, n_heads, n_kv_heads, head_dim, vocab_size, max_ctx;
    float rope_freq_base, rms_eps;
    /* sampling parameters (src/model/qwen3.h:31-37 defaults) */
    float temperature, top_p;
    int   top_k;
    float repetition_penalty, min_p;
    int   dynamic_temp;
    /* engine facts */
    int   linear_type;      /* GGML type id of the attention/FFN linears: 14 = Q6_K, 8 = Q8_0 */
    int   embd_type;        /* GGML type id of token_embd (8 = Q8_0)                        */
    int   has_qk_norm;      /* attn_q_norm/attn_k_norm present                               */
    int   n_experts, n_experts_used;
    int   kv_dtype;         /* FENCE_KV_BF16 or FENCE_KV_F16                                 */
    int   tp_rank, tp_size;
    size_t weight_bytes;    /* bytes of weights streamed per decode token (this rank)        */
} fence_config;

#define FENCE_KV_F16  0
#define FENCE_KV_BF16 1

typedef struct fence_load_opts {
    int max_ctx;        /* context length to allocate (reference default 4096)            */
    int kv_dtype;       /* FENCE_KV_F16 (default, the reference cache type) or FENCE_KV_BF16 */
    int device;         /* CUDA device ordinal                                            */
    int use_graph;      /* capture the token step in a CUDA graph (default 1)             */
    int verbose;        /* print the reference's load banner                              */
    /* tensor parallel: rank `tp_rank` of `tp_size` (see fence_tp_connect); the ranks exchange
     * inside the step kernel over NVLink peer memory, so no communicator is passed */
    int tp_rank, tp_size;
    /* 1 (default): the whole token step is one persistent kernel (weights of all phases stream
     * continuously, phases separated by a grid-wide counter); 0: one kernel per phase            */
    int step_kernel;
    /* Test only, no counterpart in the reference: index of a step-kernel phase whose grid-counter
     * wait is given a target that no CTA ever reaches, so that this bounded wait runs out (about a
     * second), the step ends early with invalid results and the error surfaces as
     * FENCE_E_DEVICE_WAIT (fence_device_error, and the status of the engine calls that sync).
     * -1 (the default) = off. */
    int wait_test_phase;
    /* Sparse MoE models under tensor parallelism (no counterpart in the reference, which has no
     * expert tensors): 0 (default) = every rank holds a 1/tp_size slice of every expert's FFN rows
     * (all ranks stream both routed experts); 1 = expert parallel, rank r holds the experts
     * [r * E / tp_size, (r + 1) * E / tp_size) whole (only the ranks holding a routed expert
     * stream). Ignored for dense models and one rank. */
    int moe_ep;
    /* 1 (default): keep the repacked row-major weights next to the step kernel's tiles so that
     * fence_prefill / fence_generate run the prompt as batched tensor-core GEMMs (one rank, dense
     * FFN; about the model's weight bytes again in device memory); 0: free them (prefill token by
     * token, as the reference does). */
    int prefill;
} fence_load_opts;

/* Fills *opts with defaults (max_ctx 4096, fp16 KV, device 0, graphs on, single rank, step kernel,
 * wait_test_phase -1, moe_ep 0, prefill 1). */
void fence_load_opts_default(fence_load_opts* opts);

/* Qwen3Model::load (src/model/qwen3.cu:116-228): mmap the GGUF, read the config from its metadata
 * (same keys, types and fallbacks), upload weights, allocate KV cache and scratch.
 * Returns NULL on failure (fence_last_error() says why). */
fence_model* fence_model_load(const char* gguf_path, const fence_load_opts* opts);
/* Qwen3Model::unload. Safe on NULL. */
void fence_model_free(fence_model* m);
int  fence_model_config(const fence_model* m, fence_config* out);
/* Sets the sampling parameters the CLI flags --temp/--top-p/--top-k/--rep-penalty set. */
int  fence_set_sampling(fence_model* m, float temperature, float top_p, int top_k,
                        float repetition_penalty);

/* Qwen3Model::forward (qwen3.cu:241-265): one token at position pos; returns the DEVICE pointer
 * of the fp32 logits [vocab] (valid until the next forward), NULL on error. */
const float* fence_forward(fence_model* m, int token_id, int pos);
/* The prefill loop of Qwen3Model::generate (qwen3.cu:478-481: forward(prompt[i], i) per token) for
 * tokens[0 .. n) at positions pos0 .. pos0 + n - 1: the same K/V cache rows and, for the last token,
 * the same logits (device pointer returned, as fence_forward). With opts.prefill on one rank and a
 * dense FFN, all tokens but the last run as batched fp16 tensor-core GEMMs (weights dequantised per
 * layer; logits within the decode path's tolerance, not bit-identical); otherwise token by token. */
const float* fence_prefill(fence_model* m, const int* tokens, int n, int pos0);
/* Qwen3Model::sample_greedy (qwen3.cu:344-349): argmax of device logits, reference tie order. */
int fence_sample_greedy(fence_model* m, const float* d_logits);
/* Qwen3Model::sample_nucleus (qwen3.cu:351-460): repetition penalty per occurrence in history,
 * min-p 0.05, entropy-scaled temperature, top-k then top-p, draw from the survivors. The draw uses
 * the engine's seeded mt19937 (fence_set_seed) where the reference seeds from random_device. */
int fence_sample_nucleus(fence_model* m, const float* d_logits, const int* history, int n_history);
int fence_set_seed(fence_model* m, uint64_t seed);
/* sample_nucleus with the sampling steps on the device (fence_sample_nucleus_dev) and only the id
 * copied back: same parameters, same engine generator (one draw per call; the host path skips
 * its draw when a single token survives top-p), top_k up to 256. The first call allocates its
 * scratch. */
int fence_sample_nucleus_device(fence_model* m, const float* d_logits, const int* history, int n_history);

/* Qwen3Model::generate (qwen3.cu:463-519): prefill of `prompt` (all but its last token batched on
 * the tensor cores, fence_prefill, where the model allows it; else token by token as in the
 * reference), then up to max_new_tokens sampled tokens, stopping at eos_id (pass -1 for no stop
 * token) or max_ctx. out receives prompt + generated ids (capacity out_cap); *n_out their count.
 * Every sampled token crosses to the host, as in the reference. */
int fence_generate(fence_model* m, const int* prompt, int n_prompt, int max_new_tokens,
                   int eos_id, int* out, int out_cap, int* n_out);

/* Device-resident greedy decode: starting from (token, pos) already fed, run n_steps token steps
 * back to back with the sampled id fed to the next step on the device (no host round trip);
 * the n_steps sampled ids are copied to out_tokens (host) at the end. */
int fence_decode_greedy(fence_model* m, int token, int pos, int n_steps, int* out_tokens);

/* Last logits of the most recent step, copied to host (for parity tests): vocab_size floats, or
 * under tensor parallelism this rank's vocabulary shard (see fence_tp_connect). */
int fence_copy_logits(fence_model* m, float* host_out);

/* Tensor parallel (no counterpart in the reference, whose forward is single-GPU; the split is the
 * Megatron one: q/k/v heads and gate/up rows per rank, o_proj and down by input columns with their
 * partial rows summed over the ranks, the tied LM head by vocabulary rows). One process per GPU
 * loads the same GGUF with opts.tp_rank / opts.tp_size (step_kernel = 1); every rank then passes
 * its handle (FENCE_TP_HANDLE_BYTES, a CUDA IPC handle of its exchange buffer) to the others by
 * any host channel, and fence_tp_connect(handles of ranks 0..tp_size-1 in rank order) maps the
 * peers' buffers (NVLink P2P) and builds the step. The ranks must then call fence_forward /
 * fence_time_decode / fence_decode_greedy in lockstep with the same arguments: each step kernel
 * sends its partial rows to every rank and waits (bounded) for theirs. fence_forward returns this
 * rank's vocabulary shard of the logits (rows [tp_rank * ceil(V / tp_size), ...)); the greedy id
 * is the global one on every rank; fence_sample_nucleus is not available per shard. */
#define FENCE_TP_HANDLE_BYTES 64
int fence_tp_handle(fence_model* m, void* out, int cap);
int fence_tp_connect(fence_model* m, const void* handles, int n_ranks);

/* No counterpart in the reference: the batched prefill's tensor-core GEMM on its own (tcgen05, fp32
 * accumulators in tensor memory): C[P][N] = A[P][K] . B[N][K]^T for fp16 row-major A and B
 * (16-byte aligned), fp32 row-major C, K % 64 == 0; asynchronous on the stream. */
int fence_gemm_f16(const uint16_t* A, const uint16_t* B, float* C, int P, int N, int K,
                   fence_stream_t stream);

/* Times n_steps device-resident decode steps with CUDA events on the engine's stream; *ms = total. */
int fence_time_decode(fence_model* m, int token, int pos, int n_steps, float* ms);
/* No counterpart in the reference (diagnostic). Runs one token step (token at pos) of a model
 * loaded with the persistent step kernel, eagerly, with phase tracing on, and copies the trace to
 * host_out: [n_ctas][n_phases][8] per CTA: globaltimer nanoseconds at the phase start (after the
 * grid-counter wait), when x is quantised (attention: when the CTA's first unit is done), when the
 * last weight stage is consumed, and at the end (before the CTA counts itself done); SM clock
 * cycles the consumers waited for filled ring slots, cycles the producer waited for free slots;
 * two reserved words. cap = capacity of host_out in entries (>= n_ctas * n_phases * 8).
 * Allocates a device buffer for the trace. */
int fence_step_trace(fence_model* m, int token, int pos, unsigned long long* host_out, int cap,
                     int* n_phases, int* n_ctas);

/* =====================================================================================
 * 3. Synthetic GGUF writer (seeded, counter-based, byte-reproducible).
 * ===================================================================================== */
typedef struct fence_synth_spec {
    const char* arch;            /* general.architecture, e.g. "qwen3" or "llama"            */
    int   n_layers, embed_dim, ff_dim, n_heads, n_kv_heads, head_dim, vocab_size;
    float rope_freq_base, rms_eps;
    int   linear_type;           /* 14 = Q6_K, 8 = Q8_0                                     */
    int   embd_type;             /* 8 = Q8_0                                                */
    int   qk_norm;               /* write attn_q_norm / attn_k_norm                         */
    int   n_experts, n_experts_used; /* 0 = dense FFN                                       */
    int   write_tokenizer;       /* write tokenizer.ggml.tokens (vocab_size strings)        */
    int   gguf_version;          /* 2 or 3                                                  */
    uint32_t alignment;          /* general.alignment                                       */
    uint64_t seed;
    float q6k_d, q8_d;           /* fp16 super-block scales (defaults 1.5e-5 / 1.6e-4)      */
    float norm_value;            /* value of every norm weight (default 1.0)                */
} fence_synth_spec;

void fence_synth_spec_default(fence_synth_spec* s);
/* Writes the model to `path` with n_threads workers. Returns 0 or a FENCE_E_* code. */
int fence_synth_write_gguf(const char* path, const fence_synth_spec* spec, int n_threads);
/* Fills a host buffer with n seeded blocks of the given type, the same generator the writer uses
 * for tensor number `stream_id`. */
int fence_synth_fill_blocks(void* dst, int ggml_type, size_t n_blocks, uint64_t seed,
                            uint64_t stream_id, float d);

/* =====================================================================================
 * 4. Tokenizer and chat prompts — the reference's Tokenizer (src/tokenizer/tokenizer.h:15-129,
 *    tokenizer.cpp:165-627) and detect_chat_format (src/model/chat_template.h:36-60), host only.
 *    Byte-level BPE read from the GGUF (tokenizer.ggml.tokens / merges / bos / eos,
 *    tokenizer.chat_template, general.architecture) with the reference's results: merges over the
 *    whole text, lowest rank then leftmost pair; greedy longest match when the file has no merges;
 *    characters missing from the vocabulary dropped; '?' for bytes that cannot be decoded.
 *    Buffers too small for a result return FENCE_E_ARG with the size needed in *n_out / *len_out.
 * ===================================================================================== */
typedef struct fence_tokenizer fence_tokenizer;

/* ChatFormat (chat_template.h:25-31), same order */
#define FENCE_CHAT_CHATML  0
#define FENCE_CHAT_LLAMA3  1
#define FENCE_CHAT_LLAMA2  2
#define FENCE_CHAT_MISTRAL 3
#define FENCE_CHAT_RAW     4

/* Tokenizer::load_from_gguf (tokenizer.cpp:165-248). NULL on failure (fence_last_error). */
fence_tokenizer* fence_tokenizer_load(const char* gguf_path);
void fence_tokenizer_free(fence_tokenizer* t);
/* chat_format(), bos_id(), eos_id(), vocab_size() (tokenizer.h:64-76); any pointer may be NULL. */
int fence_tokenizer_info(const fence_tokenizer* t, int* chat_format, int* bos_id, int* eos_id,
                         int* vocab_size);
/* Tokenizer::encode (tokenizer.cpp:265-325): len bytes of UTF-8 text -> *n_out ids in out[cap]. */
int fence_tokenize(const fence_tokenizer* t, const char* text, size_t len, int* out, int cap,
                   int* n_out);
/* Tokenizer::decode of n ids, concatenated (tokenizer.cpp:403-414): *len_out bytes plus a NUL. */
int fence_detokenize(const fence_tokenizer* t, const int* ids, int n, char* out, size_t cap,
                     size_t* len_out);
/* Tokenizer::format_chat (tokenizer.cpp:416-428): sequence start, system turn (skipped when
 * system_prompt is NULL or empty), user turn, assistant header. */
int fence_format_chat(fence_tokenizer* t, const char* system_prompt, const char* user_message,
                      int* out, int cap, int* n_out);
/* The multi-turn helpers begin_sequence / append_system_turn / append_user_turn /
 * append_assistant_header / append_turn_end (tokenizer.cpp:478-627): appends the turn's ids to
 * tokens[0 .. *n_inout) (capacity cap) and updates *n_inout. content is used by SYSTEM and USER.
 * As in the reference, a LLaMA-2 / Mistral system prompt is held in the tokenizer until the first
 * user turn, so a tokenizer carries one conversation at a time (not thread safe). When the ids do
 * not fit cap, the call returns FENCE_E_ARG with the total needed in *n_inout and leaves tokens and
 * the conversation state as they were: call again with a larger buffer and the original count. */
#define FENCE_TURN_BEGIN     0
#define FENCE_TURN_SYSTEM    1
#define FENCE_TURN_USER      2
#define FENCE_TURN_ASSISTANT 3
#define FENCE_TURN_END       4
int fence_chat_append(fence_tokenizer* t, int turn, const char* content, int* tokens, int cap,
                      int* n_inout);

#ifdef __cplusplus
} /* extern "C" */

/* ---- C++: the reference's launcher names, argument lists and default stream ---- */
#if defined(__CUDA_FP16_TYPES_EXIST__) && defined(CUDART_VERSION)
inline void gemv_q6k(const block_q6_K* W, const __half* x, float* y, int M, int K,
                     cudaStream_t s = 0) { fence_gemv_q6k(W, (const uint16_t*)x, y, M, K, s); }
inline void gemv_q6k_bias(const block_q6_K* W, const __half* x, const float* b, float* y, int M,
                          int K, cudaStream_t s = 0) {
    fence_gemv_q6k_bias(W, (const uint16_t*)x, b, y, M, K, s); }
inline void gemv_q8_0(const block_q8_0* W, const float* x, float* y, int M, int K,
                      cudaStream_t s = 0) { fence_gemv_q8_0(W, x, y, M, K, s); }
inline void embed_q8_0(float* o, const block_q8_0* w, int tok, int dim, cudaStream_t s = 0) {
    fence_embed_q8_0(o, w, tok, dim, s); }
inline void rms_norm(float* o, const float* x, const float* w, int n, float eps,
                     cudaStream_t s = 0) { fence_rms_norm(o, x, w, n, eps, s); }
inline void rms_norm_inplace(float* x, const float* w, int n, float eps, cudaStream_t s = 0) {
    fence_rms_norm_inplace(x, w, n, eps, s); }
inline void rms_norm_per_head(float* x, const float* w, int nh, int hd, float eps,
                              cudaStream_t s = 0) { fence_rms_norm_per_head(x, w, nh, hd, eps, s); }
inline void apply_rope(float* q, float* k, int hd, int nq, int nkv, int pos, float base,
                       cudaStream_t s = 0) { fence_apply_rope(q, k, hd, nq, nkv, pos, base, s); }
inline void silu_elementwise_mul(float* o, const float* g, const float* u, int n,
                                 cudaStream_t s = 0) { fence_silu_elementwise_mul(o, g, u, n, s); }
inline void residual_add(float* x, const float* r, int n, cudaStream_t s = 0) {
    fence_residual_add(x, r, n, s); }
inline void softmax(float* x, int n, cudaStream_t s = 0) { fence_softmax(x, n, s); }
inline void f32_to_f16(__half* o, const float* i, int n, cudaStream_t s = 0) {
    fence_f32_to_f16((uint16_t*)o, i, n, s); }
inline void float_to_half(__half* o, const float* i, int n, cudaStream_t s = 0) {
    fence_float_to_half((uint16_t*)o, i, n, s); }
inline void half_to_float(float* o, const __half* i, int n, cudaStream_t s = 0) {
    fence_half_to_float(o, (const uint16_t*)i, n, s); }
inline void store_kv(__half* kc, __half* vc, const float* k, const float* v, int pos, int kv_dim,
                     int max_ctx, cudaStream_t s = 0) {
    fence_store_kv((uint16_t*)kc, (uint16_t*)vc, k, v, pos, kv_dim, max_ctx, s); }
inline void gqa_attention(float* o, const float* q, const __half* kc, const __half* vc, int hd,
                          int nq, int nkv, int seq_len, int max_ctx, float* score_buf,
                          cudaStream_t s = 0) {
    fence_gqa_attention(o, q, (const uint16_t*)kc, (const uint16_t*)vc, hd, nq, nkv, seq_len,
                        max_ctx, score_buf, s); }
inline void argmax(const float* x, int* r, int n, cudaStream_t s = 0) { fence_argmax(x, r, n, s); }
#endif /* fp16 + runtime headers */
#endif /* __cplusplus */

#endif /* FENCE_B200_H */
