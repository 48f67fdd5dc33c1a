"""fence_b200 — Python view of libfence_b200.so, the B200 (sm_100a) decode engine for Fence's GGUF
token loop.

The product is the C-ABI shared library built next to this file (``make``); this module only binds
it with ctypes for the test suite and the benchmark. Everything the library computes runs in its
own CUDA kernels: if the library is missing, importing this module raises instead of falling back.

Device buffers are passed as raw addresses (e.g. ``torch.Tensor.data_ptr()``).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfence_b200.so")

FENCE_LAUNCH_PDL = 1
FENCE_KV_F16 = 0
FENCE_KV_BF16 = 1
GGML_Q8_0 = 8
GGML_Q6_K = 14

_c_float_p = ctypes.POINTER(ctypes.c_float)
_c_int_p = ctypes.POINTER(ctypes.c_int)
_vp = ctypes.c_void_p


class FenceError(RuntimeError):
    """A fence_* call returned a non-zero status."""


FENCE_TP_HANDLE_BYTES = 64


class Config(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int), ("embed_dim", ctypes.c_int), ("ff_dim", ctypes.c_int),
        ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("vocab_size", ctypes.c_int), ("max_ctx", ctypes.c_int),
        ("rope_freq_base", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("top_k", ctypes.c_int),
        ("repetition_penalty", ctypes.c_float), ("min_p", ctypes.c_float), ("dynamic_temp", ctypes.c_int),
        ("linear_type", ctypes.c_int), ("embd_type", ctypes.c_int), ("has_qk_norm", ctypes.c_int),
        ("n_experts", ctypes.c_int), ("n_experts_used", ctypes.c_int), ("kv_dtype", ctypes.c_int),
        ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int), ("weight_bytes", ctypes.c_size_t),
    ]


class LoadOpts(ctypes.Structure):
    _fields_ = [
        ("max_ctx", ctypes.c_int), ("kv_dtype", ctypes.c_int), ("device", ctypes.c_int),
        ("use_graph", ctypes.c_int), ("verbose", ctypes.c_int), ("tp_rank", ctypes.c_int),
        ("tp_size", ctypes.c_int), ("step_kernel", ctypes.c_int), ("wait_test_phase", ctypes.c_int),
        ("moe_ep", ctypes.c_int), ("prefill", ctypes.c_int),
    ]


class SynthSpec(ctypes.Structure):
    _fields_ = [
        ("arch", ctypes.c_char_p),
        ("n_layers", ctypes.c_int), ("embed_dim", ctypes.c_int), ("ff_dim", ctypes.c_int),
        ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("vocab_size", ctypes.c_int), ("rope_freq_base", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("linear_type", ctypes.c_int), ("embd_type", ctypes.c_int), ("qk_norm", ctypes.c_int),
        ("n_experts", ctypes.c_int), ("n_experts_used", ctypes.c_int), ("write_tokenizer", ctypes.c_int),
        ("gguf_version", ctypes.c_int), ("alignment", ctypes.c_uint32), ("seed", ctypes.c_uint64),
        ("q6k_d", ctypes.c_float), ("q8_d", ctypes.c_float), ("norm_value", ctypes.c_float),
    ]


# (name, restype, argtypes) of every symbol declared in include/fence_b200.h
SIGNATURES = [
    ("fence_last_error", ctypes.c_char_p, []),
    ("fence_device_error", ctypes.c_int, []),
    ("fence_set_launch_flags", ctypes.c_int, [ctypes.c_int]),
    ("fence_gemv_q6k", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("fence_gemv_q6k_bias", ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("fence_gemv_q8_0", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("fence_embed_q8_0", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("fence_rms_norm", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_float, _vp]),
    ("fence_rms_norm_inplace", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_float, _vp]),
    ("fence_rms_norm_per_head", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp]),
    ("fence_apply_rope", ctypes.c_int,
     [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp]),
    ("fence_silu_elementwise_mul", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, _vp]),
    ("fence_residual_add", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    ("fence_softmax", ctypes.c_int, [_vp, ctypes.c_int, _vp]),
    ("fence_f32_to_f16", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    ("fence_float_to_half", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    ("fence_half_to_float", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    ("fence_store_kv", ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    ("fence_gqa_attention", ctypes.c_int,
     [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp]),
    ("fence_argmax", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    ("fence_step_trace", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp]),
    ("fence_gqa_attention_static", ctypes.c_int,
     [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    ("fence_load_opts_default", None, [ctypes.POINTER(LoadOpts)]),
    ("fence_model_load", _vp, [ctypes.c_char_p, ctypes.POINTER(LoadOpts)]),
    ("fence_model_free", None, [_vp]),
    ("fence_model_config", ctypes.c_int, [_vp, ctypes.POINTER(Config)]),
    ("fence_set_sampling", ctypes.c_int, [_vp, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_float]),
    ("fence_forward", _vp, [_vp, ctypes.c_int, ctypes.c_int]),
    ("fence_sample_greedy", ctypes.c_int, [_vp, _vp]),
    ("fence_sample_nucleus", ctypes.c_int, [_vp, _vp, _c_int_p, ctypes.c_int]),
    ("fence_set_seed", ctypes.c_int, [_vp, ctypes.c_uint64]),
    ("fence_generate", ctypes.c_int,
     [_vp, _c_int_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _c_int_p, ctypes.c_int, _c_int_p]),
    ("fence_decode_greedy", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _c_int_p]),
    ("fence_copy_logits", ctypes.c_int, [_vp, _c_float_p]),
    ("fence_time_decode", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _c_float_p]),
    ("fence_tp_handle", ctypes.c_int, [_vp, _vp, ctypes.c_int]),
    ("fence_sample_scratch_bytes", ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ("fence_sample_nucleus_device", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int]),
    ("fence_sample_nucleus_dev", ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                                ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                ctypes.c_double, _vp, ctypes.c_size_t, _vp, _vp]),
    ("fence_tp_connect", ctypes.c_int, [_vp, _vp, ctypes.c_int]),
    ("fence_synth_spec_default", None, [ctypes.POINTER(SynthSpec)]),
    ("fence_synth_write_gguf", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(SynthSpec), ctypes.c_int]),
    ("fence_synth_fill_blocks", ctypes.c_int,
     [_vp, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]),
    ("fence_prefill", _vp, [_vp, _c_int_p, ctypes.c_int, ctypes.c_int]),
    ("fence_gemm_f16", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    ("fence_tokenizer_load", _vp, [ctypes.c_char_p]),
    ("fence_tokenizer_free", None, [_vp]),
    ("fence_tokenizer_info", ctypes.c_int, [_vp, _c_int_p, _c_int_p, _c_int_p, _c_int_p]),
    ("fence_tokenize", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_size_t, _c_int_p, ctypes.c_int, _c_int_p]),
    ("fence_detokenize", ctypes.c_int, [_vp, _c_int_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t,
                                        ctypes.POINTER(ctypes.c_size_t)]),
    ("fence_format_chat", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_char_p, _c_int_p, ctypes.c_int, _c_int_p]),
    ("fence_chat_append", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_char_p, _c_int_p, ctypes.c_int, _c_int_p]),
]

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libfence_b200.so (once) and declares every exported signature."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `make` in {HERE}")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().fence_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str = "fence call") -> None:
    if rc != 0:
        raise FenceError(f"{what} failed ({rc}): {last_error()}")


def call(name: str, *args) -> None:
    """Calls a status-returning entry point and raises FenceError on a non-zero status."""
    check(getattr(lib(), name)(*args), name)


# ------------------------------------------------------------------ synthetic models
CONFIGS = {
    # config 1: Qwen3-4B shape, Q6_K linears, Q8_0 embedding
    "qwen3-4b": dict(arch=b"qwen3", n_layers=36, embed_dim=2560, ff_dim=9728, n_heads=32, n_kv_heads=8,
                     head_dim=128, vocab_size=151936, rope_freq_base=1e6, rms_eps=1e-6,
                     linear_type=GGML_Q6_K, qk_norm=1),
    # config 2: Llama-3.1-8B shape, all Q8_0, no q/k-norm
    "llama3-8b-q8": dict(arch=b"llama", n_layers=32, embed_dim=4096, ff_dim=14336, n_heads=32, n_kv_heads=8,
                         head_dim=128, vocab_size=128256, rope_freq_base=5e5, rms_eps=1e-5,
                         linear_type=GGML_Q8_0, qk_norm=0),
    # config 3: Qwen3-14B shape, Q6_K linears
    "qwen3-14b": dict(arch=b"qwen3", n_layers=40, embed_dim=5120, ff_dim=17408, n_heads=40, n_kv_heads=8,
                      head_dim=128, vocab_size=151936, rope_freq_base=1e6, rms_eps=1e-6,
                      linear_type=GGML_Q6_K, qk_norm=1),
    # small shapes for fast parity runs
    "tiny-q6k": dict(arch=b"qwen3", n_layers=2, embed_dim=512, ff_dim=1024, n_heads=8, n_kv_heads=2,
                     head_dim=128, vocab_size=2048, rope_freq_base=1e6, rms_eps=1e-6,
                     linear_type=GGML_Q6_K, qk_norm=1),
    "tiny-q8": dict(arch=b"llama", n_layers=2, embed_dim=512, ff_dim=1024, n_heads=8, n_kv_heads=2,
                    head_dim=128, vocab_size=2048, rope_freq_base=5e5, rms_eps=1e-5,
                    linear_type=GGML_Q8_0, qk_norm=0),
    # wide test models: K = 4096 rows (64 items) for QKV, O, gate/up and the LM head
    "wide-q6k": dict(arch=b"qwen3", n_layers=2, embed_dim=4096, ff_dim=1024, n_heads=32, n_kv_heads=8,
                     head_dim=128, vocab_size=2048, rope_freq_base=1e6, rms_eps=1e-6,
                     linear_type=GGML_Q6_K, qk_norm=1),
    "wide-q8": dict(arch=b"llama", n_layers=2, embed_dim=4096, ff_dim=1024, n_heads=32, n_kv_heads=8,
                    head_dim=128, vocab_size=2048, rope_freq_base=5e5, rms_eps=1e-5,
                    linear_type=GGML_Q8_0, qk_norm=0),
    # config 4: Mixtral-8x7B shape, sparse MoE (8 experts, top-2), Q6_K linears, fp32 router
    "mixtral-8x7b": dict(arch=b"llama", n_layers=32, embed_dim=4096, ff_dim=14336, n_heads=32, n_kv_heads=8,
                         head_dim=128, vocab_size=32000, rope_freq_base=1e6, rms_eps=1e-5,
                         linear_type=GGML_Q6_K, qk_norm=0, n_experts=8, n_experts_used=2),
    # small sparse-MoE shapes for parity runs (FFN rows split 2/4/8 ways in whole 64-input items;
    # tiny-moe-q8's 8 experts split 2/4/8 ways for expert parallelism)
    "tiny-moe": dict(arch=b"llama", n_layers=2, embed_dim=512, ff_dim=1024, n_heads=8, n_kv_heads=8,
                     head_dim=128, vocab_size=2048, rope_freq_base=1e6, rms_eps=1e-5,
                     linear_type=GGML_Q6_K, qk_norm=0, n_experts=4, n_experts_used=2),
    "tiny-moe-q8": dict(arch=b"llama", n_layers=2, embed_dim=512, ff_dim=512, n_heads=8, n_kv_heads=8,
                        head_dim=128, vocab_size=2048, rope_freq_base=1e6, rms_eps=1e-5,
                        linear_type=GGML_Q8_0, qk_norm=0, n_experts=8, n_experts_used=2),
}


def synth_spec(**kw) -> SynthSpec:
    s = SynthSpec()
    lib().fence_synth_spec_default(ctypes.byref(s))
    for k, v in kw.items():
        setattr(s, k, v)
    return s


def synth_write(path: str, config: str | None = None, threads: int = 0, **kw) -> None:
    """Writes a seeded synthetic GGUF model (one of CONFIGS, overridden by keyword fields)."""
    fields = dict(CONFIGS[config]) if config else {}
    fields.update(kw)
    spec = synth_spec(**fields)
    check(lib().fence_synth_write_gguf(path.encode(), ctypes.byref(spec), threads), "synth_write_gguf")


def synth_blocks(ggml_type: int, n_blocks: int, seed: int, stream: int = 0, d: float | None = None) -> bytes:
    if d is None:
        d = 1.5e-5 if ggml_type == GGML_Q6_K else 1.6e-4
    size = n_blocks * (210 if ggml_type == GGML_Q6_K else 34)
    buf = ctypes.create_string_buffer(size)
    check(lib().fence_synth_fill_blocks(buf, ggml_type, n_blocks, seed, stream, d), "synth_fill_blocks")
    return buf.raw


# ------------------------------------------------------------------ engine
class Model:
    """The reference's Qwen3Model API over the engine handle."""

    def __init__(self, path: str, max_ctx: int = 4096, kv_dtype: int = FENCE_KV_F16, device: int = 0,
                 use_graph: bool = True, verbose: bool = False, step_kernel: bool = True,
                 tp_rank: int = 0, tp_size: int = 1, wait_test_phase: int = -1, moe_ep: bool = False,
                 prefill: bool = True):
        L = lib()
        o = LoadOpts()
        L.fence_load_opts_default(ctypes.byref(o))
        o.max_ctx, o.kv_dtype, o.device, o.use_graph, o.verbose = max_ctx, kv_dtype, device, int(use_graph), int(verbose)
        o.step_kernel = int(step_kernel)
        o.tp_rank, o.tp_size = tp_rank, tp_size
        o.wait_test_phase = wait_test_phase  # test only: a step-kernel phase whose counter wait runs out
        o.moe_ep = int(moe_ep)  # sparse MoE over tp_size ranks: whole experts per rank instead of slices
        o.prefill = int(prefill)  # keep the repacked weights for the batched (tensor-core) prefill
        h = L.fence_model_load(path.encode(), ctypes.byref(o))
        if not h:
            raise FenceError(f"model load failed: {last_error()}")
        self._h = h
        c = Config()
        check(L.fence_model_config(h, ctypes.byref(c)), "model_config")
        self.config = c

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().fence_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, token: int, pos: int) -> int:
        p = lib().fence_forward(self._h, token, pos)
        if not p:
            raise FenceError(f"forward failed: {last_error()}")
        return p

    def prefill(self, tokens, pos0: int = 0) -> int:
        """fence_prefill: tokens at positions pos0.. (batched where the model allows it); returns the
        device address of the last token's logits."""
        ids = list(tokens)
        arr = (ctypes.c_int * len(ids))(*ids)
        p = lib().fence_prefill(self._h, arr, len(ids), pos0)
        if not p:
            raise FenceError(f"prefill failed: {last_error()}")
        return p

    def vocab_shard(self):
        """(first row, rows) of this rank's LM-head vocabulary shard ((0, vocab) without TP)."""
        V, n, r = self.config.vocab_size, max(1, self.config.tp_size), self.config.tp_rank
        per = (V + n - 1) // n
        return r * per, min(V, (r + 1) * per) - r * per

    def tp_handle(self) -> bytes:
        """This rank's exchange-buffer handle, to give every other rank (tensor parallel)."""
        buf = ctypes.create_string_buffer(FENCE_TP_HANDLE_BYTES)
        check(lib().fence_tp_handle(self._h, buf, FENCE_TP_HANDLE_BYTES), "tp_handle")
        return buf.raw

    def tp_connect(self, handles) -> None:
        """Maps every rank's exchange buffer (handles in rank order) and builds the step."""
        blob = b"".join(handles)
        check(lib().fence_tp_connect(self._h, blob, len(handles)), "tp_connect")

    def logits(self):
        import numpy as np
        out = np.empty(self.vocab_shard()[1], dtype=np.float32)
        check(lib().fence_copy_logits(self._h, out.ctypes.data_as(_c_float_p)), "copy_logits")
        return out

    def sample_greedy(self, d_logits: int) -> int:
        r = lib().fence_sample_greedy(self._h, d_logits)
        if r < 0:
            raise FenceError(last_error())
        return r

    def sample_nucleus(self, d_logits: int, history) -> int:
        arr = (ctypes.c_int * len(history))(*history)
        r = lib().fence_sample_nucleus(self._h, d_logits, arr, len(history))
        if r < 0:
            raise FenceError(last_error())
        return r

    def sample_nucleus_device(self, d_logits: int, history) -> int:
        """sample_nucleus with the sampling steps on the device (only the id comes back)."""
        arr = (ctypes.c_int * max(1, len(history)))(*history)
        r = lib().fence_sample_nucleus_device(self._h, d_logits, arr, len(history))
        if r < 0:
            raise FenceError(last_error())
        return r

    def set_sampling(self, temperature: float, top_p: float, top_k: int, rep_penalty: float) -> None:
        check(lib().fence_set_sampling(self._h, temperature, top_p, top_k, rep_penalty), "set_sampling")

    def set_seed(self, seed: int) -> None:
        check(lib().fence_set_seed(self._h, seed), "set_seed")

    def generate(self, prompt, max_new: int, eos_id: int = -1):
        n = len(prompt)
        arr = (ctypes.c_int * n)(*prompt)
        cap = n + max_new + 1
        out = (ctypes.c_int * cap)()
        n_out = ctypes.c_int(0)
        check(lib().fence_generate(self._h, arr, n, max_new, eos_id, out, cap, ctypes.byref(n_out)), "generate")
        return list(out[: n_out.value])

    def decode_greedy(self, token: int, pos: int, n_steps: int):
        out = (ctypes.c_int * max(n_steps, 1))()
        check(lib().fence_decode_greedy(self._h, token, pos, n_steps, out), "decode_greedy")
        return list(out[:n_steps])

    def time_decode(self, token: int, pos: int, n_steps: int) -> float:
        ms = ctypes.c_float(0)
        check(lib().fence_time_decode(self._h, token, pos, n_steps, ctypes.byref(ms)), "time_decode")
        return ms.value

    def step_trace(self, token: int, pos: int):
        """One traced token step (persistent step kernel): array [n_ctas, n_phases, 8]: globaltimer ns
        at phase start, x ready, stages done, end; consumer and producer ring-wait cycles."""
        import numpy as np
        nph, nct = ctypes.c_int(0), ctypes.c_int(0)
        cap = 4096 * 1024
        buf = np.zeros(cap, np.uint64)
        check(lib().fence_step_trace(self._h, token, pos, buf.ctypes.data, cap, ctypes.byref(nph), ctypes.byref(nct)),
              "step_trace")
        return buf[: nct.value * nph.value * 8].reshape(nct.value, nph.value, 8)


# ------------------------------------------------------------------ tokenizer and chat prompts
CHAT_FORMATS = ("ChatML", "LLaMA-3", "LLaMA-2", "Mistral", "Raw")  # FENCE_CHAT_* order
TURN_BEGIN, TURN_SYSTEM, TURN_USER, TURN_ASSISTANT, TURN_END = range(5)


def _b(text) -> bytes:
    return text if isinstance(text, bytes) else text.encode("utf-8")


class Tokenizer:
    """The reference's Tokenizer API (src/tokenizer/tokenizer.h) over fence_tokenizer_*."""

    def __init__(self, gguf_path: str):
        h = lib().fence_tokenizer_load(gguf_path.encode())
        if not h:
            raise FenceError(f"tokenizer load failed: {last_error()}")
        self._h = h
        f, b, e, v = (ctypes.c_int() for _ in range(4))
        check(lib().fence_tokenizer_info(h, ctypes.byref(f), ctypes.byref(b), ctypes.byref(e), ctypes.byref(v)))
        self.chat_format, self.bos_id, self.eos_id, self.vocab_size = f.value, b.value, e.value, v.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().fence_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _ids_call(fn, *args, cap=256):
        n = ctypes.c_int(0)
        while True:
            buf = (ctypes.c_int * max(cap, 1))()
            rc = fn(*args, buf, cap, ctypes.byref(n))
            if rc == 0:
                return list(buf[:n.value])
            if n.value <= cap:
                check(rc)
            cap = n.value

    def encode(self, text) -> list:
        t = _b(text)
        return self._ids_call(lib().fence_tokenize, self._h, t, len(t), cap=len(t) + 8)

    def decode(self, ids) -> bytes:
        ids = list(ids)
        arr = (ctypes.c_int * max(len(ids), 1))(*ids)
        need = ctypes.c_size_t(0)
        cap = 64 + 8 * len(ids)
        while True:
            buf = ctypes.create_string_buffer(cap)
            rc = lib().fence_detokenize(self._h, arr, len(ids), buf, cap, ctypes.byref(need))
            if rc == 0:
                return buf.raw[:need.value]
            if need.value + 1 <= cap:
                check(rc)
            cap = need.value + 1

    def format_chat(self, system_prompt, user_message) -> list:
        return self._ids_call(lib().fence_format_chat, self._h, _b(system_prompt), _b(user_message), cap=1024)

    def append(self, tokens: list, turn: int, content=None) -> list:
        """One multi-turn helper (TURN_*) appended to tokens; returns the new list."""
        c = None if content is None else _b(content)
        cap = len(tokens) + 64 + (4 * len(c) if c else 0)
        while True:  # a buffer too small leaves the conversation unchanged and reports the size needed
            buf = (ctypes.c_int * cap)(*tokens)
            n = ctypes.c_int(len(tokens))
            rc = lib().fence_chat_append(self._h, turn, c, buf, cap, ctypes.byref(n))
            if rc == 0:
                return list(buf[:n.value])
            if n.value <= cap:
                check(rc, "chat_append")
            cap = n.value
