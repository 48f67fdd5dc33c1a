"""ctypes view of the checker libraries under oracle/ — TEST INFRASTRUCTURE ONLY.

* liboracle.so       : the CPU restatement of the reference's token loop (fence_oracle.c)
* _ref/libref_cpu.so : the reference's own fp64 host oracle and golden blocks, compiled from the
                       reference tree (tests/test_gemv_q6k.cu, tests/test_q6k_dot.cu)
* _ref/ref_model     : the reference's CUDA forward rebuilt for sm_100a (GPU only)
* _ref/ref_model_tsw : the same forward, restated with a per-linear type switch to the reference's
                       own gemv_q8_0 for Q8_0 linears (all-Q8_0 config 2; GPU only)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_CPU_SO = os.path.join(HERE, "_ref", "libref_cpu.so")
REF_MODEL = os.path.join(HERE, "_ref", "ref_model")
# oracle extension: the reference's forward restated with a per-linear type switch to its own
# gemv_q8_0 (all-Q8_0 models, which the reference's loader cannot run); GPU only
REF_MODEL_TSW = os.path.join(HERE, "_ref", "ref_model_tsw")

_vp = ctypes.c_void_p
_o = None
_r = None


def oracle() -> ctypes.CDLL:
    global _o
    if _o is None:
        L = ctypes.CDLL(ORACLE_SO)
        sig = {
            "oracle_h2f": (ctypes.c_float, [ctypes.c_uint16]),
            "oracle_f2h": (ctypes.c_uint16, [ctypes.c_float]),
            "oracle_bf2f": (ctypes.c_float, [ctypes.c_uint16]),
            "oracle_f2bf": (ctypes.c_uint16, [ctypes.c_float]),
            "oracle_q6k_dequant": (None, [_vp, _vp]),
            "oracle_q6k_dot_block": (ctypes.c_double, [_vp, _vp]),
            "oracle_gemv_q6k": (None, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
            "oracle_gemv_q8_0": (None, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
            "oracle_embed_q8_0": (None, [_vp, _vp, ctypes.c_int, ctypes.c_int]),
            "oracle_rms_norm": (None, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_float]),
            "oracle_rms_norm_per_head": (None, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float]),
            "oracle_rope": (None, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]),
            "oracle_silu_mul": (None, [_vp, _vp, _vp, ctypes.c_int]),
            "oracle_softmax": (None, [_vp, ctypes.c_int]),
            "oracle_attention": (None, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_long, ctypes.c_long,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
            "oracle_argmax": (ctypes.c_int, [_vp, ctypes.c_int]),
            "oracle_sample_nucleus": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_float,
                                                     ctypes.c_float, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                                     ctypes.c_int, ctypes.c_double, _vp, _vp]),
            "oracle_model_open": (_vp, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
            "oracle_model_close": (None, [_vp]),
            "oracle_model_dims": (None, [_vp, _vp]),
            "oracle_forward": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
            "oracle_last_hidden": (None, [_vp, _vp]),
            "oracle_model_fill_kv": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_uint64]),
            "oracle_model_moe": (None, [_vp, _vp, _vp]),
            "oracle_last_route": (ctypes.c_float, [_vp, _vp]),
            "oracle_moe_ffn_apply": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp]),
        }
        for n, (res, args) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = res, args
        _o = L
    return _o


def ref_cpu() -> ctypes.CDLL | None:
    """The reference's compiled host oracle, or None when oracle/_ref was not built."""
    global _r
    if _r is None:
        if not os.path.exists(REF_CPU_SO):
            return None
        L = ctypes.CDLL(REF_CPU_SO)
        L.ref_cpu_gemv_q6k.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
        L.ref_cpu_gemv_q6k.restype = None
        L.ref_cpu_q6k_dot_block.argtypes = [_vp, _vp]
        L.ref_cpu_q6k_dot_block.restype = ctypes.c_double
        L.ref_set_q6.argtypes = [_vp, ctypes.c_int, ctypes.c_int]
        L.ref_set_q6.restype = None
        L.ref_dot_case.argtypes = [ctypes.c_int, _vp, _vp, ctypes.POINTER(ctypes.c_double)]
        L.ref_dot_case.restype = ctypes.c_int
        L.ref_dot_case_name.argtypes = [ctypes.c_int]
        L.ref_dot_case_name.restype = ctypes.c_char_p
        _r = L
    return _r


SYNTH_SO = os.path.join(HERE, "libsynth.so")
_s = None


REF_TOK = os.path.join(HERE, "_ref", "libref_tok.so")
_rt = None


def ref_tok() -> ctypes.CDLL | None:
    """The reference's own Tokenizer (src/tokenizer/tokenizer.cpp) behind ref_tok_harness.cpp, or
    None when it was not built (no reference tree when `make` ran)."""
    global _rt
    if _rt is None and os.path.exists(REF_TOK):
        L = ctypes.CDLL(REF_TOK)
        L.ref_tok_load.restype, L.ref_tok_load.argtypes = _vp, [ctypes.c_char_p]
        L.ref_tok_free.argtypes = [_vp]
        L.ref_tok_info.argtypes = [_vp] + [ctypes.POINTER(ctypes.c_int)] * 4
        L.ref_tok_encode.restype = ctypes.c_int
        L.ref_tok_encode.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t, _vp, ctypes.c_int]
        L.ref_tok_decode.restype = ctypes.c_size_t
        L.ref_tok_decode.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        L.ref_tok_format_chat.restype = ctypes.c_int
        L.ref_tok_format_chat.argtypes = [_vp, ctypes.c_char_p, ctypes.c_char_p, _vp, ctypes.c_int]
        L.ref_tok_append.restype = ctypes.c_int
        L.ref_tok_append.argtypes = [_vp, ctypes.c_int, ctypes.c_char_p, _vp, ctypes.c_int, ctypes.c_int]
        L.ref_tok_last.restype = ctypes.c_int
        L.ref_tok_last.argtypes = [_vp, ctypes.c_int]
        _rt = L
    return _rt


class RefTokenizer:
    """Python face of the reference tokenizer harness (same methods as fence_b200.Tokenizer)."""

    def __init__(self, path: str):
        L = ref_tok()
        self._L = L
        self._h = L.ref_tok_load(path.encode())
        if not self._h:
            raise RuntimeError(f"reference tokenizer could not load {path}")
        v = [ctypes.c_int() for _ in range(4)]
        L.ref_tok_info(self._h, *[ctypes.byref(x) for x in v])
        self.chat_format, self.bos_id, self.eos_id, self.vocab_size = (x.value for x in v)

    def close(self):
        if self._h:
            self._L.ref_tok_free(self._h)
            self._h = None

    def encode(self, text) -> list:
        t = text if isinstance(text, bytes) else text.encode("utf-8")
        cap = len(t) + 8
        buf = np.zeros(cap, np.int32)
        n = self._L.ref_tok_encode(self._h, t, len(t), buf.ctypes.data, cap)
        return [int(x) for x in buf[:n]]

    def decode(self, ids) -> bytes:
        a = np.asarray(list(ids) or [0], np.int32)
        cap = 64 + 8 * len(a)
        out = ctypes.create_string_buffer(cap)
        n = self._L.ref_tok_decode(self._h, a.ctypes.data, len(list(ids)), out, cap)
        return out.raw[:n]

    def format_chat(self, system_prompt, user_message) -> list:
        buf = np.zeros(4096, np.int32)
        b = [x if isinstance(x, bytes) else x.encode("utf-8") for x in (system_prompt, user_message)]
        n = self._L.ref_tok_format_chat(self._h, b[0], b[1], buf.ctypes.data, 4096)
        if n > 4096:
            buf = np.zeros(n, np.int32)
            self._L.ref_tok_last(buf.ctypes.data, n)
        return [int(x) for x in buf[:n]]

    def append(self, tokens: list, turn: int, content=None) -> list:
        c = b"" if content is None else (content if isinstance(content, bytes) else content.encode("utf-8"))
        cap = len(tokens) + 64 + 4 * len(c)
        buf = np.zeros(cap, np.int32)
        buf[:len(tokens)] = tokens
        n = self._L.ref_tok_append(self._h, turn, c, buf.ctypes.data, len(tokens), cap)
        if n > cap:  # a held system prompt came out with this turn: the whole result, not a second call
            buf = np.zeros(n, np.int32)
            self._L.ref_tok_last(buf.ctypes.data, n)
        return [int(x) for x in buf[:n]]


def synth_write(path: str, spec_cls, fields: dict, threads: int = 0) -> None:
    """Writes a seeded synthetic GGUF through oracle/libsynth.so (the package's writer built on its
    own), byte-identical to the product library's fence_synth_write_gguf. spec_cls is the
    fence_synth_spec ctypes structure; fields override its defaults."""
    global _s
    if _s is None:
        L = ctypes.CDLL(SYNTH_SO)
        L.fence_synth_spec_default.argtypes = [ctypes.c_void_p]
        L.fence_synth_spec_default.restype = None
        L.fence_synth_write_gguf.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int]
        L.fence_synth_write_gguf.restype = ctypes.c_int
        L.oracle_synth_last_error.restype = ctypes.c_char_p
        _s = L
    spec = spec_cls()
    _s.fence_synth_spec_default(ctypes.byref(spec))
    for k, v in fields.items():
        setattr(spec, k, v)
    rc = _s.fence_synth_write_gguf(path.encode(), ctypes.byref(spec), threads)
    if rc != 0:
        raise RuntimeError(f"synth_write failed ({rc}): {_s.oracle_synth_last_error().decode()}")


def _p(a: np.ndarray):
    return a.ctypes.data_as(_vp)


# ------------------------------------------------------------------ array helpers
def f2h_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bit patterns (round to nearest even)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def gemv_q6k(W: bytes | np.ndarray, x_f16_bits: np.ndarray, M: int, K: int, threads: int = 8) -> np.ndarray:
    Wb = np.frombuffer(W, dtype=np.uint8) if isinstance(W, (bytes, bytearray)) else W
    y = np.zeros(M, dtype=np.float64)
    xb = np.ascontiguousarray(x_f16_bits, dtype=np.uint16)
    oracle().oracle_gemv_q6k(_p(Wb), _p(xb), _p(y), M, K, threads)
    return y


def gemv_q8_0(W: bytes | np.ndarray, x: np.ndarray, M: int, K: int, threads: int = 8) -> np.ndarray:
    Wb = np.frombuffer(W, dtype=np.uint8) if isinstance(W, (bytes, bytearray)) else W
    y = np.zeros(M, dtype=np.float64)
    xf = np.ascontiguousarray(x, dtype=np.float32)
    oracle().oracle_gemv_q8_0(_p(Wb), _p(xf), _p(y), M, K, threads)
    return y


def argmax(x: np.ndarray) -> int:
    xf = np.ascontiguousarray(x, dtype=np.float32)
    return int(oracle().oracle_argmax(_p(xf), xf.size))


class OracleModel:
    """CPU restatement of Qwen3Model over a GGUF file (kv_bf16 selects the cache rounding)."""

    def __init__(self, path: str, max_ctx: int = 4096, kv_bf16: bool = True, threads: int = 8):
        self._h = oracle().oracle_model_open(path.encode(), max_ctx, int(kv_bf16), threads)
        if not self._h:
            raise RuntimeError(f"oracle could not open {path}")
        d = np.zeros(10, dtype=np.int32)
        oracle().oracle_model_dims(self._h, _p(d))
        (self.n_layers, self.embed_dim, self.ff_dim, self.n_heads, self.n_kv_heads, self.head_dim,
         self.vocab_size, self.max_ctx, self.linear_type, self.qk_norm) = (int(v) for v in d)
        ne, nu = ctypes.c_int(0), ctypes.c_int(0)
        oracle().oracle_model_moe(self._h, ctypes.byref(ne), ctypes.byref(nu))
        self.n_experts, self.n_experts_used = ne.value, nu.value

    def last_route(self):
        """(experts chosen per layer at the last forward [L, n_used], smallest router-logit gap between
        the last chosen expert and the best unchosen one): MoE models only."""
        sel = np.zeros((self.n_layers, max(1, self.n_experts_used)), dtype=np.int32)
        margin = oracle().oracle_last_route(self._h, _p(sel))
        return sel, float(margin)

    def moe_ffn(self, layer: int, normed: np.ndarray):
        """The oracle's sparse-MoE FFN of one layer on a given normed input: (output [H] before the
        residual add, chosen experts [n_used])."""
        x = np.ascontiguousarray(normed, dtype=np.float32)
        out = np.empty(self.embed_dim, dtype=np.float32)
        sel = np.zeros(max(1, self.n_experts_used), dtype=np.int32)
        if oracle().oracle_moe_ffn_apply(self._h, layer, _p(x), _p(out), _p(sel)) != 0:
            raise ValueError("moe_ffn: not a MoE model or bad layer")
        return out, sel

    def fill_kv(self, n_pos: int, seed: int = 1) -> None:
        """Seeded K/V rows for positions [0, n_pos): stands in for a prefill (benchmark use)."""
        if oracle().oracle_model_fill_kv(self._h, n_pos, seed) != 0:
            raise ValueError("fill_kv: bad position count")

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab_size, dtype=np.float32)
        if oracle().oracle_forward(self._h, token, pos, _p(out)) != 0:
            raise RuntimeError("oracle forward failed")
        return out

    def close(self):
        if self._h:
            oracle().oracle_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def read_ref_dump(path: str):
    """Reads the file written by _ref/ref_model: (vocab, n_prompt, ids[steps], logits[steps, vocab] or None)."""
    raw = np.fromfile(path, dtype=np.int32, count=4)
    magic, V, n_prompt, steps = (int(v) for v in raw)
    if magic != 0x46524546:
        raise ValueError("not a reference dump")
    body = np.fromfile(path, dtype=np.uint8, offset=16)
    rec = 4 + 4 * V
    with_logits = body.size == steps * rec
    ids = np.empty(steps, dtype=np.int32)
    logits = np.empty((steps, V), dtype=np.float32) if with_logits else None
    for s in range(steps):
        if with_logits:
            chunk = body[s * rec:(s + 1) * rec]
            ids[s] = chunk[:4].view(np.int32)[0]
            logits[s] = chunk[4:].view(np.float32)
        else:
            ids[s] = body[s * 4:(s + 1) * 4].view(np.int32)[0]
    return V, n_prompt, ids, logits
