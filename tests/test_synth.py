"""Synthetic GGUF models (the benchmark's inputs): metadata typed exactly as the reference loader
demands (src/model/qwen3.cu:121-160), the reference's tensor-name contract (:180-212), seeded
byte-reproducibility, and the value distributions of the configs."""
import hashlib

import numpy as np
import pytest

from gguf_py import Reader


def _sha(path):
    return hashlib.sha256(open(path, "rb").read()).hexdigest()


def test_metadata_types_and_tensor_contract(fb, tmp_path):
    p = str(tmp_path / "t.gguf")
    fb.synth_write(p, "tiny-q6k")
    r = Reader(p)
    assert r.version == 3
    assert r.meta["general.architecture"] == "qwen3" and r.types["general.architecture"] == 8
    for k in ["block_count", "embedding_length", "feed_forward_length", "attention.head_count",
              "attention.head_count_kv", "attention.key_length"]:
        assert r.types["qwen3." + k] == 4, k  # UINT32, get_u32 is strict (gguf_parser.cpp:422-428)
    for k in ["rope.freq_base", "attention.layer_norm_rms_epsilon"]:
        assert r.types["qwen3." + k] == 6, k  # FLOAT32
    assert r.meta["qwen3.embedding_length"] == 512
    names = set(r.tensors)
    assert {"token_embd.weight", "output_norm.weight"} <= names
    for l in range(2):
        for s in ["attn_norm", "attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm", "attn_output",
                  "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"]:
            assert f"blk.{l}.{s}.weight" in names
    dims, ty, _ = r.tensors["blk.0.attn_q.weight"]
    assert dims == [512, 8 * 128] and ty == 14  # [K=input, M=output]
    dims, ty, _ = r.tensors["blk.0.ffn_down.weight"]
    assert dims == [1024, 512] and ty == 14
    dims, ty, _ = r.tensors["token_embd.weight"]
    assert dims == [512, 2048] and ty == 8
    assert all(off % 32 == 0 for _, _, off in r.tensors.values())
    assert r.data_start % 32 == 0


def test_byte_reproducible_and_seed_sensitive(fb, tmp_path):
    a, b, c = (str(tmp_path / n) for n in ("a.gguf", "b.gguf", "c.gguf"))
    fb.synth_write(a, "tiny-q8", threads=1)
    fb.synth_write(b, "tiny-q8", threads=7)
    fb.synth_write(c, "tiny-q8", seed=99)
    assert _sha(a) == _sha(b)
    assert _sha(a) != _sha(c)


def test_value_distributions(fb, orc):
    n = 20000
    q6 = np.frombuffer(fb.synth_blocks(fb.GGML_Q6_K, n, seed=3), np.uint8).reshape(n, 210)
    sc = q6[:, 192:208].view(np.int8)
    assert sc.min() >= -127 and sc.max() <= 127 and abs(float(sc.mean())) < 0.5
    assert np.all(q6[:, 208:210].copy().view(np.float16) == np.float16(1.5e-5))
    # dequantised weights: quants uniform in [-32, 31] -> std ~ d * rms(scale) * 18.5 ~ 0.02
    w = np.empty(256, np.float64)
    ws = []
    for i in range(0, 2000, 7):
        orc.oracle().oracle_q6k_dequant(q6[i].ctypes.data_as(__import__("ctypes").c_void_p),
                                        w.ctypes.data_as(__import__("ctypes").c_void_p))
        ws.append(w.copy())
    std = float(np.std(np.concatenate(ws)))
    assert 0.015 < std < 0.025
    q8 = np.frombuffer(fb.synth_blocks(fb.GGML_Q8_0, n, seed=3), np.uint8).reshape(n, 34)
    qs = q8[:, 2:].view(np.int8)
    assert qs.min() >= -127 and qs.max() <= 127
    assert np.all(q8[:, :2].copy().view(np.float16) == np.float16(1.6e-4))


def test_gguf_v2_and_alignment_64(fb, tmp_path):
    p = str(tmp_path / "v2.gguf")
    fb.synth_write(p, "tiny-q6k", gguf_version=2, alignment=64)
    r = Reader(p)
    assert r.version == 2 and r.meta["general.alignment"] == 64
    assert all(off % 64 == 0 for _, _, off in r.tensors.values())


def test_tokenizer_tokens_written(fb, tmp_path):
    p = str(tmp_path / "tok.gguf")
    fb.synth_write(p, "tiny-q8", write_tokenizer=1)
    r = Reader(p)
    toks = r.arrays["tokenizer.ggml.tokens"]
    assert len(toks) == 2048 and toks[5] == "<5>"
    assert r.meta["tokenizer.ggml.eos_token_id"] == 2048


@pytest.mark.parametrize("cfg", ["tiny-q6k", "tiny-q8"])
def test_oracle_forward_runs_on_synthetic_model(fb, orc, tmp_path, cfg):
    p = str(tmp_path / "m.gguf")
    fb.synth_write(p, cfg)
    m = orc.OracleModel(p, max_ctx=64, kv_bf16=True, threads=4)
    assert (m.n_layers, m.embed_dim, m.vocab_size) == (2, 512, 2048)
    l0 = m.forward(3, 0)
    l1 = m.forward(17, 1)
    assert np.isfinite(l0).all() and np.isfinite(l1).all()
    assert 0.05 < float(np.std(l1)) < 5.0
    m.close()
