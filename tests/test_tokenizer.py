"""The tokenizer and chat prompts (fence_tokenizer_* / fence_format_chat / fence_chat_append) against
the reference's own Tokenizer (src/tokenizer/tokenizer.cpp): committed golden results of the
reference build (tests/golden/tokenizer_golden.json, make_tokenizer_golden.py) on the seeded
vocabularies of tests/tok_vocab.py, and, where oracle/_ref/libref_tok.so is built, the reference
itself on further seeded texts. CPU only."""
import json
import os
import time

import numpy as np
import pytest

import tok_vocab as tv

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tokenizer_golden.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def vocab_files(tmp_path_factory):
    d = tmp_path_factory.mktemp("tok")
    out = {}
    for name, kw in tv.VARIANTS.items():
        p = str(d / f"{name}.gguf")
        out[name] = (p, tv.write_gguf(p, *tv.build(**kw)))
    return out


@pytest.mark.parametrize("name", list(tv.VARIANTS))
def test_tokenizer_matches_reference_golden(fb, golden, vocab_files, name):
    path, sha = vocab_files[name]
    g = golden[name]
    assert sha == g["sha256"], "the vocabulary generator changed: regenerate the golden file"
    t = fb.Tokenizer(path)
    assert [t.chat_format, t.bos_id, t.eos_id, t.vocab_size] == g["info"]
    for text_hex, ids in g["encode"]:
        assert t.encode(bytes.fromhex(text_hex)) == ids, bytes.fromhex(text_hex)
    for ids, out_hex in g["decode"]:
        assert t.decode(ids) == bytes.fromhex(out_hex), ids
    for s, u, ids in g["chat"]:
        assert t.format_chat(s, u) == ids, (s, u)
    h = t.append([], fb.TURN_BEGIN)
    h = t.append(h, fb.TURN_SYSTEM, "be brief")
    h = t.append(h, fb.TURN_USER, "q1 ?")
    h = t.append(h, fb.TURN_ASSISTANT)
    h = t.append(h + [5, 6], fb.TURN_END)
    h = t.append(h, fb.TURN_USER, "second question")
    assert t.append(h, fb.TURN_ASSISTANT) == g["conversation"]
    t.close()


@pytest.mark.parametrize("name", list(tv.VARIANTS))
def test_tokenizer_matches_reference_build(fb, orc, vocab_files, name):
    if orc.ref_tok() is None:
        pytest.skip("oracle/_ref/libref_tok.so not built (no reference tree)")
    path, _ = vocab_files[name]
    a, r = fb.Tokenizer(path), orc.RefTokenizer(path)
    for text in tv.random_texts(200, seed=11):
        assert a.encode(text) == r.encode(text), text
    rng = np.random.default_rng(5)
    for _ in range(100):
        ids = [int(i) for i in rng.integers(0, a.vocab_size, int(rng.integers(1, 60)))]
        assert a.decode(ids) == r.decode(ids)
        # round trip: decoding and re-encoding keeps the bytes
        assert a.decode(a.encode(a.decode(ids))) == a.decode(ids)
    a.close()
    r.close()


def test_roundtrip_bytes(fb, vocab_files):
    """Every byte string survives encode -> decode when the vocabulary holds all 256 byte symbols."""
    t = fb.Tokenizer(vocab_files["chatml"][0])
    for text in tv.random_texts(100, seed=3) + [bytes(range(256))]:
        assert t.decode(t.encode(text)) == text
    t.close()


def test_long_text_is_fast(fb, vocab_files):
    t = fb.Tokenizer(vocab_files["chatml"][0])
    text = tv.corpus(99, 20000).encode("utf-8")  # ~130 KB, merged as one word, as the reference does
    t0 = time.perf_counter()
    ids = t.encode(text)
    assert time.perf_counter() - t0 < 5.0
    assert t.decode(ids) == text and len(ids) < len(text) // 2
    t.close()


def test_small_buffers_report_the_size_needed(fb, vocab_files):
    import ctypes
    t = fb.Tokenizer(vocab_files["chatml"][0])
    L = fb.lib()
    n = ctypes.c_int(0)
    buf = (ctypes.c_int * 2)()
    rc = L.fence_tokenize(t._h, b"hello world again", 17, buf, 2, ctypes.byref(n))
    assert rc == -1 and n.value == len(t.encode("hello world again"))
    need = ctypes.c_size_t(0)
    out = ctypes.create_string_buffer(3)
    ids = (ctypes.c_int * 2)(*t.encode("hello")[:2])
    rc = L.fence_detokenize(t._h, ids, 2, out, 3, ctypes.byref(need))
    assert rc == -1 and need.value == len(t.decode(list(ids)))
    t.close()


def test_load_rejects_a_file_without_tokens(fb, tmp_path):
    p = str(tmp_path / "empty.gguf")
    tv.write_gguf(p, [], [], {"general.architecture": "qwen3"})
    with pytest.raises(fb.FenceError, match="tokenizer"):
        fb.Tokenizer(p)


@pytest.mark.parametrize("name", ["llama2", "chatml"])
def test_chat_append_small_buffer_keeps_the_conversation(fb, vocab_files, name):
    """fence_chat_append with a buffer too small reports the total needed and changes neither the
    caller's ids nor the conversation (a LLaMA-2 system prompt held for the first user turn stays
    held), so a retry with the reported size gives the ids of an uninterrupted conversation."""
    import ctypes
    L = fb.lib()
    path = vocab_files[name][0]
    user = "a user message long enough to need many ids " * 4
    ref = fb.Tokenizer(path)
    want = ref.append(ref.append(ref.append([], fb.TURN_BEGIN), fb.TURN_SYSTEM, "be brief"), fb.TURN_USER, user)
    ref.close()
    t = fb.Tokenizer(path)
    h = t.append(t.append([], fb.TURN_BEGIN), fb.TURN_SYSTEM, "be brief")
    cap = len(h) + 2
    buf = (ctypes.c_int * cap)(*h)
    n = ctypes.c_int(len(h))
    rc = L.fence_chat_append(t._h, fb.TURN_USER, user.encode(), buf, cap, ctypes.byref(n))
    assert rc == -1 and n.value == len(want) and list(buf[:len(h)]) == h
    buf = (ctypes.c_int * n.value)(*h)
    need, n = n.value, ctypes.c_int(len(h))
    assert L.fence_chat_append(t._h, fb.TURN_USER, user.encode(), buf, need, ctypes.byref(n)) == 0
    assert list(buf[:n.value]) == want
    t.close()


def test_chat_append_grows_its_buffer(fb, orc, vocab_files):
    """A LLaMA-2 system prompt is held until the first user turn and emitted with it, so a short user
    turn can need far more ids than its own text: the Python helper retries with the size the C
    call reports."""
    path = vocab_files["llama2"][0]
    system = "a long system prompt for the whole conversation " * 6
    t = fb.Tokenizer(path)
    h = t.append(t.append(t.append([], fb.TURN_BEGIN), fb.TURN_SYSTEM, system), fb.TURN_USER, "hi")
    assert len(h) > 64 + 4 * len("hi") + 1  # more than the helper's first buffer
    h = t.append(h, fb.TURN_ASSISTANT)
    t.close()
    if orc.ref_tok() is not None:
        r = orc.RefTokenizer(path)
        want = r.append(r.append(r.append(r.append([], fb.TURN_BEGIN), fb.TURN_SYSTEM, system), fb.TURN_USER, "hi"),
                        fb.TURN_ASSISTANT)
        r.close()
        assert h == want
