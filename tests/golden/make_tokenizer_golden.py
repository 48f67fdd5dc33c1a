"""Writes tests/golden/tokenizer_golden.json: the reference's own Tokenizer (src/tokenizer/tokenizer.cpp,
compiled unmodified into oracle/_ref/libref_tok.so by oracle/Makefile) run on the seeded vocabularies
of tests/tok_vocab.py. For each variant: the GGUF file's sha256 (the generator is pinned with it),
format / bos / eos / vocabulary size, the ids of fixed and seeded texts, the bytes of seeded id
sequences, format_chat for three prompt pairs and one multi-turn conversation.

    python tests/golden/make_tokenizer_golden.py      (needs the reference tree built into oracle/_ref)
"""
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
import oracle as orc  # noqa: E402
import tok_vocab as tv  # noqa: E402

CHATS = [("You are a helpful assistant.", "Hello there!"), ("", "hi"), ("sys ß", "日本語 user\n")]


def conversation(t):
    """begin, system, user, assistant header, a 2-token reply, turn end, user, assistant header."""
    h = t.append([], tv_turn("BEGIN"))
    h = t.append(h, tv_turn("SYSTEM"), "be brief")
    h = t.append(h, tv_turn("USER"), "q1 ?")
    h = t.append(h, tv_turn("ASSISTANT"))
    h = h + [5, 6]
    h = t.append(h, tv_turn("END"))
    h = t.append(h, tv_turn("USER"), "second question")
    return t.append(h, tv_turn("ASSISTANT"))


def tv_turn(name):
    return ["BEGIN", "SYSTEM", "USER", "ASSISTANT", "END"].index(name)


def decode_cases(vocab, seed=2, n=40):
    rng = np.random.default_rng(seed)
    return [[int(i) for i in rng.integers(-3, vocab + 3, int(rng.integers(0, 30)))] for _ in range(n)]


def main():
    if orc.ref_tok() is None:
        sys.exit("oracle/_ref/libref_tok.so is not built (run make -C oracle with the reference tree present)")
    out = {}
    with tempfile.TemporaryDirectory() as d:
        for name, kw in tv.VARIANTS.items():
            p = os.path.join(d, f"{name}.gguf")
            sha = tv.write_gguf(p, *tv.build(**kw))
            r = orc.RefTokenizer(p)
            texts = [t.encode("utf-8") for t in tv.TEXTS] + tv.random_texts(40, seed=1)
            dec = decode_cases(r.vocab_size)
            out[name] = {
                "sha256": sha,
                "info": [r.chat_format, r.bos_id, r.eos_id, r.vocab_size],
                "encode": [[t.hex(), r.encode(t)] for t in texts],
                "decode": [[ids, r.decode(ids).hex()] for ids in dec],
                "chat": [[s, u, r.format_chat(s, u)] for s, u in CHATS],
                "conversation": conversation(r),
            }
            r.close()
    with open(os.path.join(HERE, "tokenizer_golden.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("wrote", os.path.join(HERE, "tokenizer_golden.json"))


if __name__ == "__main__":
    main()
