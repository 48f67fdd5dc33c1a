"""Seeded byte-level BPE vocabularies written as tensor-less GGUF files, for the tokenizer tests.

The vocabulary is trained here on a seeded synthetic corpus (syllables, digits, punctuation and a
few multi-byte scripts), so every byte-mapping, merge and fallback path of the tokenizer is
exercised without any real model file. Variants differ in the metadata that selects the chat
format (general.architecture, tokenizer.chat_template), in the special tokens present, and in
holes: `drop` removes some byte symbols and merge results from the vocabulary so that the
reference's per-character fallback and dropping paths run.
"""
import hashlib
import struct

import numpy as np

SYLLABLES = ["ka", "to", "ri", "men", "sha", "lo", "vin", "que", "tra", "el", "an", "th", "ing", "ou", "st",
             "re", "de", "pa", "zo", "ix", "ß", "é", "ü", "ñ", "日", "本", "語", "ж", "ы", "€", "😀"]
PUNCT = [" ", " ", " ", " ", ",", ".", "\n", "!", "?", "-", "'", "\t", "  "]


def corpus(seed=7, n_words=3000):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_words):
        w = "".join(SYLLABLES[int(i)] for i in rng.integers(0, len(SYLLABLES), int(rng.integers(1, 4))))
        if rng.random() < 0.1:
            w = str(int(rng.integers(0, 1000)))
        if rng.random() < 0.2:
            w = w.capitalize()
        out.append(w + PUNCT[int(rng.integers(0, len(PUNCT)))])
    return "".join(out)


def byte_map():
    """GPT-2's byte -> code point table (printable ASCII / Latin-1 keep their value)."""
    m, n = {}, 0
    for b in range(256):
        if 0x21 <= b <= 0x7E or 0xA1 <= b <= 0xAC or 0xAE <= b <= 0xFF:
            m[b] = b
        else:
            m[b] = 256 + n
            n += 1
    return m


def mapped(text):
    bm = byte_map()
    return "".join(chr(bm[b]) for b in text.encode("utf-8"))


def train_bpe(text, n_merges):
    """Classic pair-count BPE over space-split chunks of the mapped text: returns the merges
    ("a b" strings) in rank order."""
    words = {}
    for w in mapped(text).split(chr(byte_map()[0x20])):
        if w:
            key = tuple(w)
            words[key] = words.get(key, 0) + 1
    merges = []
    for _ in range(n_merges):
        counts = {}
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + c
        if not counts:
            break
        (a, b), _ = max(counts.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append(a + " " + b)
        new = {}
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and w[i] == a and w[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            new[tuple(out)] = new.get(tuple(out), 0) + c
        words = new
    return merges


def build(arch, template=None, specials=(), with_merges=True, drop=0, n_merges=300, bos=None, eos=None,
          seed=7):
    """(tokens, merges, metadata) of one vocabulary variant."""
    bm = byte_map()
    tokens = [chr(bm[b]) for b in range(256)]
    merges = train_bpe(corpus(seed), n_merges) if with_merges else []
    for m in merges:
        t = m.replace(" ", "")
        if t not in tokens:
            tokens.append(t)
    if not with_merges:  # longest-match vocabularies: a few multi-symbol tokens from the merges
        for m in train_bpe(corpus(seed), 120):
            t = m.replace(" ", "")
            if t not in tokens:
                tokens.append(t)
    if drop:
        rng = np.random.default_rng(seed + 1)
        idx = sorted(set(int(i) for i in rng.integers(0, len(tokens), drop)), reverse=True)
        for i in idx:
            tokens.pop(i)
    tokens += list(specials)
    meta = {"general.architecture": arch}
    if template is not None:
        meta["tokenizer.chat_template"] = template
    if bos is not None:
        meta["tokenizer.ggml.bos_token_id"] = ("u32", bos)
    if eos is not None:
        meta["tokenizer.ggml.eos_token_id"] = ("i32", eos)
    return tokens, merges, meta


def write_gguf(path, tokens, merges, meta):
    """A GGUF v3 file with no tensors: metadata, the token strings and the merges."""
    out = bytearray()

    def s(x):
        b = x if isinstance(x, bytes) else x.encode("utf-8")
        out.extend(struct.pack("<Q", len(b)))
        out.extend(b)

    kvs = [(k, v) for k, v in meta.items()]
    n_kv = len(kvs) + 1 + (1 if merges else 0)
    out.extend(struct.pack("<IIQQ", 0x46554747, 3, 0, n_kv))
    for k, v in kvs:
        s(k)
        if isinstance(v, tuple):
            out.extend(struct.pack("<I", 4 if v[0] == "u32" else 5))
            out.extend(struct.pack("<I" if v[0] == "u32" else "<i", v[1]))
        else:
            out.extend(struct.pack("<I", 8))
            s(v)
    for key, arr in (("tokenizer.ggml.tokens", tokens), ("tokenizer.ggml.merges", merges)):
        if key.endswith("merges") and not merges:
            continue
        s(key)
        out.extend(struct.pack("<IIQ", 9, 8, len(arr)))
        for t in arr:
            s(t)
    while len(out) % 32:
        out.append(0)
    with open(path, "wb") as f:
        f.write(out)
    return hashlib.sha256(bytes(out)).hexdigest()


L3 = ["<|begin_of_text|>", "<|start_header_id|>", "<|end_header_id|>", "<|eot_id|>"]
MI = ["<s>", "</s>", "[INST]", "[/INST]"]
VARIANTS = {
    # ChatML by architecture (fixed <|im_start|> / <|im_end|> ids), full merges
    "chatml": dict(arch="qwen3"),
    # LLaMA-3 by architecture, its four markers present: bos / eos come from them
    "llama3": dict(arch="llama", specials=L3, bos=1, eos=2),
    # Mistral by a template containing [INST]; markers present, eos from </s>
    "mistral": dict(arch="llama", template="{% for m in messages %}[INST] {{ m }} [/INST]{% endfor %}",
                    specials=MI),
    # LLaMA-2 by a <<SYS>> template; a hole-punched vocabulary (fallback and dropped characters)
    "llama2": dict(arch="llama", template="[INST] <<SYS>>\n{{ sys }}\n<</SYS>>\n\n", specials=MI, drop=40),
    # template naming im_start wins over the architecture
    "chatml_tmpl": dict(arch="llama", template="<|im_start|>{{ role }}", specials=L3),
    # raw (unknown architecture), no merges: greedy longest match; eos given as int32
    "raw": dict(arch="gpt2", with_merges=False, eos=5),
    # raw without merges and with holes; a few token strings that are not clean GPT-2 symbols
    # (truncated UTF-8, code points outside the byte map) for the decoder's '?' paths
    "raw_holes": dict(arch="phi9", with_merges=False, drop=30,
                      specials=[b"\xc3", b"\xe6\x97", b"\xf0\x9f\x98", b"\xff\xfe", "\u017f", "\u65e5x", b"\x80a"]),
}

TEXTS = [
    "", "a", " ", "hello world", "Hello, world! 123", "katomen shalo vinque.", "  double  spaces\tand\ttabs\n",
    "ßéüñ straße café", "日本語のテキスト", "жыр жыр", "€100 😀 end", "tra-la-la? re:de;pa",
    "\x00\x01\x7f control", "ingthou stre dezo ix", "Zo Pa De Re", "x" * 300,
]


def random_texts(n, seed):
    """Texts as bytes: slices of another seeded corpus, and arbitrary byte strings (invalid UTF-8
    included: the byte map covers every byte)."""
    rng = np.random.default_rng(seed)
    c = corpus(seed + 100, 400)
    out = []
    for _ in range(n):
        i = int(rng.integers(0, len(c) - 1))
        out.append(c[i:i + int(rng.integers(1, 200))].encode("utf-8"))
    for _ in range(n // 4):
        out.append(bytes(rng.integers(0, 256, int(rng.integers(1, 40)), dtype=np.uint8)))
    return out
