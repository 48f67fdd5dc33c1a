"""Corrupted GGUF files through the host-side loader (csrc/gguf.cpp, the zero-copy parser the
reference's GGUFFile contract describes, src/gguf/gguf_parser.h) and the tokenizer built on it:
truncations, flipped bytes and huge counts / lengths must give a load error or a working
tokenizer, never a crash. Seeded; run in a child process so that a crash fails the test instead of
ending pytest. CPU only."""
import os
import random
import subprocess
import sys

import tok_vocab as tv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import sys
sys.path.insert(0, sys.argv[1])
from __graft_entry__ import _load_pkg
fb = _load_pkg()
loaded = 0
for p in sys.argv[2:]:
    try:
        t = fb.Tokenizer(p)
    except fb.FenceError:
        continue
    loaded += 1
    t.encode(b"hello world, \xe4\xb8\xad \xff")
    t.decode([0, 1, 2, t.vocab_size - 1])
    t.format_chat("sys", "user")
    t.close()
print("LOADED", loaded)
'''


def _corrupt(data: bytes, rng: random.Random, kind: int) -> bytes:
    b = bytearray(data)
    if kind == 0:  # truncated anywhere
        return bytes(b[:rng.randrange(len(b))])
    if kind == 1:  # bytes flipped in the header / metadata
        for _ in range(rng.randint(1, 8)):
            b[rng.randrange(min(len(b), 4096))] = rng.randrange(256)
    elif kind == 2:  # bytes flipped anywhere
        for _ in range(rng.randint(1, 32)):
            b[rng.randrange(len(b))] = rng.randrange(256)
    elif kind == 3:  # a huge 64-bit count or length
        off = rng.randrange(8, min(len(b) - 8, 2048))
        b[off:off + 8] = rng.choice([b"\xff" * 8, (2**31).to_bytes(8, "little"), (2**62).to_bytes(8, "little")])
    else:  # a 32-bit type tag or count replaced
        off = rng.randrange(8, len(b) - 4)
        b[off:off + 4] = rng.choice([b"\xff" * 4, (2**31).to_bytes(4, "little"), (0).to_bytes(4, "little"),
                                     (9).to_bytes(4, "little")])
    return bytes(b)


def test_corrupted_files_fail_cleanly(fb, tmp_path):
    base = str(tmp_path / "base.gguf")
    tv.write_gguf(base, *tv.build(**tv.VARIANTS["llama2"]))
    data = open(base, "rb").read()
    rng = random.Random(2024)
    paths = []
    for i in range(250):
        p = str(tmp_path / f"c{i}.gguf")
        with open(p, "wb") as f:
            f.write(_corrupt(data, rng, i % 5))
        paths.append(p)
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT] + paths, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "LOADED" in r.stdout, r.stderr[-2000:]
    loaded = int(r.stdout.split("LOADED")[1].split()[0])
    assert 0 < loaded < len(paths)  # some corruptions are harmless (string bytes), most are not
