"""The C-ABI boundary on the CPU: every symbol declared in include/fence_b200.h is exported by
libfence_b200.so and bound by the Python module; argument validation happens on the host and
reports errors without touching a device; the CLI keeps the reference's flag surface."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fence_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    c_part = text.split("#ifdef __cplusplus\n} /* extern \"C\" */")[0]
    return sorted(set(re.findall(r"\b(fence_[a-z0-9_]+)\s*\(", c_part)))


def test_header_symbols_exported(fb):
    names = declared_symbols()
    assert len(names) >= 35
    lib = fb.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header(fb):
    bound = {n for n, _, _ in fb.SIGNATURES}
    assert set(declared_symbols()) <= bound


def test_no_oracle_in_product_library(fb):
    out = subprocess.run(["nm", "-D", fb.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle_" not in out and "ref_cpu" not in out


def test_dropin_argument_errors_are_host_side(fb):
    L = fb.lib()
    assert L.fence_gemv_q6k(None, None, None, 4, 256, None) == -1
    assert "gemv_q6k" in fb.last_error()
    assert L.fence_gemv_q6k(1, 2, 3, 4, 300, None) == -1  # K % 256 != 0
    assert L.fence_gemv_q8_0(1, 2, 3, 4, 33, None) == -1  # K % 32 != 0
    assert L.fence_gqa_attention(1, 2, 3, 4, 128, 32, 5, 10, 4096, 5, None) == -1  # 32 % 5 != 0
    assert L.fence_gqa_attention(1, 2, 16, 16, 128, 32, 2, 10, 4096, 5, None) == -4  # G = 16 > 8
    assert L.fence_gqa_attention(1, 2, 16, 16, 96, 8, 2, 10, 4096, 5, None) == -4  # head_dim 96
    assert L.fence_store_kv(1, 2, 3, 4, 4096, 1024, 4096, None) == -1  # pos out of range
    assert L.fence_argmax(None, None, 10, None) == -1
    # the static-scratch attention variant checks its arguments and its scratch bound on the host
    assert L.fence_gqa_attention_static(1, 2, 3, 4, 128, 32, 5, 10, 4096, None) == -1
    assert L.fence_gqa_attention_static(1, 2, 16, 16, 96, 8, 2, 10, 4096, None) == -4
    assert L.fence_gqa_attention_static(1, 2, 16, 16, 128, 64, 8, 8320, 8320, None) == -8  # 64 chunks
    assert "static scratch" in fb.last_error()


def test_model_load_rejects_bad_files_on_host(fb, tmp_path):
    with pytest.raises(fb.FenceError, match="cannot open"):
        fb.Model(str(tmp_path / "missing.gguf"))
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(fb.FenceError, match="invalid magic"):
        fb.Model(str(bad))
    v9 = tmp_path / "v9.gguf"
    v9.write_bytes(b"GGUF" + (9).to_bytes(4, "little") + b"\0" * 16)
    with pytest.raises(fb.FenceError, match="unsupported version"):
        fb.Model(str(v9))


def test_model_load_rejects_truncated_and_missing(fb, tmp_path):
    p = str(tmp_path / "m.gguf")
    fb.synth_write(p, "tiny-q6k")
    data = open(p, "rb").read()
    t = tmp_path / "trunc.gguf"
    t.write_bytes(data[: len(data) - 4096])
    with pytest.raises(fb.FenceError, match="exceeds file size"):
        fb.Model(str(t))
    # a model whose head_dim is not 128 is refused with a reason
    p2 = str(tmp_path / "hd64.gguf")
    fb.synth_write(p2, "tiny-q6k", head_dim=64)
    with pytest.raises(fb.FenceError, match="head_dim"):
        fb.Model(p2)


def test_cli_flags(fb):
    exe = os.path.join(fb.HERE, "fence")
    r = subprocess.run([exe, "--help"], capture_output=True, text=True)
    assert r.returncode == 0
    for flag in ["--model", "--prompt", "--system", "--max-tokens", "--max-ctx", "--temp", "--top-p",
                 "--top-k", "--rep-penalty", "--debug", "--help"]:
        assert flag in r.stdout
    r = subprocess.run([exe, "--bogus"], capture_output=True, text=True)
    assert r.returncode == 1 and "Unknown option" in r.stderr
    r = subprocess.run([exe], capture_output=True, text=True)
    assert r.returncode == 1 and "--model PATH is required" in r.stderr
