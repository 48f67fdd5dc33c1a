"""Q6_K / Q8_0 GEMV kernels through the C-ABI against the oracle and the reference's golden cases.

Tolerance (stated by BASELINE.json's north star): relative 1e-3 of max(|y_ref|, 1) per row against
the fp64 host dequant-dot. The reference's own test (tests/test_gemv_q6k.cu:134-164) fails a row
only if |err| > 0.5 AND rel > 5e-3; the bound used here is stricter.
"""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
RTOL = 1e-3


def dev_bytes(torch, b, offset=0):
    """Device copy of raw bytes, starting `offset` bytes into a 256-aligned allocation."""
    arr = np.frombuffer(bytes(b), np.uint8)
    t = torch.zeros(arr.size + offset + 16, dtype=torch.uint8, device="cuda")
    t[offset:offset + arr.size] = torch.from_numpy(arr.copy()).cuda()
    return t, t.data_ptr() + offset


def run_q6k(fb, torch, W, x_bits, M, K, offset=0, bias=None):
    tw, pw = dev_bytes(torch, W, offset)
    tx = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16).copy()).cuda()
    y = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    if bias is None:
        fb.call("fence_gemv_q6k", pw, tx.data_ptr(), y.data_ptr(), M, K, None)
    else:
        tb = torch.from_numpy(bias).cuda()
        fb.call("fence_gemv_q6k_bias", pw, tx.data_ptr(), tb.data_ptr(), y.data_ptr(), M, K, None)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def run_q8(fb, torch, W, x, M, K, offset=0):
    tw, pw = dev_bytes(torch, W, offset)
    tx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    y = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    fb.call("fence_gemv_q8_0", pw, tx.data_ptr(), y.data_ptr(), M, K, None)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def assert_close(got, ref, rtol=RTOL):
    ref = np.asarray(ref, np.float64)
    err = np.abs(got.astype(np.float64) - ref) / np.maximum(np.abs(ref), 1.0)
    assert np.isfinite(got).all()
    assert err.max() <= rtol, f"max rel err {err.max():.3e} at row {int(err.argmax())}"


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.mark.parametrize("name", ["ref_gemv_64x256", "ref_gemv_128x512"])
def test_reference_seeded_cases(fb, torch_cuda, name):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    y = run_q6k(fb, torch_cuda, g["W"].tobytes(), g["x"], int(g["M"]), int(g["K"]))
    assert_close(y, g["y"])


def test_reference_dot_blocks(fb, torch_cuda):
    g = np.load(os.path.join(GOLDEN, "ref_q6k_dot_cases.npz"))
    for i in range(6):
        y = run_q6k(fb, torch_cuda, g[f"blk{i}"].tobytes(), g[f"x{i}"], 1, 256)
        exp = float(g["expected"][i])
        # the reference's per-block criterion (tests/test_q6k_dot.cu:168,214-216)
        assert abs(y[0] - exp) < 1e-2 or abs(y[0] - exp) / max(abs(exp), 1e-6) < 1e-3, (i, y[0], exp)


def test_config0_4096x4096(fb, orc, torch_cuda):
    M = K = 4096
    W = fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=11)
    x = np.random.default_rng(11).standard_normal(K).astype(np.float32).astype(np.float16).view(np.uint16)
    y = run_q6k(fb, torch_cuda, W, x, M, K)
    assert_close(y, orc.gemv_q6k(W, x, M, K))


@pytest.mark.parametrize("M,K", [(1, 256), (3, 512), (37, 2560), (1024, 2560), (515, 5120), (96, 9728),
                                 (200, 17408), (6144, 2560), (2, 4096)])
def test_q6k_shapes(fb, orc, torch_cuda, M, K):
    W = fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=M * 7 + K)
    x = (np.random.default_rng(K).standard_normal(K) * 3).astype(np.float32).astype(np.float16).view(np.uint16)
    assert_close(run_q6k(fb, torch_cuda, W, x, M, K), orc.gemv_q6k(W, x, M, K))


@pytest.mark.parametrize("M,K", [(1, 2048), (300, 2048), (4096, 2048), (149, 4096), (10000, 4096), (6144, 4096)])
def test_q6k_shapes_with_bias(fb, orc, torch_cuda, M, K):
    W = fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=M * 3 + K)
    x = (np.random.default_rng(M).standard_normal(K) * 2).astype(np.float32).astype(np.float16).view(np.uint16)
    ref = orc.gemv_q6k(W, x, M, K)
    assert_close(run_q6k(fb, torch_cuda, W, x, M, K), ref)
    bias = np.random.default_rng(M + 1).standard_normal(M).astype(np.float32)
    assert_close(run_q6k(fb, torch_cuda, W, x, M, K, bias=bias), ref + bias)


def test_q6k_pdl_chain_reads_the_previous_kernels_output(fb, orc, torch_cuda):
    """With FENCE_LAUNCH_PDL the GEMV streams its weights before the previous kernel ends, but its x
    (here written by the kernel just before it) is read only after griddepcontrol.wait: x2 starts as
    NaN bits each round and every round uses a new x, so an early read would show in y2."""
    torch = torch_cuda
    M = K = 4096
    W1 = fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=31)
    W2 = fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=32)
    t1, p1 = dev_bytes(torch, W1, 0)
    t2, p2 = dev_bytes(torch, W2, 0)
    old = fb.lib().fence_set_launch_flags(fb.FENCE_LAUNCH_PDL)
    try:
        for r in range(3):
            x = np.random.default_rng(40 + r).standard_normal(K).astype(np.float32).astype(np.float16).view(np.uint16)
            tx = torch.from_numpy(x.view(np.int16).copy()).cuda()
            y1 = torch.empty(M, dtype=torch.float32, device="cuda")
            x2 = torch.full((M,), 0x7E00, dtype=torch.int16, device="cuda")  # fp16 NaN
            y2 = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            fb.call("fence_gemv_q6k", p1, tx.data_ptr(), y1.data_ptr(), M, K, None)
            fb.call("fence_f32_to_f16", x2.data_ptr(), y1.data_ptr(), M, None)
            fb.call("fence_gemv_q6k", p2, x2.data_ptr(), y2.data_ptr(), M, K, None)
            torch.cuda.synchronize()
            got_y1 = y1.cpu().numpy()
            got_x2 = x2.cpu().numpy().view(np.uint16)
            assert_close(got_y1, orc.gemv_q6k(W1, x, M, K))
            assert np.array_equal(got_x2, got_y1.astype(np.float16).view(np.uint16))
            assert_close(y2.cpu().numpy(), orc.gemv_q6k(W2, got_x2, M, K))
    finally:
        fb.lib().fence_set_launch_flags(old)


def test_q6k_misaligned_pointer_and_bias(fb, orc, torch_cuda):
    M, K = 129, 1024
    W = fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=5)
    x = np.random.default_rng(5).standard_normal(K).astype(np.float32).astype(np.float16).view(np.uint16)
    ref = orc.gemv_q6k(W, x, M, K)
    assert_close(run_q6k(fb, torch_cuda, W, x, M, K, offset=2), ref)  # 2-byte aligned: fallback kernel
    bias = np.random.default_rng(6).standard_normal(M).astype(np.float32)
    assert_close(run_q6k(fb, torch_cuda, W, x, M, K, bias=bias), ref + bias)


def test_q6k_extreme_values(fb, orc, torch_cuda):
    """Scales at +-127/-128, all quants at the range ends and large activations stay exact-range."""
    M, K = 64, 1024
    W = np.frombuffer(fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=9), np.uint8).copy().reshape(-1, 210)
    W[::3, 0:192] = 0x00      # q = 0 -> -32
    W[1::3, 0:192] = 0xFF     # q = 63 -> 31
    W[:, 192:208] = np.where(np.arange(16) % 2 == 0, 127, -128).astype(np.int8).view(np.uint8)
    W[:, 208:210] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    x = np.full(K, 60000.0, np.float32)
    x[::2] = -65504.0
    xb = x.astype(np.float16).view(np.uint16)
    assert_close(run_q6k(fb, torch_cuda, W.tobytes(), xb, M, K), orc.gemv_q6k(W.tobytes(), xb, M, K))


def test_q6k_deterministic(fb, torch_cuda):
    M, K = 2048, 4096
    W = fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=2)
    x = np.random.default_rng(2).standard_normal(K).astype(np.float32).astype(np.float16).view(np.uint16)
    a = run_q6k(fb, torch_cuda, W, x, M, K)
    b = run_q6k(fb, torch_cuda, W, x, M, K)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("M,K", [(1, 64), (5, 2560), (1000, 4096), (3000, 14336), (151936, 2560), (77, 96), (33, 32)])
def test_q8_0_shapes(fb, orc, torch_cuda, M, K):
    W = fb.synth_blocks(fb.GGML_Q8_0, M * K // 32, seed=M + K)
    x = np.random.default_rng(M).standard_normal(K).astype(np.float32)
    assert_close(run_q8(fb, torch_cuda, W, x, M, K), orc.gemv_q8_0(W, x, M, K))


def test_q8_0_misaligned_fallback(fb, orc, torch_cuda):
    M, K = 50, 512
    W = fb.synth_blocks(fb.GGML_Q8_0, M * K // 32, seed=3)
    x = np.random.default_rng(3).standard_normal(K).astype(np.float32)
    assert_close(run_q8(fb, torch_cuda, W, x, M, K, offset=2), orc.gemv_q8_0(W, x, M, K))


def test_embed_q8_0(fb, orc, torch_cuda):
    V, H = 300, 2560
    W = fb.synth_blocks(fb.GGML_Q8_0, V * H // 32, seed=4)
    tw, pw = dev_bytes(torch_cuda, W)
    out = torch_cuda.zeros(H, dtype=torch_cuda.float32, device="cuda")
    for tok in [0, 1, 299]:
        fb.call("fence_embed_q8_0", out.data_ptr(), pw, tok, H, None)
        ref = np.empty(H, np.float32)
        Wb = np.frombuffer(W, np.uint8)
        orc.oracle().oracle_embed_q8_0(ref.ctypes.data_as(ctypes.c_void_p), Wb.ctypes.data_as(ctypes.c_void_p), tok, H)
        assert np.array_equal(out.cpu().numpy(), ref)  # exact: d * q is representable
