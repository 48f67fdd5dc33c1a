"""Pins the CPU oracle (oracle/fence_oracle.c) to the reference's own known answers before any
kernel is compared with it:

* the six hand-built Q6_K blocks of tests/test_q6k_dot.cu:242-332 and their fp64 host oracle,
* the seeded GEMV cases of tests/test_gemv_q6k.cu:167-269 (64x256, 128x512), regenerated with the
  same glibc rand() sequence, and the reference's cpu_gemv_q6k on config 0 (4096x4096),
* the committed golden fixtures in tests/golden/ (made by tests/golden/make_golden.py from the
  reference's compiled host oracle).
"""
import ctypes
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_dot_golden_blocks_match_reference(orc):
    ref = orc.ref_cpu()
    data = np.load(os.path.join(GOLDEN, "ref_q6k_dot_cases.npz"))
    for idx in range(6):
        blk = data[f"blk{idx}"]
        x = data[f"x{idx}"]
        expected = float(data["expected"][idx])
        got = orc.oracle().oracle_q6k_dot_block(_p(blk), _p(x))
        assert got == expected, (idx, got, expected)  # same fp64 operations, same order
        if ref is not None:
            b2 = np.zeros(210, np.uint8)
            x2 = np.zeros(256, np.uint16)
            e2 = ctypes.c_double()
            assert ref.ref_dot_case(idx, _p(b2), _p(x2), ctypes.byref(e2)) == 0
            assert np.array_equal(b2, blk) and np.array_equal(x2, x) and e2.value == expected


def test_dot_golden_blocks_analytic(orc):
    data = np.load(os.path.join(GOLDEN, "ref_q6k_dot_cases.npz"))
    exp = data["expected"]
    assert exp[0] == 0.0  # all quants 32 -> zero-centred
    assert exp[4] == 0.0  # alternating +-4 scales cancel
    d01 = float(np.float16(0.1))
    assert exp[5] == pytest.approx(d01 * 10 * 13 * 16, rel=1e-12)  # one sub-block, q-32 = 13
    d05 = float(np.float16(0.05))
    assert exp[1] == pytest.approx(d05 * 3 * (-32) * 0.5 * 256, rel=1e-12)
    assert exp[2] == pytest.approx(d05 * 3 * 31 * 0.5 * 256, rel=1e-12)


@pytest.mark.parametrize("name", ["ref_gemv_64x256", "ref_gemv_128x512"])
def test_seeded_gemv_fixture(orc, name):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    W, x, y, M, K = g["W"], g["x"], g["y"], int(g["M"]), int(g["K"])
    got = orc.gemv_q6k(W, x, M, K)
    assert np.array_equal(got, y)  # bit-exact against the reference's cpu_gemv_q6k


def _glibc():
    return ctypes.CDLL("libc.so.6")


def regen_reference_case(orc, seed, M, K, d, scale_mod, x_lo, x_span):
    """tests/test_gemv_q6k.cu:167-191 / :222-244 — same rand() call order."""
    ref = orc.ref_cpu()
    libc = _glibc()
    libc.srand(seed)
    nb = K // 256
    W = np.zeros(M * nb * 210, np.uint8)
    dbits = np.float16(d).view(np.uint16)
    for b in range(M * nb):
        blk = W[b * 210:(b + 1) * 210]
        blk[208:210] = np.frombuffer(np.uint16(dbits).tobytes(), np.uint8)
        for s in range(16):
            blk[192 + s] = np.int8((libc.rand() % scale_mod) - scale_mod // 2).view(np.uint8)
        for i in range(256):
            ref.ref_set_q6(_p(blk), i, libc.rand() % 64)
    RAND_MAX = np.float32(2147483647)
    x = np.empty(K, np.float32)
    for i in range(K):
        r = np.float32(libc.rand())
        x[i] = np.float32(x_lo) + (np.float32(x_span) * r) / RAND_MAX
    return W, x.astype(np.float16).view(np.uint16)


def test_seeded_cases_regenerate_from_reference_rng(orc):
    if orc.ref_cpu() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    g = np.load(os.path.join(GOLDEN, "ref_gemv_64x256.npz"))
    W, x = regen_reference_case(orc, 123, 64, 256, 0.05, 21, -1.0, 2.0)
    assert np.array_equal(W, g["W"]) and np.array_equal(x, g["x"])


def test_config0_oracle_equals_reference_host_gemv(fb, orc):
    ref = orc.ref_cpu()
    if ref is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    M = K = 4096
    W = np.frombuffer(fb.synth_blocks(fb.GGML_Q6_K, M * K // 256, seed=7), np.uint8)
    x = np.random.default_rng(0).standard_normal(K).astype(np.float32).astype(np.float16).view(np.uint16)
    y_ref = np.zeros(M, np.float64)
    ref.ref_cpu_gemv_q6k(_p(W), _p(x), _p(y_ref), M, K)
    y = orc.gemv_q6k(W, x, M, K)
    assert np.array_equal(y, y_ref)
    assert 1.0 < float(np.sqrt(np.mean(y ** 2))) < 1.6  # analytic rms ~1.28


def test_fp16_bf16_conversions_match_numpy(orc):
    o = orc.oracle()
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                           np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 6e-8, 5.96e-8, 1e5, -1e5,
                                     np.inf, -np.inf], np.float32)])
    for v in vals:
        assert o.oracle_f2h(float(v)) == int(np.float16(v).view(np.uint16)), v
        h = int(np.float16(v).view(np.uint16))
        back = o.oracle_h2f(h)
        assert (np.isnan(back) and np.isnan(np.float16(v))) or back == float(np.float16(v))
    import torch
    t = torch.from_numpy(vals[np.isfinite(vals)])
    bf = t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    for v, b in zip(vals[np.isfinite(vals)], bf):
        assert o.oracle_f2bf(float(v)) == int(b), v


def ref_argmax_py(x):
    """Pure-Python run of the reference argmax kernel (ops.cuh:467-499) with 256 threads."""
    bv = [-1e30] * 256
    bi = [0] * 256
    for t in range(256):
        for i in range(t, len(x), 256):
            if x[i] > bv[t]:
                bv[t], bi[t] = x[i], i
    s = 128
    while s > 0:
        for t in range(s):
            if bv[t + s] > bv[t]:
                bv[t], bi[t] = bv[t + s], bi[t + s]
        s //= 2
    return bi[0]


def test_argmax_tie_order(orc):
    x = np.zeros(1000, np.float32)
    x[[10, 256]] = 5.0  # threads 0 and 10: 0 wins
    assert orc.argmax(x) == 256 == ref_argmax_py(x)
    x = np.zeros(1000, np.float32)
    x[[300, 5]] = 5.0  # threads 44 (bit-reversed 52) and 5 (bit-reversed 160): 44 wins
    assert orc.argmax(x) == 300 == ref_argmax_py(x)
    x = np.full(600, -np.inf, np.float32)
    assert orc.argmax(x) == 0  # nothing above -1e30
    x = np.zeros(600, np.float32)
    x[7] = np.nan
    x[9] = 1.0
    assert orc.argmax(x) == 9  # NaN never wins
    x = np.zeros(513, np.float32)
    x[[1, 257, 258]] = 2.0  # thread 1 keeps 1 (first of 1, 257); thread 2 (rev 64) beats thread 1 (rev 128)
    assert orc.argmax(x) == 258 == ref_argmax_py(x)


def test_argmax_random_ties_match_python_restatement(orc):
    rng = np.random.default_rng(5)
    for n in [1, 7, 255, 256, 257, 1000, 4099]:
        for _ in range(5):
            x = rng.integers(0, 4, n).astype(np.float32)  # many exact ties
            assert orc.argmax(x) == ref_argmax_py(x.tolist())


def test_oracle_nucleus_known_answers(orc):
    """Hand-checkable draws of the oracle's sample_nucleus (qwen3.cu:351-460) with explicit u."""
    import ctypes
    O = orc.oracle()

    def draw(logits, hist, temp, top_p, top_k, rp, min_p, dyn, u):
        l = np.asarray(logits, np.float32)
        h = np.asarray(hist, np.int32)
        hp = h.ctypes.data_as(ctypes.c_void_p) if h.size else None
        return O.oracle_sample_nucleus(l.ctypes.data_as(ctypes.c_void_p), l.size, hp, h.size, temp, top_p, top_k,
                                       rp, min_p, dyn, u, None, None)

    # top_p reached by the first entry: always the argmax, whatever u
    assert draw([0.0, 5.0, 1.0, 2.0], [], 1.0, 0.5, 4, 1.0, 0.0, 0, 0.99) == 1
    # two kept entries with probabilities 1/(1+e^-1) and e^-1/(1+e^-1): u picks one or the other
    p0 = 1.0 / (1.0 + np.exp(-1.0))
    assert draw([1.0, 0.0, -9.0], [], 1.0, 0.99, 2, 1.0, 0.0, 0, p0 - 1e-3) == 0
    assert draw([1.0, 0.0, -9.0], [], 1.0, 0.99, 2, 1.0, 0.0, 0, p0 + 1e-3) == 1
    # penalty twice on id 0 (2.0 / 1.5 / 1.5 = 0.889 < 1.0): id 1 becomes the argmax
    assert draw([2.0, 1.0, -9.0], [0, 0], 1.0, 0.1, 3, 1.5, 0.0, 0, 0.5) == 1
    # a negative logit is multiplied: id 0 goes from -0.1 to -0.15, below id 1 at -0.12
    assert draw([-0.1, -0.12, -9.0], [0], 1.0, 0.1, 3, 1.5, 0.0, 0, 0.5) == 1
    # min-p drops everything more than log(1/min_p) below the max: only id 2 survives
    assert draw([0.0, 1.0, 5.0], [], 1.0, 1.0, 3, 1.0, 0.05, 1, 0.999) == 2
