"""Drop-in ops of src/kernels/ops.cuh through the C-ABI against the oracle (fp32 tolerance 1e-5
relative unless the op is bit-exact: conversions, KV stores, argmax)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def T():
    import torch
    assert torch.cuda.is_available()
    return torch


def P(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def cu(T, a):
    return T.from_numpy(np.ascontiguousarray(a)).cuda()


def test_rms_norm_and_inplace(fb, orc, T):
    rng = np.random.default_rng(0)
    for n in [1, 100, 2560, 4096, 5120, 17408]:
        x = rng.standard_normal(n).astype(np.float32) * 3
        w = rng.standard_normal(n).astype(np.float32)
        ref = np.empty(n, np.float32)
        orc.oracle().oracle_rms_norm(P(ref), P(x), P(w), n, 1e-6)
        dx, dw, dout = cu(T, x), cu(T, w), T.empty(n, device="cuda")  # all kept alive across the launches
        fb.call("fence_rms_norm", dout.data_ptr(), dx.data_ptr(), dw.data_ptr(), n, 1e-6, None)
        fb.call("fence_rms_norm_inplace", dx.data_ptr(), dw.data_ptr(), n, 1e-6, None)
        np.testing.assert_allclose(dout.cpu().numpy(), ref, rtol=2e-5, atol=1e-6)
        np.testing.assert_allclose(dx.cpu().numpy(), ref, rtol=2e-5, atol=1e-6)


def test_rms_norm_per_head(fb, orc, T):
    rng = np.random.default_rng(1)
    for nh, hd in [(32, 128), (8, 128), (5, 64), (3, 256)]:
        x = rng.standard_normal(nh * hd).astype(np.float32)
        w = rng.standard_normal(hd).astype(np.float32)
        ref = x.copy()
        orc.oracle().oracle_rms_norm_per_head(P(ref), P(w), nh, hd, 1e-6)
        dx, dw = cu(T, x), cu(T, w)
        fb.call("fence_rms_norm_per_head", dx.data_ptr(), dw.data_ptr(), nh, hd, 1e-6, None)
        np.testing.assert_allclose(dx.cpu().numpy(), ref, rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("pos", [0, 1, 17, 1000, 4095, 131071])
def test_apply_rope(fb, orc, T, pos):
    rng = np.random.default_rng(pos)
    hd, nq, nkv = 128, 32, 8
    q = rng.standard_normal(nq * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    rq, rk = q.copy(), k.copy()
    orc.oracle().oracle_rope(P(rq), P(rk), hd, nq, nkv, pos, 1e6)
    dq, dk = cu(T, q), cu(T, k)
    fb.call("fence_apply_rope", dq.data_ptr(), dk.data_ptr(), hd, nq, nkv, pos, 1e6, None)
    np.testing.assert_allclose(dq.cpu().numpy(), rq, rtol=0, atol=2e-6 * 4)
    np.testing.assert_allclose(dk.cpu().numpy(), rk, rtol=0, atol=2e-6 * 4)


def test_silu_residual_softmax_convert(fb, orc, T):
    rng = np.random.default_rng(2)
    n = 17408
    g = (rng.standard_normal(n) * 4).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    ref = np.empty(n, np.float32)
    orc.oracle().oracle_silu_mul(P(ref), P(g), P(u), n)
    out = T.empty(n, device="cuda")
    dg, du = cu(T, g), cu(T, u)  # keep the inputs alive: launches are asynchronous
    fb.call("fence_silu_elementwise_mul", out.data_ptr(), dg.data_ptr(), du.data_ptr(), n, None)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-6, atol=1e-7)
    x, r = cu(T, g), cu(T, u)
    fb.call("fence_residual_add", x.data_ptr(), r.data_ptr(), n, None)
    assert np.array_equal(x.cpu().numpy(), g + u)
    s = (rng.standard_normal(151936) * 2).astype(np.float32)
    rs = s.copy()
    orc.oracle().oracle_softmax(P(rs), rs.size)
    ds = cu(T, s)
    fb.call("fence_softmax", ds.data_ptr(), s.size, None)
    np.testing.assert_allclose(ds.cpu().numpy(), rs, rtol=2e-5, atol=1e-12)
    h = T.empty(n, dtype=T.int16, device="cuda")
    fb.call("fence_f32_to_f16", h.data_ptr(), dg.data_ptr(), n, None)
    assert np.array_equal(h.cpu().numpy().view(np.uint16), g.astype(np.float16).view(np.uint16))
    back = T.empty(n, device="cuda")
    fb.call("fence_half_to_float", back.data_ptr(), h.data_ptr(), n, None)
    assert np.array_equal(back.cpu().numpy(), g.astype(np.float16).astype(np.float32))


def test_store_kv(fb, T):
    kv_dim, max_ctx = 1024, 64
    kc = T.zeros(max_ctx * kv_dim, dtype=T.int16, device="cuda")
    vc = T.zeros(max_ctx * kv_dim, dtype=T.int16, device="cuda")
    k = np.random.default_rng(3).standard_normal(kv_dim).astype(np.float32)
    v = np.random.default_rng(4).standard_normal(kv_dim).astype(np.float32)
    dk, dv = cu(T, k), cu(T, v)
    fb.call("fence_store_kv", kc.data_ptr(), vc.data_ptr(), dk.data_ptr(), dv.data_ptr(), 63, kv_dim, max_ctx, None)
    kh = kc.cpu().numpy().view(np.uint16).reshape(max_ctx, kv_dim)
    assert np.array_equal(kh[63], k.astype(np.float16).view(np.uint16)) and not kh[:63].any()
    assert np.array_equal(vc.cpu().numpy().view(np.uint16).reshape(max_ctx, kv_dim)[63],
                          v.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("nq,nkv,hd,seq,max_ctx", [
    (32, 8, 128, 1, 4096), (32, 8, 128, 129, 4096), (32, 8, 128, 4000, 4096), (40, 8, 128, 517, 1024),
    (8, 8, 64, 300, 300), (16, 2, 256, 77, 77), (32, 8, 128, 140, 140), (4, 4, 128, 4096, 4096)])
def test_gqa_attention(fb, orc, T, nq, nkv, hd, seq, max_ctx):
    rng = np.random.default_rng(seq)
    kvd = nkv * hd
    q = rng.standard_normal(nq * hd).astype(np.float32)
    kc = (rng.standard_normal((max_ctx, kvd)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((max_ctx, kvd)).astype(np.float16)
    ref = np.empty(nq * hd, np.float32)
    orc.oracle().oracle_attention(P(ref), P(q), P(kc.view(np.uint16)), P(vc.view(np.uint16)), 0, kvd, hd, hd, nq,
                                  nkv, seq)
    out = T.empty(nq * hd, device="cuda")
    score = T.full((nq * max_ctx,), float("nan"), device="cuda")
    dk, dv, dq = cu(T, kc.view(np.int16)), cu(T, vc.view(np.int16)), cu(T, q)
    fb.call("fence_gqa_attention", out.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), hd, nq, nkv,
            seq, max_ctx, score.data_ptr(), None)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=2e-5)


def test_argmax_reference_order(fb, orc, T):
    rng = np.random.default_rng(6)
    cases = [rng.integers(0, 3, n).astype(np.float32) for n in [1, 255, 256, 1000, 151936]]
    x = np.zeros(1000, np.float32)
    x[[300, 5]] = 5
    cases.append(x)
    x = np.zeros(600, np.float32)
    x[7] = np.nan
    x[9] = 1
    cases.append(x)
    cases.append(np.full(300, -np.inf, np.float32))
    cases.append(rng.standard_normal(128256).astype(np.float32))
    res = T.zeros(1, dtype=T.int32, device="cuda")
    for x in cases:
        dx = cu(T, x)
        fb.call("fence_argmax", dx.data_ptr(), res.data_ptr(), x.size, None)
        assert int(res.item()) == orc.argmax(x)
