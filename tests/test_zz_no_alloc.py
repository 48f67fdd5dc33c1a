"""fence_gqa_attention_static (no counterpart in the reference): the drop-in GQA attention with its
split-context partials in a fixed per-device static array instead of the caller's score_buf.

Called through the C-ABI and compared with fence_gqa_attention (which uses a caller score_buf) and
the oracle, twice in a row per shape so the second call runs over partials the first one left in
the static array. Collected last (file name) so it also runs after every other GPU test; it passes
alone in a fresh process too.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# same bound as the score_buf entry point's test (fp32 accumulation, different summation order
# from the fp64 oracle)
RTOL, ATOL = 1e-4, 2e-5


@pytest.fixture(scope="module")
def T():
    import torch
    assert torch.cuda.is_available()
    return torch


def P(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def case(rng, nq, nkv, hd, max_ctx):
    kvd = nkv * hd
    q = rng.standard_normal(nq * hd).astype(np.float32)
    kc = (rng.standard_normal((max_ctx, kvd)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((max_ctx, kvd)).astype(np.float16)
    return q, kc, vc


@pytest.mark.parametrize("nq,nkv,hd,seq,max_ctx", [
    (32, 8, 128, 4000, 4096),   # 31 chunks: 128,960 floats of partials
    (40, 8, 128, 9000, 9000),   # 64 chunks: 332,800 floats
    (40, 8, 128, 517, 1024),    # 9 chunks
    (16, 2, 256, 77, 77),       # single chunk: direct output, scratch unused
    (8, 8, 64, 300, 300)])
def test_static_matches_score_buf_entry(fb, orc, T, nq, nkv, hd, seq, max_ctx):
    rng = np.random.default_rng(1000 + seq)
    outs = []
    for call in range(2):  # two calls in a row, different inputs
        q, kc, vc = case(rng, nq, nkv, hd, max_ctx)
        kvd = nkv * hd
        ref = np.empty(nq * hd, np.float32)
        orc.oracle().oracle_attention(P(ref), P(q), P(kc.view(np.uint16)), P(vc.view(np.uint16)), 0, kvd, hd, hd,
                                      nq, nkv, seq)
        dq = T.from_numpy(q).cuda()
        dk = T.from_numpy(kc.view(np.int16)).cuda()
        dv = T.from_numpy(vc.view(np.int16)).cuda()
        score = T.full((nq * max_ctx,), float("nan"), device="cuda")
        out_buf = T.empty(nq * hd, device="cuda")
        out_static = T.full((nq * hd,), float("nan"), device="cuda")
        fb.call("fence_gqa_attention", out_buf.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), hd, nq, nkv,
                seq, max_ctx, score.data_ptr(), None)
        fb.call("fence_gqa_attention_static", out_static.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                hd, nq, nkv, seq, max_ctx, None)
        T.cuda.synchronize()
        a, b = out_static.cpu().numpy(), out_buf.cpu().numpy()
        np.testing.assert_allclose(a, b, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(a, ref, rtol=RTOL, atol=ATOL)
        outs.append(a)
    assert not np.array_equal(outs[0], outs[1])


def test_static_rejects_oversized_request(fb, T):
    """64 query heads x 64 chunks x 130 floats = 532,480 > 524,288: rejected before any launch."""
    nq, nkv, hd, seq, max_ctx = 64, 8, 128, 8320, 8320
    dk = T.zeros(max_ctx * nkv * hd, dtype=T.int16, device="cuda")
    dq = T.zeros(nq * hd, device="cuda")
    out = T.full((nq * hd,), 7.0, device="cuda")
    rc = fb.lib().fence_gqa_attention_static(out.data_ptr(), dq.data_ptr(), dk.data_ptr(), dk.data_ptr(), hd, nq,
                                             nkv, seq, max_ctx, None)
    assert rc == -8, rc
    assert "static scratch" in fb.last_error()
    T.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
