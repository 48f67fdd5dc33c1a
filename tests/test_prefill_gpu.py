"""Batched prefill on the tensor cores (csrc/prefill.cu) against the token-by-token prefill of the
reference's generate (src/model/qwen3.cu:478-481), which the engine's decode step reproduces (its
parity with the reference and the oracle is tested elsewhere).

  * the tcgen05 GEMM alone (fence_gemm_f16) against torch on fp16 operands, fp32 accumulation;
  * fence_prefill of n tokens vs n fence_forward calls on the same model: the last token's logits,
    and the logits of greedy decode steps that read the K/V rows the prefill wrote, within the
    north-star logit bound (the GEMMs take fp16 activations and fp16-rounded weights where the
    decode path keeps 16-bit integer activations and exact weights).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2  # north-star bound per logit (the decode step's own bound vs the oracle is 2e-3)


@pytest.mark.parametrize("P,N,K", [(1, 16, 64), (100, 256, 128), (128, 300, 4096), (300, 1024, 512),
                                   (257, 512, 1024), (4000, 256, 256)])
def test_gemm_f16_matches_torch(fb, P, N, K):
    import torch
    g = torch.Generator(device="cpu").manual_seed(P * 7 + N + K)
    A = torch.randn(P, K, generator=g).half().cuda()
    B = (torch.randn(N, K, generator=g) * 0.05).half().cuda()
    C = torch.full((P, N), float("nan"), dtype=torch.float32, device="cuda")
    fb.call("fence_gemm_f16", A.data_ptr(), B.data_ptr(), C.data_ptr(), P, N, K, None)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().T
    err = (C - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item() + 1e-5, err


def test_gemm_f16_rejects_bad_shapes(fb):
    with pytest.raises(fb.FenceError, match="K % 64"):
        fb.call("fence_gemm_f16", 16, 16, 16, 4, 4, 48, None)


def _tokenwise(fb, path, toks, steps, kv):
    m = fb.Model(path, max_ctx=4096, kv_dtype=kv)
    d = None
    for pos, t in enumerate(toks):
        d = m.forward(t, pos)
    out = [m.logits()]
    tok = m.sample_greedy(d)
    ids = [tok]
    for i in range(steps):
        d = m.forward(tok, len(toks) + i)
        out.append(m.logits())
        tok = m.sample_greedy(d)
        ids.append(tok)
    m.close()
    return np.stack(out), ids


def _batched(fb, path, toks, ids, kv):
    """fence_prefill, then decode steps fed the token-wise run's ids (teacher forcing)."""
    m = fb.Model(path, max_ctx=4096, kv_dtype=kv)
    m.prefill(toks)
    out = [m.logits()]
    for i, tok in enumerate(ids[:-1]):
        m.forward(tok, len(toks) + i)
        out.append(m.logits())
    m.close()
    return np.stack(out)


@pytest.mark.parametrize("cfg,n,kv", [("tiny-q6k", 40, 0), ("tiny-q8", 40, 0), ("wide-q6k", 200, 0),
                                      ("wide-q8", 200, 1), ("tiny-q6k", 1, 0)])
def test_prefill_matches_tokenwise(fb, tmp_path, cfg, n, kv):
    p = str(tmp_path / f"{cfg}.gguf")
    fb.synth_write(p, cfg, seed=61)
    toks = [int(t) for t in np.random.default_rng(n).integers(0, 2048, n)]
    ref, ids = _tokenwise(fb, p, toks, 8, kv)
    got = _batched(fb, p, toks, ids, kv)
    err = np.abs(got - ref).max(axis=1)
    assert err.max() < LOGIT_ATOL, err


def test_prefill_long_prompt_in_chunks(fb, tmp_path):
    """More tokens than one chunk holds (2048), attention over many 64-position tiles, and a
    prefill that continues at pos0 > 0 after earlier tokens."""
    p = str(tmp_path / "long.gguf")
    fb.synth_write(p, "wide-q8", seed=67, n_layers=1)
    toks = [int(t) for t in np.random.default_rng(5).integers(0, 2048, 2600)]
    ref, ids = _tokenwise(fb, p, toks, 4, 0)
    m = fb.Model(p, max_ctx=4096)
    m.prefill(toks[:1000])
    m.prefill(toks[1000:], pos0=1000)
    got = [m.logits()]
    for i, tok in enumerate(ids[:-1]):
        m.forward(tok, len(toks) + i)
        got.append(m.logits())
    m.close()
    err = np.abs(np.stack(got) - ref).max(axis=1)
    assert err.max() < LOGIT_ATOL, err


def test_prefill_off_is_tokenwise_exactly(fb, tmp_path):
    """prefill=False keeps no repacked copy and runs the prompt through the decode step: the same bits
    as calling fence_forward per token."""
    p = str(tmp_path / "t.gguf")
    fb.synth_write(p, "tiny-q8", seed=71)
    toks = [3, 1, 4, 1, 5, 9, 2, 6]
    m = fb.Model(p, max_ctx=64, prefill=False)
    m.prefill(toks)
    a = m.logits()
    m.close()
    ref, _ = _tokenwise(fb, p, toks, 0, 0)
    assert np.array_equal(a, ref[0])
