"""The device nucleus sampler (fence_sample_nucleus_dev, the reference's
Qwen3Model::sample_nucleus, src/model/qwen3.cu:351-460, run where the logits are) against the
oracle's restatement of the reference (float arithmetic, sequential sums, full sort) with the
same explicit uniform draw u. The device sums in a tree order, so a draw is compared only where
it is stable: the top-p cumulative and u each farther than a small margin from the boundary
rounding could move them across (the oracle reports both distances)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CUT_MARGIN, U_MARGIN = 1e-5, 1e-6


@pytest.fixture(scope="module")
def T():
    import torch
    assert torch.cuda.is_available()
    return torch


def P(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def device_sample(fb, T, logits, hist, params, u):
    V = logits.size
    need = fb.lib().fence_sample_scratch_bytes(V, params["top_k"])
    assert need > 0
    dl = T.from_numpy(logits).cuda()
    dh = T.from_numpy(np.asarray(hist, np.int32)).cuda() if len(hist) else None
    scratch = T.empty(need, dtype=T.uint8, device="cuda")
    out = T.full((1,), -1, dtype=T.int32, device="cuda")
    fb.call("fence_sample_nucleus_dev", dl.data_ptr(), V, dh.data_ptr() if dh is not None else None, len(hist),
            params["temperature"], params["top_p"], params["top_k"], params["rep_penalty"], params["min_p"],
            params["dyn"], u, scratch.data_ptr(), need, out.data_ptr(), None)
    T.cuda.synchronize()
    assert np.array_equal(dl.cpu().numpy(), logits)  # the logits are not modified
    return int(out.item())


def oracle_sample(orc, logits, hist, params, u):
    h = np.asarray(hist, np.int32)
    cm, um = ctypes.c_double(), ctypes.c_double()
    i = orc.oracle().oracle_sample_nucleus(P(logits), logits.size, P(h) if h.size else None, h.size,
                                           params["temperature"], params["top_p"], params["top_k"],
                                           params["rep_penalty"], params["min_p"], params["dyn"], u,
                                           ctypes.byref(cm), ctypes.byref(um))
    return i, cm.value, um.value


DEFAULTS = dict(temperature=0.7, top_p=0.8, top_k=50, rep_penalty=1.15, min_p=0.05, dyn=1)  # the CLI defaults


@pytest.mark.parametrize("vocab", [151936, 2051])
@pytest.mark.parametrize("variant", ["defaults", "no_penalty", "no_minp_static_temp", "topk256", "topk2"])
def test_device_sampler_matches_oracle(fb, orc, T, vocab, variant):
    params = dict(DEFAULTS)
    if variant == "no_penalty":
        params["rep_penalty"] = 1.0
    elif variant == "no_minp_static_temp":
        params.update(min_p=0.0, dyn=0)
    elif variant == "topk256":
        params.update(top_k=256, top_p=0.95, min_p=0.01)
    elif variant == "topk2":
        params.update(top_k=2)
    rng = np.random.default_rng(vocab + len(variant))
    stable = agree = 0
    for trial in range(6):
        scale = [0.6, 2.0, 4.0][trial % 3]  # flat (many min-p survivors) to peaked
        logits = (rng.standard_normal(vocab) * scale).astype(np.float32)
        # history with repeats, some of them of the current best tokens (the penalty matters)
        top = np.argsort(-logits)[:20]
        hist = list(rng.integers(0, vocab, 200)) + list(rng.choice(top, 60))
        for u in (0.013, 0.37, 0.71, 0.9991):
            want, cm, um = oracle_sample(orc, logits, hist, params, u)
            got = device_sample(fb, T, logits, hist, params, u)
            assert 0 <= got < vocab
            if cm > CUT_MARGIN and um > U_MARGIN:
                stable += 1
                agree += got == want
                assert got == want, (variant, trial, u, got, want)
    assert stable >= 18, stable


def test_device_sampler_rejects(fb, T):
    V = 2051
    logits = T.zeros(V, device="cuda")
    need = fb.lib().fence_sample_scratch_bytes(V, 50)
    scratch = T.empty(need, dtype=T.uint8, device="cuda")
    out = T.zeros(1, dtype=T.int32, device="cuda")
    L = fb.lib()
    assert fb.lib().fence_sample_scratch_bytes(V, 257) == 0
    rc = L.fence_sample_nucleus_dev(logits.data_ptr(), V, None, 0, 0.7, 0.8, 300, 1.1, 0.05, 1, 0.5,
                                    scratch.data_ptr(), need, out.data_ptr(), None)
    assert rc != 0 and "top_k" in fb.last_error()
    rc = L.fence_sample_nucleus_dev(logits.data_ptr(), V, None, 0, 0.7, 0.8, 50, 1.1, 0.05, 1, 0.5,
                                    scratch.data_ptr(), need - 8, out.data_ptr(), None)
    assert rc != 0 and "scratch" in fb.last_error()


def test_engine_device_sampler_follows_host_sampler(fb, tmp_path):
    """After the same seed the engine's device path and its host path (the reference's code path)
    make the same single draw from the same generator, so they pick the same id but for rounding
    at a boundary."""
    p = str(tmp_path / "m.gguf")
    fb.synth_write(p, "tiny-q6k", seed=41)
    m = fb.Model(p, max_ctx=128)
    hist = [3, 17, 17, 99, 256, 3, 1024]
    agree = 0
    for pos, tok in enumerate([5, 77, 300, 1200, 42, 7, 1999, 64, 512, 900]):
        d = m.forward(tok, pos)
        m.set_seed(1000 + pos)
        a = m.sample_nucleus(d, hist)
        m.set_seed(1000 + pos)
        b = m.sample_nucleus_device(d, hist)
        agree += a == b
        hist.append(a)
    m.close()
    assert agree >= 9, agree
