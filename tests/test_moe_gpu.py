"""Sparse mixture-of-experts decode (config 4's Mixtral shape; the reference has no expert tensors,
so the checker is the CPU oracle's restatement of Mixtral routing over the reference's per-op math,
oracle/fence_oracle.c moe_ffn, itself pinned to transformers' Mixtral sparse-MoE block by
tests/test_moe_hf_pin.py).

One GPU: the step kernel routes in every CTA (fp32 router, top-k, softmax over the chosen logits)
and streams only the routed experts' tiles. Tensor parallel: every rank holds a slice of every
expert (moe_ep = 0) or whole experts (moe_ep = 1, expert parallel); the down partial rows of the
routed slots are summed over the ranks inside the step kernel.

A router near-tie (oracle gap between the last chosen and the best unchosen expert below
ROUTE_GAP) lets rounding pick either expert, and the choice then also changes the KV cache of the
later layers: comparison stops at the first such step (the tests require enough steps before it).
"""
import os
import socket

import numpy as np
import pytest

from conftest import load_pkg

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-3  # engine vs fp64 oracle on the tiny models, as for the dense FFN
ROUTE_GAP = 1e-3   # router-logit gap below which the choice is a numerical tie
STEPS = 24
MIN_STEPS = 12


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(n=STEPS, vocab=2048, seed=3):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def _oracle_run(orc, path, tokens):
    """Teacher-forced oracle logits, the experts it chose and the steps before the first router tie."""
    ora = orc.OracleModel(path, max_ctx=256, kv_bf16=False, threads=8)
    assert ora.n_experts > 0
    logits, sels, ok = [], [], len(tokens)
    for pos, t in enumerate(tokens):
        logits.append(ora.forward(t, pos))
        sel, gap = ora.last_route()
        sels.append(sel.copy())
        if gap < ROUTE_GAP and ok == len(tokens):
            ok = pos
    ora.close()
    return np.stack(logits), sels, ok


@pytest.fixture(scope="module")
def moe_models(fb, tmp_path_factory):
    d = tmp_path_factory.mktemp("moe")
    out = {}
    for cfg in ("tiny-moe", "tiny-moe-q8"):
        for k in (1, 2):
            p = str(d / f"{cfg}-top{k}.gguf")
            fb.synth_write(p, cfg, seed=43, n_experts_used=k)
            out[(cfg, k)] = p
    return out


@pytest.mark.parametrize("cfg", ["tiny-moe", "tiny-moe-q8"])
@pytest.mark.parametrize("k", [1, 2])
def test_moe_matches_oracle(fb, orc, moe_models, cfg, k):
    path = moe_models[(cfg, k)]
    toks = _tokens()
    ref, sels, n_ok = _oracle_run(orc, path, toks)
    assert n_ok >= MIN_STEPS, f"router tie at step {n_ok}: pick another seed"
    m = fb.Model(path, max_ctx=256)
    assert m.config.n_experts == (4 if cfg == "tiny-moe" else 8) and m.config.n_experts_used == k
    got, ids = [], []
    for pos, t in enumerate(toks):
        d = m.forward(t, pos)
        got.append(m.logits())
        ids.append(m.sample_greedy(d))
    m.close()
    got = np.stack(got)
    err = np.abs(got[:n_ok].astype(np.float64) - ref[:n_ok]).max(axis=1)
    assert err.max() < LOGIT_ATOL, err
    for s in range(n_ok):
        top2 = np.sort(ref[s])[-2:]
        if top2[1] - top2[0] > 2 * LOGIT_ATOL:
            assert ids[s] == orc.argmax(ref[s]), s


def test_moe_routing_reaches_every_expert(orc, moe_models):
    """The seeded router spreads the tokens over all experts (so the tests above cover every
    expert's tiles, not only one or two)."""
    _, sels, n_ok = _oracle_run(orc, moe_models[("tiny-moe-q8", 2)], _tokens(48, seed=5))
    seen = set(int(e) for s in sels[:n_ok] for e in s.ravel())
    assert seen == set(range(8)), seen


def test_moe_needs_the_step_kernel(fb, moe_models):
    with pytest.raises(fb.FenceError, match="step kernel"):
        fb.Model(moe_models[("tiny-moe", 2)], max_ctx=64, step_kernel=False)


def test_moe_graph_and_eager_are_identical(fb, moe_models):
    p = moe_models[("tiny-moe", 2)]
    outs = []
    for graph in (True, False):
        m = fb.Model(p, max_ctx=64, use_graph=graph)
        for pos, t in enumerate([5, 9, 1000, 3, 77, 2047, 0]):
            m.forward(t, pos)
        outs.append(m.logits())
        m.close()
    assert np.array_equal(outs[0], outs[1])


def test_moe_decode_greedy_matches_stepwise(fb, moe_models):
    p = moe_models[("tiny-moe-q8", 2)]
    m = fb.Model(p, max_ctx=128)
    prompt = [11, 22, 33, 44]
    for pos, t in enumerate(prompt[:-1]):
        m.forward(t, pos)
    dev_ids = m.decode_greedy(prompt[-1], len(prompt) - 1, 20)
    m.close()
    m = fb.Model(p, max_ctx=128)
    ids, tok = [], None
    for pos, t in enumerate(prompt):
        d = m.forward(t, pos)
        tok = m.sample_greedy(d)
    ids.append(tok)
    for pos in range(len(prompt), len(prompt) + 19):
        d = m.forward(tok, pos)
        tok = m.sample_greedy(d)
        ids.append(tok)
    m.close()
    assert list(dev_ids) == ids


# ---------------------------------------------------------------- tensor / expert parallel
def _rank(rank, world, port, path, out_dir, ep):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        fb = load_pkg()
        import fence_b200.tp as tp
        m = fb.Model(path, max_ctx=256, device=rank, tp_rank=rank, tp_size=world, moe_ep=ep)
        tp.connect(m)
        logits, ids = [], []
        for pos, t in enumerate(_tokens()):
            d = m.forward(t, pos)
            logits.append(m.logits())
            ids.append(m.sample_greedy(d))
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), logits=np.stack(logits), ids=np.array(ids))
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("ep", [False, True])
def test_moe_parallel_matches_oracle(fb, orc, moe_models, world, ep):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    path = moe_models[("tiny-moe-q8" if ep else "tiny-moe", 2)]
    d = os.path.join(os.path.dirname(path), f"par{world}{int(ep)}")
    os.makedirs(d, exist_ok=True)
    mp.spawn(_rank, args=(world, _free_port(), path, d, ep), nprocs=world, join=True)
    r = [np.load(os.path.join(d, f"r{k}.npz")) for k in range(world)]
    for k in range(1, world):
        assert (r[k]["ids"] == r[0]["ids"]).all()
    got = np.concatenate([r[k]["logits"] for k in range(world)], axis=1)
    ref, _, n_ok = _oracle_run(orc, path, _tokens())
    assert n_ok >= MIN_STEPS
    np.testing.assert_allclose(got[:n_ok], ref[:n_ok], rtol=0, atol=LOGIT_ATOL)
