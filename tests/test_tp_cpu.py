"""Tensor-parallel host logic on the CPU: the shard plan (engine.cu's split restated in tp.py) and
the handle exchange between ranks over a world-size-2 gloo process group."""
import os
import socket

import pytest

from conftest import load_pkg

CFG3 = dict(n_heads=40, n_kv_heads=8, head_dim=128, ff_dim=17408, vocab=151936)  # Qwen3-14B shape


def tp():
    load_pkg()
    import fence_b200.tp as t
    return t


@pytest.mark.parametrize("size", [1, 2, 4])
def test_shards_cover_config3(size):
    t = tp()
    plans = [t.shard_plan(**CFG3, rank=r, size=size) for r in range(size)]
    for key, total in [("q_rows", 40 * 128), ("kv_rows", 8 * 128), ("ffn_rows", 17408), ("o_cols", 40 * 128),
                       ("down_cols", 17408), ("vocab_rows", 151936)]:
        pos = 0
        for p in plans:  # contiguous, in rank order, exactly covering [0, total)
            a, b = p[key]
            assert a == pos and b > a
            pos = b
        assert pos == total, key
    for p in plans:
        assert (p["o_cols"][1] - p["o_cols"][0]) % 256 == 0 and (p["down_cols"][1] - p["down_cols"][0]) % 256 == 0
        assert p["q_heads"] * size == 40 and p["kv_heads"] * size == 8


def test_config3_eight_ranks_refused():
    """640 o_proj columns per rank is 2.5 Q6_K super-blocks: the engine refuses, and so does the plan."""
    with pytest.raises(ValueError, match="whole number of quant blocks"):
        tp().shard_plan(**CFG3, rank=0, size=8)
    # the same split with Q8_0 linears (64-element blocks) is fine
    tp().shard_plan(**CFG3, rank=3, size=8, o_type=8, down_type=8)


def test_uneven_vocab_and_bad_heads():
    t = tp()
    a = t.shard_plan(8, 4, 128, 2048, 2051, 0, 2)
    b = t.shard_plan(8, 4, 128, 2048, 2051, 1, 2)
    assert a["vocab_rows"] == (0, 1026) and b["vocab_rows"] == (1026, 2051)
    with pytest.raises(ValueError):
        t.shard_plan(8, 3, 128, 2048, 2048, 0, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        t = tp()
        mine = bytes([rank]) * 64
        got = t.exchange_handles(mine)
        assert got == [bytes([r]) * 64 for r in range(world)], got
        # a model-free connect: the handles reach tp_connect in rank order
        class FakeModel:
            def tp_handle(self):
                return mine

            def tp_connect(self, handles):
                self.handles = handles

        m = FakeModel()
        t.connect(m)
        assert m.handles == got
        open(os.path.join(out_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()


def test_handle_exchange_two_ranks_gloo(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert sorted(os.listdir(tmp_path)) == ["ok0", "ok1"]
