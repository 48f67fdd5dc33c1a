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


@pytest.mark.parametrize("size", [1, 2, 4, 8])
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
        assert (p["o_cols"][1] - p["o_cols"][0]) % 64 == 0 and (p["down_cols"][1] - p["down_cols"][0]) % 64 == 0
        assert p["q_heads"] * size == 40 and p["kv_heads"] * size == 8


def test_config3_eight_ranks_cut_super_blocks():
    """At 8 ranks a rank holds 640 o_proj columns (2.5 Q6_K super-blocks) and 2176 down columns
    (8.5): the odd ranks start in the middle of a super-block (its d goes to both neighbours)."""
    p1 = tp().shard_plan(**CFG3, rank=1, size=8)
    assert p1["o_cols"] == (640, 1280) and (640 // 64) % 4 == 2
    assert p1["down_cols"] == (2176, 4352) and (2176 // 64) % 4 == 2
    with pytest.raises(ValueError, match="64-input items"):
        tp().shard_plan(n_heads=8, n_kv_heads=8, head_dim=32, ff_dim=1024, vocab=100, rank=0, size=8)


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
