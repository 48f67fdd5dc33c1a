"""Tensor-parallel bring-up of the engine over torch.distributed.

One process per GPU loads the same GGUF with ``Model(path, tp_rank=r, tp_size=n)``; the ranks then
swap the CUDA IPC handles of their exchange buffers over any process group (``exchange_handles``)
and connect (``connect``). From then on the ranks' step kernels exchange their partial rows over
NVLink inside every token step, so the host only has to call the same decode functions on every
rank in lockstep.

``shard_plan`` restates the engine's split (engine.cu, model load) for callers that want to check
a configuration before loading: q/k/v heads and gate/up rows per rank (column-parallel), o_proj
and down by input columns (row-parallel; a rank's columns must be whole quant blocks), the tied
LM head by vocabulary rows (ceil(V / n) per rank, the last rank the remainder).
"""
from __future__ import annotations

GGML_Q6_K, GGML_Q8_0 = 14, 8


def shard_plan(n_heads: int, n_kv_heads: int, head_dim: int, ff_dim: int, vocab: int, rank: int, size: int,
               o_type: int = GGML_Q6_K, down_type: int = GGML_Q6_K) -> dict:
    """Rows / columns of one rank's shard; raises ValueError where the engine refuses to load."""
    if size not in (1, 2, 4, 8) or not 0 <= rank < size:
        raise ValueError(f"rank {rank} of {size} (tp_size 1, 2, 4 or 8)")
    if n_heads % size or n_kv_heads % size or ff_dim % size:
        raise ValueError("heads / FFN rows do not split evenly")
    qd, kvd, F = n_heads * head_dim // size, n_kv_heads * head_dim // size, ff_dim // size
    if qd % 64 or F % 64:  # whole 64-input items (a Q6_K super-block may be cut between two ranks)
        raise ValueError("a rank's o_proj / down column slice is not a whole number of 64-input items")
    per = (vocab + size - 1) // size
    v0 = rank * per
    return {
        "q_rows": (rank * qd, (rank + 1) * qd),
        "kv_rows": (rank * kvd, (rank + 1) * kvd),
        "ffn_rows": (rank * F, (rank + 1) * F),
        "o_cols": (rank * qd, (rank + 1) * qd),
        "down_cols": (rank * F, (rank + 1) * F),
        "vocab_rows": (v0, min(vocab, v0 + per)),
        "q_heads": n_heads // size,
        "kv_heads": n_kv_heads // size,
    }


def exchange_handles(handle: bytes, group=None) -> list:
    """All ranks' handles in rank order (an all_gather over the group; any backend that carries
    Python objects, e.g. gloo)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


def connect(model, group=None) -> None:
    """Swaps exchange-buffer handles with the other ranks and connects ``model`` to them."""
    model.tp_connect(exchange_handles(model.tp_handle(), group))
