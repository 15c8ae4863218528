"""Tensor-parallel sharding and collectives on world-size-2 gloo CPU ranks.

* Column shards of an AWQ linear, gathered along the last dimension, and row
  shards, all-reduced, reproduce the full linear (the reference's
  tests/test_awq.py:204-234 property, here across real processes); the
  uneven vocab-style gather pads and trims like distributed.py:199-224.
* A rank that leaves before a collective makes the survivor's collective fail
  within the process-group timeout instead of hanging (host-side failure
  detection; no GPU involved).
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from light_vllm_b200.collectives import (
    TensorParallelCollectives,
    awq_column_shard,
    awq_row_shard,
    partition_dimension,
)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank: int, world: int, port: int, results) -> None:
    import numpy as np

    from oracle import awq as oawq

    _init(rank, world, port, 60)
    try:
        coll = TensorParallelCollectives()
        k, n, g = 256, 192, 64
        qweight, qzeros, scales = (torch.from_numpy(a) for a in oawq.random_checkpoint(k, n, g, seed=5))
        rng = np.random.default_rng(6)
        x = torch.from_numpy(rng.standard_normal((3, k)).astype(np.float32))
        bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(torch.float16)
        full = oawq.torch_linear(x, qweight, qzeros, scales.to(torch.float16), g, None)

        col = partition_dimension(n, rank, world)
        cq, cz, cs, cb = awq_column_shard(qweight, qzeros, scales, bias, col)
        local = oawq.torch_linear(x, cq, cz, cs, g, None)
        gathered = coll.all_gather_last_dim(local, col.sizes)

        row = partition_dimension(k, rank, world)
        rq, rz, rs = awq_row_shard(qweight, qzeros, scales, g, row)
        partial = oawq.torch_linear(x[:, row.start:row.end].contiguous(), rq, rz, rs, g, None)
        reduced = coll.all_reduce_sum(partial.contiguous())

        uneven = partition_dimension(5, rank, world)
        piece = torch.arange(uneven.start, uneven.end, dtype=torch.float32).repeat(2, 1)
        uneven_gather = coll.all_gather_last_dim(piece, uneven.sizes)
        results[rank] = (
            float((gathered - full).abs().max()),
            float((reduced - full).abs().max()),
            uneven_gather.tolist(),
        )
    finally:
        torch.distributed.destroy_process_group()


def test_awq_shards_and_collectives_match_the_full_linear():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        mp.start_processes(_shard_worker, args=(world, port, results), nprocs=world, start_method="spawn")
        for rank in range(world):
            gather_err, reduce_err, uneven = results[rank]
            assert gather_err < 1e-4
            assert reduce_err < 1e-3
            assert uneven == [[0.0, 1.0, 2.0, 3.0, 4.0]] * 2


def _leaving_worker(rank: int, world: int, port: int, results) -> None:
    _init(rank, world, port, 5)
    coll = TensorParallelCollectives()
    t = torch.ones(4)
    coll.all_reduce_sum(t)  # both ranks take this step
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        coll.all_reduce_sum(torch.ones(4))
        results[rank] = "completed"
    except Exception as exc:  # the survivor must see an error, not hang
        results[rank] = type(exc).__name__


def test_a_rank_that_leaves_makes_the_next_collective_fail():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        ctx = mp.start_processes(_leaving_worker, args=(world, port, results), nprocs=world,
                                 start_method="spawn", join=False)
        while not ctx.join(timeout=60):
            pass
        assert results.get(0) not in (None, "completed")


def test_partition_and_alignment_rules():
    assert partition_dimension(5, 0, 2).sizes == (3, 2)  # reference tests/test_tensor_parallel.py:165-171
    assert partition_dimension(5, 1, 2).start == 3
    with pytest.raises(ValueError):
        partition_dimension(1, 0, 2)
    q = torch.zeros(256, 24, dtype=torch.int32)
    with pytest.raises(ValueError, match="align to 8"):
        awq_column_shard(q, q[:2], torch.zeros(2, 192), None, partition_dimension(192, 0, 5))
    with pytest.raises(ValueError, match="align to group_size"):
        awq_row_shard(q, q[:2], torch.zeros(2, 192), 128, partition_dimension(256, 0, 4))


def test_qwen2_rank_layout_matches_the_reference_shard_declarations():
    """The runner's tensor-parallel layout against the reference's declared
    checkpoint slices (tests/test_tensor_parallel.py:231-256): 4 query / 2 KV
    heads at TP=2 give 2 / 1 per rank, rank 1's vocabulary shard starts at 5;
    with 1 KV head both ranks hold the whole KV head (start 0, length 2)."""

    from light_vllm_b200.qwen2 import Qwen2Shape, RankLayout

    cfg = dict(vocab_size=10, hidden_size=8, intermediate_size=12, num_hidden_layers=1, num_attention_heads=4,
               num_key_value_heads=2, max_position_embeddings=16)
    lay = RankLayout.of(Qwen2Shape(**cfg), 1, 2)
    assert (lay.q_heads, lay.kv_heads) == (2, 1)
    assert lay.vocab_part.start == 5
    assert (lay.q_part.start, lay.q_part.local_size) == (4, 4)
    for rank in range(2):
        rep = RankLayout.of(Qwen2Shape(**dict(cfg, num_key_value_heads=1)), rank, 2)
        assert rep.kv_heads == 1
        assert (rep.kv_part.start, rep.kv_part.local_size) == (0, 2)
    with pytest.raises(ValueError, match="query heads"):
        RankLayout.of(Qwen2Shape(**dict(cfg, num_attention_heads=6, num_key_value_heads=3)), 0, 4)
