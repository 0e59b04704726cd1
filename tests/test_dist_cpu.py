"""Query-sharded attention host logic on CPU ranks (torch.distributed gloo, world size 2).

The GPU path (hi3d_b200.dist) splits the query rows of each object over ranks and all-gathers
the token-major K/V shards; softmax rows never cross ranks, so local queries against the
gathered keys must reproduce the unsharded attention exactly (up to fp summation order).
Failure handling is tested here too: a rank that dies before a collective makes the others'
collective fail within the process-group timeout instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    sys.path.insert(0, os.path.join(REPO, "hi3dv1.0-mlx_b200"))
    sys.path.insert(0, REPO)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _sharded_attention(rank, world, port):
    _init(rank, world, port)
    from hi3d_b200.dist import gather_rows, shard_slice
    from oracle import ops

    rng = np.random.default_rng(0)
    t, h, d = 96, 2, 16
    q, k, v = (rng.standard_normal((t, h, d)).astype(np.float32) for _ in range(3))
    rows = shard_slice(t, rank, world)
    k_all = gather_rows(torch.from_numpy(k[rows]))
    v_all = gather_rows(torch.from_numpy(v[rows]))
    assert torch.equal(k_all, torch.from_numpy(k)) and torch.equal(v_all, torch.from_numpy(v))
    local = ops.attention_varlen(q[rows], k_all.numpy(), v_all.numpy(), [0, t // world], [0, t], d ** -0.5)
    out = gather_rows(torch.from_numpy(local))
    full = ops.attention_varlen(q, k, v, [0, t], [0, t], d ** -0.5)
    np.testing.assert_allclose(out.numpy(), full, rtol=1e-12, atol=1e-12)
    dist.barrier()
    dist.destroy_process_group()


def _dying_rank(rank, world, port):
    _init(rank, world, port, timeout_s=5)
    from hi3d_b200.dist import gather_rows

    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    with pytest.raises(RuntimeError):
        gather_rows(torch.ones(4, 2))  # the peer never joins: fails within the timeout
    os._exit(0)


def _object_groups(rank, world, port):
    """cfg4's object-aware sharding: 4 ranks over 2 objects pair up; over 4 objects, each rank
    owns one object and needs no exchange."""
    _init(rank, world, port)
    from hi3d_b200.dist import gather_rows, object_group

    assert object_group(4) is None
    sub = object_group(2)
    assert dist.get_world_size(sub) == 2
    got = gather_rows(torch.tensor([[float(rank)]]), group=sub)
    mate = rank ^ 1
    assert got.flatten().tolist() == [float(min(rank, mate)), float(max(rank, mate))]
    with pytest.raises(ValueError):
        object_group(3)
    dist.barrier()
    dist.destroy_process_group()


def _kv_gather_in_place(rank, world, port):
    """Each rank writes its slice into its own rows of the gather buffers; the in-place gather
    fills the other ranks' rows in rank order and leaves the own rows as they were."""
    _init(rank, world, port)
    from hi3d_b200.dist import gather_kv, kv_gather_buffers, own_rows

    t = 3
    k_all, v_all = kv_gather_buffers(t, 2, 4, torch.float32, "cpu")
    own_rows(k_all)[0].copy_(torch.full((t, 2, 4), float(rank)))
    own_rows(v_all)[0].copy_(torch.full((t, 2, 4), float(100 + rank)))
    gather_kv(k_all, v_all)
    for r in range(world):
        assert torch.equal(k_all[r * t:(r + 1) * t], torch.full((t, 2, 4), float(r)))
        assert torch.equal(v_all[r * t:(r + 1) * t], torch.full((t, 2, 4), float(100 + r)))
    dist.barrier()
    dist.destroy_process_group()


def test_kv_gather_in_place_fills_every_rank_slot():
    mp.spawn(_kv_gather_in_place, args=(4, _free_port()), nprocs=4, join=True)


def test_object_groups_pair_the_ranks_of_one_object():
    mp.spawn(_object_groups, args=(4, _free_port()), nprocs=4, join=True)


def test_query_sharded_attention_matches_unsharded():
    mp.spawn(_sharded_attention, args=(2, _free_port()), nprocs=2, join=True)


def test_shard_slice():
    sys.path.insert(0, os.path.join(REPO, "hi3dv1.0-mlx_b200"))
    from hi3d_b200.dist import shard_slice

    assert [shard_slice(32768, r, 4) for r in range(4)] == [slice(0, 8192), slice(8192, 16384),
                                                           slice(16384, 24576), slice(24576, 32768)]
    with pytest.raises(ValueError):
        shard_slice(10, 0, 3)


def test_auto_transport_follows_the_measurements():
    """Peer stores at 2 ranks, multicast stores above when the device offers NVLink multicast,
    the NCCL all-gather otherwise (a CPU device has none); unknown transports are refused."""
    sys.path.insert(0, os.path.join(REPO, "hi3dv1.0-mlx_b200"))
    from hi3d_b200.dist import ShardedBlockStack, auto_transport

    assert auto_transport(2) == "peer"
    assert auto_transport(4) == "multicast" and auto_transport(8) == "multicast"
    assert auto_transport(8, "cpu") == "nccl"
    with pytest.raises(ValueError):
        ShardedBlockStack([], 4, transport="ring")


def test_dead_rank_fails_collective_in_bounded_time():
    import time

    t0 = time.time()
    mp.spawn(_dying_rank, args=(2, _free_port()), nprocs=2, join=True)
    assert time.time() - t0 < 120
