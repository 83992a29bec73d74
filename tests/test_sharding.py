"""Multi-GPU host logic on CPU: layer sharding over ranks (no data-path
collective) and the max-over-ranks timing reduction, run as two gloo ranks."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from int_crush_converter_b200 import sharding as S

# a DiT-like model: 28 blocks of qkv/proj/mlp_up/mlp_down
SHAPES = [(12288, 4096), (4096, 4096), (16384, 4096), (4096, 16384)] * 28


def test_shard_covers_every_layer_once():
    for world in (1, 2, 3, 4, 8):
        table = S.shard_layers([S.layer_cost(m, n) for m, n in SHAPES], world)
        flat = sorted(i for idx in table for i in idx)
        assert flat == list(range(len(SHAPES)))
        loads = [sum(S.layer_cost(*SHAPES[i]) for i in idx) for idx in table]
        # longest-first balance: within one mlp_down of perfect
        assert max(loads) - min(loads) <= S.layer_cost(4096, 16384) + 1


def test_shard_is_deterministic_and_validates():
    a = S.shard_layers([3.0, 1.0, 2.0, 2.0], 2)
    assert a == S.shard_layers([3.0, 1.0, 2.0, 2.0], 2) == [[0, 1], [2, 3]]
    with pytest.raises(ValueError):
        S.shard_layers([1.0], 0)
    with pytest.raises(ValueError):
        S.my_layers([(4, 4)], 2, 2)
    own = S.owners(["a", "b"], [(8, 8), (8, 8)], 2)
    assert sorted(own.values()) == [0, 1]


def test_max_over_ranks_without_group():
    assert S.max_over_ranks(3.5) == 3.5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = S.my_layers(SHAPES, rank, world)
        # every rank derives the same table without communication; check it against the others
        gathered = [None] * world
        torch.distributed.all_gather_object(gathered, mine)
        t = S.max_over_ranks(10.0 + rank)
        q.put((rank, mine, gathered, t))
    finally:
        torch.distributed.destroy_process_group()


def test_two_gloo_ranks_shard_disjointly_and_time_with_max():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    mine0, mine1 = res[0][1], res[1][1]
    assert not set(mine0) & set(mine1)
    assert sorted(mine0 + mine1) == list(range(len(SHAPES)))
    for r in res:
        assert r[2] == [mine0, mine1]
        assert r[3] == 11.0
