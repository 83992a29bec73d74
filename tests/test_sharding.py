"""Multi-GPU host logic on CPU: layer sharding over ranks (no data-path
collective), the work queue and gather, and the max-over-ranks timing reduction,
run as gloo ranks."""

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


# ---------------------------------------------------------------- row sharding of one layer
def test_row_slices_partition_the_rows():
    for rows in (0, 1, 7, 4096, 12289):
        for world in (1, 2, 3, 8):
            sl = [S.row_slice(rows, r, world) for r in range(world)]
            assert sl[0][0] == 0 and sl[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))
            assert max(b - a for a, b in sl) - min(b - a for a, b in sl) <= 1
    with pytest.raises(ValueError):
        S.row_slice(8, 2, 2)


def _row_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows = 7
        full = torch.arange(rows * 3, dtype=torch.float32).reshape(rows, 3)
        codes = (torch.arange(rows * 5) % 16 - 8).to(torch.int8).reshape(rows, 5)
        r0, r1 = S.row_slice(rows, rank, world)
        g = S.gather_rows(full[r0:r1].clone(), rows)
        gc = S.gather_rows(codes[r0:r1].clone(), rows)
        sq, mx = S.reduce_row_stats(torch.tensor(1.5 + rank, dtype=torch.float64),
                                    torch.tensor(float(rank), dtype=torch.float32))
        q.put((rank, torch.equal(g, full), torch.equal(gc, codes), sq, mx))
    finally:
        torch.distributed.destroy_process_group()


def test_two_gloo_ranks_gather_row_slices_and_reduce_stats():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_f, ok_c, sq, mx in res:
        assert ok_f and ok_c
        assert sq == 1.5 + 2.5 and mx == 1.0


def test_row_sharded_validates_without_a_gpu():
    W = torch.zeros(4, 8)
    with pytest.raises(ValueError):
        S.gptq_quantize_layer_row_sharded(W, torch.zeros(2, 8, 8))
    with pytest.raises(ValueError):
        S.gptq_quantize_layer_row_sharded(W, torch.eye(8), int_bits=3)
    with pytest.raises(ValueError):
        S.gptq_quantize_layer_row_sharded(W, torch.eye(8), src=1)


def _fail_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60))
    out = []
    try:
        # a source rank that raises: every rank raises, none waits
        def boom():
            raise ValueError("inverse failed here")
        try:
            S.run_on_source(boom, 0, device="cpu")
            out.append("no error")
        except ValueError as e:
            out.append(("ValueError", str(e)))
        except RuntimeError as e:
            out.append(("RuntimeError", str(e)))
        # a source rank that succeeds: every rank gets its code
        out.append(S.run_on_source(lambda: (2, "payload"), 1, device="cpu")[0])
        # a NaN max error on one rank stays NaN after the reduction
        sq, mx = S.reduce_row_stats(torch.tensor(1.0, dtype=torch.float64),
                                    torch.tensor(float("nan") if rank == 1 else 3.0))
        out.append((sq, mx != mx))
        q.put((rank, out))
    finally:
        torch.distributed.destroy_process_group()


def test_two_gloo_ranks_source_failure_and_nan_stats():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[0][0] == ("ValueError", "inverse failed here")
    assert res[1][0][0] == "RuntimeError"
    for r in (0, 1):
        assert res[r][1] == 2
        assert res[r][2] == (2.0, True)
    assert all(p.exitcode == 0 for p in procs)


def _queue_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60))
    try:
        costs = [float(c) for c in (5, 1, 9, 3, 7, 2, 8)]
        order = S.longest_first(costs)
        wq = S.WorkQueue(order, "t0")
        taken = []
        while True:
            i = wq.take()
            if i is None:
                break
            taken.append(i)
        # each rank "quantizes" its layers: outputs derived from the index
        res = {i: {"packed": torch.full((2, 3), i, dtype=torch.uint8), "scales": torch.full((2, 1), float(i)),
                   "zero_points": None, "stats": torch.tensor([i, 0.0, 0.0], dtype=torch.float64)} for i in taken}

        def specs(i):
            return {"packed": ((2, 3), torch.uint8), "scales": ((2, 1), torch.float32), "zero_points": (None, None),
                    "stats": ((3,), torch.float64)}
        got = S.gather_results(res, len(costs), specs, dst=0)
        ok = rank != 0 or (sorted(got) == list(range(len(costs))) and all(
            int(got[i]["packed"][1, 2]) == i and float(got[i]["scales"][0, 0]) == i and got[i]["zero_points"] is None
            and float(got[i]["stats"][0]) == i for i in got))
        q.put((rank, taken, ok))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_work_queue_and_gather(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_queue_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    taken = [r[1] for r in res]
    flat = [i for t in taken for i in t]
    assert len(flat) == len(set(flat)) and sorted(flat) == list(range(7))  # every layer exactly once
    assert all(r[2] for r in res)
    # each rank takes in longest-first order
    costs = [5, 1, 9, 3, 7, 2, 8]
    for t in taken:
        assert [costs[i] for i in t] == sorted((costs[i] for i in t), reverse=True)


def test_work_queue_without_a_process_group():
    wq = S.WorkQueue([2, 0, 1], "local")
    assert [wq.take(), wq.take(), wq.take(), wq.take()] == [2, 0, 1, None]
