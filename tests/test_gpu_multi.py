"""Two-GPU paths (skipped on a box with fewer than two GPUs): one layer's rows
spread over two NCCL ranks, H^-1 broadcast from rank 0, results gathered;
every rank's result equals the one-GPU layer bit for bit."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.golden import inputs as gi

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(dev):
    W = torch.from_numpy(np.ascontiguousarray(gi.weight_outlier_cols(95, 777, 768))).to(dev)
    H = torch.from_numpy(np.ascontiguousarray(gi.hessian_lognormal(96, 768, 1536))).to(dev)
    return W, H


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    # a lost peer ends the next collective with an error instead of a hang
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                         timeout=datetime.timedelta(seconds=60))
    try:
        import int_crush_converter_b200 as B
        from int_crush_converter_b200 import sharding as S
        W, H = _inputs(dev)
        got = S.gptq_quantize_layer_row_sharded(W, H)
        ref = B.gptq_quantize_layer(W, H)
        q.put((rank, torch.equal(got.quantized_W, ref.quantized_W), torch.equal(got.scales, ref.scales),
               torch.equal(got.zero_points, ref.zero_points), abs(got.mse - ref.mse) <= 1e-12 * ref.mse,
               got.max_err == ref.max_err, got.fallbacks))
    finally:
        torch.distributed.destroy_process_group()


def test_row_sharded_layer_on_two_gpus():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=300) for _ in range(world)]
    finally:
        # a worker that died leaves its peer in a collective: end both
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    for p in procs:
        assert p.exitcode == 0
    for r in res:
        assert all(r[1:6]), r
        assert r[6] == []
