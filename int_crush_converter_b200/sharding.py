"""Multi-GPU layout of the per-layer quantization path.

The reference quantizes a model's linear layers one after another on one
device (pipeline.py:702-809, the per-layer loop).  Layers are independent
given their Hessians, so across GPUs the path shards with no data-path
collective: one process per GPU, each rank quantizes its own subset of the
layers on its own device, and the only communication is host-side
bookkeeping (which rank owns which layer) and, for timing, a max over ranks.

Assignment is longest-processing-time-first on the estimated cost of a layer,
M*N^2 (the GPTQ trailing updates) + N^3 (the Hessian inverse), so that the
ranks finish together even though one mlp_down layer costs as much as twenty
qkv layers.  It is deterministic: every rank computes the same table without
exchanging anything.
"""

from __future__ import annotations

from typing import Iterable, Mapping, Sequence

import torch


def layer_cost(out_features: int, in_features: int) -> float:
    """Estimated device work of one GPTQ layer [out, in]: M*N^2 + N^3."""
    m, n = float(out_features), float(in_features)
    return m * n * n + n ** 3


def shard_layers(costs: Sequence[float], world: int) -> list[list[int]]:
    """Indices of the layers each rank owns (longest first onto the least loaded rank;
    ties broken by index, so every rank computes the same table)."""
    if world < 1:
        raise ValueError(f"world size must be >= 1, got {world}")
    load = [0.0] * world
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owned[r].append(i)
        load[r] += costs[i]
    for o in owned:
        o.sort()
    return owned


def my_layers(shapes: Sequence[tuple[int, int]], rank: int, world: int) -> list[int]:
    """The indices of `shapes` ([out, in] per layer) that `rank` quantizes."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    return shard_layers([layer_cost(m, n) for m, n in shapes], world)[rank]


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """Max of a per-rank scalar (e.g. a device-event time) over the process group;
    the value itself without an initialised group."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def quantize_layers_sharded(layers: Mapping[str, tuple[torch.Tensor, torch.Tensor]], rank: int, world: int,
                            streams: int = 4, device=None, **kw) -> dict[str, dict]:
    """Quantize this rank's share of `layers` (name -> (W [out,in], H [in,in])) with
    :class:`~int_crush_converter_b200.gptq.LayerStreams` on `device`; keyword
    arguments go to :func:`~int_crush_converter_b200.gptq.quantize_gptq_layer`.
    Returns name -> result for the layers this rank owns (device tensors)."""
    from .gptq import LayerStreams
    names = list(layers)
    mine = my_layers([tuple(layers[n][0].shape) for n in names], rank, world)
    out: dict[str, dict] = {}
    pool = LayerStreams(streams, device)
    with pool:
        for i in mine:
            W, H = layers[names[i]]
            out[names[i]] = pool.submit(W, H, **kw)
    return out


def _default_store():
    """The key-value store of the initialised default process group (the rendezvous
    TCPStore under torchrun), or None without one."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return None
    from torch.distributed import distributed_c10d as c10d
    return c10d._get_default_store()


class WorkQueue:
    """Work items handed out one at a time, in a fixed order (longest first), to
    whichever rank asks next: the next index is an atomic counter in the process
    group's key-value store (``store.add``), so a rank that runs ahead takes more
    of the remaining layers (list scheduling) and a slow GPU -- these machines
    are shared -- takes fewer, instead of every rank following a precomputed
    table.  Each round of work uses its own ``key``.  Without a process group it
    is a local counter."""

    def __init__(self, order: Sequence[int], key: str, store=None):
        self.order = list(order)
        self.key = f"icq/{key}"
        self.store = store if store is not None else _default_store()
        self._local = 0

    def take(self) -> int | None:
        if self.store is None:
            i = self._local
            self._local += 1
        else:
            i = int(self.store.add(self.key, 1)) - 1
        return self.order[i] if i < len(self.order) else None


def longest_first(costs: Sequence[float]) -> list[int]:
    """Indices by descending cost (ties by index)."""
    return sorted(range(len(costs)), key=lambda i: (-costs[i], i))


def quantize_from_queue(queue: WorkQueue, fetch, pool, depth: int = 6) -> dict[int, dict]:
    """Pull layers from `queue` and issue them on `pool` (a LayerStreams) until
    the queue is empty.  ``fetch(i)`` returns (W, H, kwargs) of layer i (kwargs
    may hold ``before`` / ``then`` hooks and the layer call's keyword
    arguments).  A rank takes its next layer only while fewer than `depth` of
    its layers are unfinished on the GPU, so the queue hands the rest to ranks
    that are ahead.  Returns index -> asynchronous result for the layers this
    rank quantized."""
    inflight: list = []
    out: dict[int, dict] = {}
    while True:
        while len(inflight) >= depth:
            inflight.pop(0).synchronize()
        i = queue.take()
        if i is None:
            return out
        W, H, kw = fetch(i)
        res = pool.submit(W, H, **kw)
        out[i] = res
        inflight.append(res["done"])


def owner_table(mine: Iterable[int], n: int, device=None) -> list[int]:
    """Which rank holds each of `n` items (-1: none), from each rank's own list
    (one MAX all-reduce of an int32 vector)."""
    rank, world = _group_info(None)
    t = torch.full((n,), -1, dtype=torch.int32, device=device)
    idx = list(mine)
    if idx:
        t[torch.tensor(idx, dtype=torch.long, device=device)] = rank
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


def gather_results(results: dict[int, dict], n: int, specs, dst: int = 0,
                   keys: Sequence[str] = ("packed", "scales", "zero_points", "stats"), device=None) -> dict[int, dict]:
    """Bring every layer's outputs to rank `dst` (point-to-point sends over the
    process group: NVLink with NCCL).  ``results`` are this rank's (index ->
    dict of device tensors); ``specs(i)`` gives {key: (shape, dtype)} of layer
    i's outputs, for the receive buffers.  On `dst` returns all n layers; on
    other ranks, after their sends complete, an empty dict.  Call it after the
    results are ready on the current stream (e.g. LayerStreams.join)."""
    rank, world = _group_info(None)
    if world == 1:
        return dict(results)
    owner = owner_table(results.keys(), n, device)
    missing = [i for i, r in enumerate(owner) if r < 0]
    if missing:
        raise RuntimeError(f"gather_results: no rank holds layers {missing[:8]}")
    ops = []
    got: dict[int, dict] = {}
    if rank == dst:
        got = {i: results[i] for i in results}
        for i in range(n):
            if owner[i] == dst:
                continue
            bufs = {}
            for k in keys:
                shape, dtype = specs(i)[k]
                if shape is None:
                    bufs[k] = None
                    continue
                bufs[k] = torch.empty(shape, dtype=dtype, device=device)
                ops.append(torch.distributed.P2POp(torch.distributed.irecv, bufs[k], owner[i]))
            got[i] = bufs
    else:
        for i in sorted(results):
            for k in keys:
                if results[i].get(k) is not None:
                    ops.append(torch.distributed.P2POp(torch.distributed.isend, results[i][k].contiguous(), dst))
    if ops:
        for w in torch.distributed.batch_isend_irecv(ops):
            w.wait()
    return got if rank == dst else {}


def owners(names: Iterable[str], shapes: Sequence[tuple[int, int]], world: int) -> dict[str, int]:
    """name -> owning rank, for gathering results on the host afterwards."""
    table = shard_layers([layer_cost(m, n) for m, n in shapes], world)
    names = list(names)
    return {names[i]: r for r, idx in enumerate(table) for i in idx}


# ---------------------------------------------------------------------------
# Row sharding of one layer.  Given H^-1, GPTQ's rows are independent: the
# column loop (rounding.py:37-103) and the lazy update W[:, after] -= E Hinv
# act row by row and the scales / zero-points are per row (gptq.py:254-317).
# So one rank inverts the damped Hessian, broadcasts the H^-1 pair (NCCL over
# NVLink; 2 x 1 GiB at N = 16384), every rank runs its contiguous share of the
# rows, and the codes, scales and zero-points are all-gathered.  Results are
# identical to the one-GPU layer: each output element of the trailing-update
# GEMM sums the same K chunks in the same order whatever the row tiling.  The
# inverse itself (most of an mlp_down layer's flops) is not sharded, so this
# pays off only to balance the tail of a layer-sharded job.

def row_slice(rows: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous balanced share [r0, r1) of `rows` for `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    return rows * rank // world, rows * (rank + 1) // world


def _group_info(group) -> tuple[int, int]:
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return 0, 1
    return torch.distributed.get_rank(group), torch.distributed.get_world_size(group)


def gather_rows(local: torch.Tensor, rows: int, group=None) -> torch.Tensor:
    """All-gather each rank's row slice (``row_slice`` of `rows`) into the full
    [rows, ...] tensor on every rank (slices padded to a common size)."""
    rank, world = _group_info(group)
    if world == 1:
        return local
    pad = -(-rows // world)
    buf = torch.zeros((pad,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    torch.distributed.all_gather(parts, buf, group=group)
    out = []
    for r, p in enumerate(parts):
        r0, r1 = row_slice(rows, r, world)
        out.append(p[:r1 - r0])
    return torch.cat(out, 0)


def reduce_row_stats(sq: torch.Tensor, mx: torch.Tensor, group=None) -> tuple[float, float]:
    """Sum of the ranks' squared errors (fp64) and max of their max errors."""
    rank, world = _group_info(group)
    sq = sq.reshape(1).to(torch.float64).clone()
    mx = mx.reshape(1).to(torch.float32).clone()
    if world > 1:
        # a NaN max error on any rank stays NaN, as torch's max() on one GPU does
        # (a MAX all-reduce need not propagate NaN)
        nan = torch.isnan(mx).to(torch.int32)
        torch.distributed.all_reduce(sq, op=torch.distributed.ReduceOp.SUM, group=group)
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX, group=group)
        torch.distributed.all_reduce(nan, op=torch.distributed.ReduceOp.MAX, group=group)
        if int(nan.item()):
            mx.fill_(float("nan"))
    return float(sq.item()), float(mx.item())


def _quantize_rows(Wd: torch.Tensor, hi: torch.Tensor, lo: torch.Tensor, r0: int, r1: int, block_size: int,
                   int_bits: int, asymmetric: bool):
    """GPTQ over rows [r0, r1) of the fp32 device weight `Wd` given the H^-1
    pair: (codes int8, scale f32, zp f32 or None, sum of squared errors fp64,
    max error f32) for those rows."""
    from . import _native as nat
    from .gptq import _run_loop
    dev = Wd.device
    N = Wd.shape[1]
    qmin, qmax = (-128, 127) if int_bits == 8 else (-8, 7)
    Wl = Wd[r0:r1].contiguous()
    m = Wl.shape[0]
    scale = torch.empty(m, dtype=torch.float32, device=dev)
    zp = torch.empty(m, dtype=torch.float32, device=dev) if (int_bits == 4 or asymmetric) else None
    Q = torch.zeros(m, N, dtype=torch.int8, device=dev)
    if m == 0 or N == 0:
        z = torch.zeros((), dtype=torch.float64, device=dev)
        return Q, scale, zp, z, z.float()
    lib = nat.load()
    nat.check(lib.ic_gptq_row_params(Wl.data_ptr(), m, N, N, int_bits, int(asymmetric), scale.data_ptr(),
                                     nat.ptr(zp), nat.stream_ptr(dev)), "gptq_row_params")
    rsq, rmx = _run_loop(Wl.clone(), Wl, 0, N, hi, lo, hi.shape[1], block_size, scale, zp, qmin, qmax, Q)
    return Q, scale, zp, rsq.sum(), rmx.max()


def run_on_source(fn, src: int, group=None, device=None):
    """Run ``fn() -> (code >= 0, payload)`` on group rank `src` and broadcast its
    status before anything else: every rank returns (code, payload or None),
    and if `fn` raised on the source every rank raises (the source re-raises
    its own exception), instead of the other ranks waiting in a collective
    that never comes."""
    rank, world = _group_info(group)
    if world == 1:
        return fn()
    err, code, payload = None, -1, None
    if rank == src:
        try:
            code, payload = fn()
        except Exception as e:  # noqa: BLE001 - re-raised below on every rank
            err, code = e, -1
    g_src = torch.distributed.get_global_rank(group, src) if group is not None else src
    t = torch.tensor([code], dtype=torch.int32, device=device)
    torch.distributed.broadcast(t, g_src, group=group)
    c = int(t.item())
    if c < 0:
        if err is not None:
            raise err
        raise RuntimeError(f"row-sharded layer: the work of source rank {g_src} failed")
    return c, payload


def gptq_quantize_layer_row_sharded(W: torch.Tensor, hessian: torch.Tensor, group=None, src: int = 0,
                                    block_size: int = 128, damping: float = 0.01, int_bits: int = 4,
                                    asymmetric: bool = False):
    """:func:`~int_crush_converter_b200.gptq.gptq_quantize_layer` (gptq.py:137-417,
    dense 2-D Hessian) with the rows of one layer spread over the process
    group: rank `src` (group rank) inverts the damped Hessian on its GPU and
    broadcasts the H^-1 pair; every rank quantizes its ``row_slice``; every rank
    returns the full :class:`QuantizationResult`.  Call it on every rank with
    the same W and H.  Without an initialised process group it is the one-GPU
    layer."""
    from ._dev import back, device_of, f32, round4
    from .config import SCALE_DTYPE
    from .hessian import hessian_pair, inverse_pair
    from .types import QuantizationResult
    if int_bits not in (4, 8):
        raise ValueError(f"int_bits must be 4 or 8, got {int_bits}")
    if W.dim() != 2:
        raise ValueError(f"Expected 2D weight tensor, got {W.dim()}D")
    if not isinstance(hessian, torch.Tensor) or hessian.dim() != 2:
        raise ValueError("row sharding takes a dense 2-D Hessian")
    rank, world = _group_info(group)
    if not 0 <= src < world:
        raise ValueError(f"src {src} outside group of size {world}")
    dev = device_of(W, hessian)
    Wd = f32(W, dev)
    M, N = Wd.shape
    if tuple(hessian.shape) != (N, N):
        raise ValueError(f"Hessian shape {tuple(hessian.shape)} != ({N}, {N})")
    paths = ("cholesky", "inv", "pinv")

    def invert():
        Hd = f32(hessian, dev)
        hi, lo, n = hessian_pair(Hd, 0, dev, rotate=False)
        return paths.index(inverse_pair(hi, lo, n, damping, H_fallback=Hd)), (hi, lo)

    code, res = run_on_source(invert, src, group, dev)
    if res is None:
        hi = torch.empty(N, round4(N), dtype=torch.float32, device=dev)
        lo = torch.empty_like(hi)
    else:
        hi, lo = res
    if world > 1:
        g_src = torch.distributed.get_global_rank(group, src) if group is not None else src
        torch.distributed.broadcast(hi, g_src, group=group)
        torch.distributed.broadcast(lo, g_src, group=group)
    path = paths[code]
    r0, r1 = row_slice(M, rank, world)
    Q, scale, zp, sq, mx = _quantize_rows(Wd, hi, lo, r0, r1, block_size, int_bits, asymmetric)
    Q = gather_rows(Q, M, group)
    scale = gather_rows(scale, M, group)
    zp = gather_rows(zp, M, group) if zp is not None else None
    sq, mx = reduce_row_stats(sq, mx, group)
    mse = sq / (M * N) if M * N else 0.0
    zp8 = None if zp is None else zp.reshape(M, 1).to(torch.int8)
    return QuantizationResult(
        quantized_W=back(Q, W),
        scales=back(scale.reshape(M, 1).to(SCALE_DTYPE), W),
        zero_points=back(zp8, W),
        mse=mse,
        max_err=mx if M * N else 0.0,
        method_used="gptq_b200",
        fallbacks=[] if path == "cholesky" else [f"hessian_{path}"],
    )
