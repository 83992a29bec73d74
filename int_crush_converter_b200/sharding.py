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


def owners(names: Iterable[str], shapes: Sequence[tuple[int, int]], world: int) -> dict[str, int]:
    """name -> owning rank, for gathering results on the host afterwards."""
    table = shard_layers([layer_cost(m, n) for m, n in shapes], world)
    names = list(names)
    return {names[i]: r for r, idx in enumerate(table) for i in idx}
