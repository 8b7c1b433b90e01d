"""Sharding of a model's decode across GPUs (one process per GPU).

The decode has no data exchange: every tensor, and every LZ4 block in it, is
independent, so a model is split into per-rank units of work and each rank
decodes its own units into its own HBM.  The only collective is the
max-over-ranks of the timed region.

* ``layer_ranges`` -- contiguous layer ranges per rank, the
  ``PipelineParallel`` rule of ModelPartition::create_for_layers
  (crates/haagenti-distributed/src/partition.rs:114-125): ``ceil(L / N)``
  layers per rank, the last ranks possibly short or empty.
* ``assign_units`` -- non-layer tensors (embeddings, lm_head, norms) placed
  by decode cost: largest first onto the least-loaded rank.
* ``max_over_ranks`` -- the job's elapsed time (max over ranks) through
  whatever process group is initialised (NCCL on GPUs, gloo on CPU).
* ``replicate_units`` -- the optional replicated-weights mode: after each
  rank has decoded its own units, they are exchanged so that every rank
  holds the whole model (all-gathers of equal-shaped units, broadcasts for
  the rest; NCCL over NVLink on GPUs).  It is not part of the decode and is
  timed apart from it.
"""
from __future__ import annotations


def layer_ranges(total_layers: int, world: int) -> list[range]:
    """Layer range of every rank (partition.rs:114-125 with num_stages = world).

    The reference returns ``(start, end)`` pairs whose ``start`` may exceed
    ``end`` for trailing stages when the layers run out; both mean an empty
    range here.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    if total_layers < 0:
        raise ValueError("total_layers must be non-negative")
    per = -(-total_layers // world) if total_layers else 0
    out = []
    for i in range(world):
        start = i * per
        end = min((i + 1) * per, total_layers)
        out.append(range(start, max(start, end)))
    return out


def assign_units(costs: dict, world: int) -> list[list]:
    """Greedy longest-processing-time placement of named units by cost.

    Returns one list of unit names per rank; ties go to the lower rank and
    units of equal cost keep their name order, so every rank computes the
    same assignment without communicating.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    load = [0.0] * world
    out: list[list] = [[] for _ in range(world)]
    for name, cost in sorted(costs.items(), key=lambda kv: (-kv[1], str(kv[0]))):
        r = min(range(world), key=lambda i: (load[i], i))
        out[r].append(name)
        load[r] += float(cost)
    return out


def max_over_ranks(value: float, device=None) -> float:
    """Max of ``value`` over the ranks of the default process group (the
    value itself when no group is initialised)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def replicate_units(units: dict, owner: dict, specs: dict) -> dict:
    """Every rank's copy of every unit.

    ``units`` holds this rank's decoded tensors by name; ``owner`` maps every
    unit name to the rank that decoded it; ``specs`` maps every name to its
    ``(shape, dtype, device)``.  Units of one spec with one owner per rank
    travel together in an all-gather (every rank sends and receives at
    once, so both directions of each link carry data); the remaining units
    are broadcast from their owner.  The rounds are built in a fixed order
    from ``owner`` and ``specs`` alone, the same on every rank.  Without an
    initialised group of more than one rank, ``units`` is returned as it is.
    """
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return dict(units)
    rank, world = dist.get_rank(), dist.get_world_size()

    def key(spec):
        shape, dtype, device = spec
        return (tuple(shape), str(dtype), str(device))

    # per spec, each rank's units in name order
    queues: dict = {}
    for name in sorted(owner, key=str):
        q = queues.setdefault(key(specs[name]), [[] for _ in range(world)])
        q[owner[name]].append(name)
    out = {}
    for k in sorted(queues, key=str):
        q = queues[k]
        while all(q):  # one unit from every rank: an all-gather round
            names = [q[r].pop(0) for r in range(world)]
            shape, dtype, device = specs[names[0]]
            buf = torch.empty((world,) + tuple(shape), dtype=dtype, device=device)
            mine = units[names[rank]].contiguous()
            if dist.get_backend() == "nccl":  # straight into one buffer, no copy-out
                dist.all_gather_into_tensor(buf, mine)
            else:
                dist.all_gather(list(buf.unbind(0)), mine)
            for r, n in enumerate(names):
                out[n] = buf[r]
        for r in range(world):  # the rest, one broadcast each
            for n in q[r]:
                shape, dtype, device = specs[n]
                t = units[n] if r == rank else torch.empty(shape, dtype=dtype, device=device)
                dist.broadcast(t, src=r)
                out[n] = t
    return out
