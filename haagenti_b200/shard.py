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
