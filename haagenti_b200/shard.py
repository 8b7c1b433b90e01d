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


# ------------------------------------------------------------------ models

# Decoder architectures of the whole-model decode (shapes as the reference's
# safetensors_to_int4_hct example sees a checkpoint: [out, in] row-major, the
# RMSNorm weights 1-D).
ARCHS = {
    "llama2-70b": dict(layers=80, hidden=8192, intermediate=28672, heads=64, kv_heads=8,
                       head_dim=128, vocab=32000),
    "llama3-8b": dict(layers=32, hidden=4096, intermediate=14336, heads=32, kv_heads=8,
                      head_dim=128, vocab=128256),
}


def model_units(arch) -> list[tuple[str, tuple, int]]:
    """Every tensor of the model as (name, shape, layer); layer -1 for the
    embedding, the final norm and lm_head.  ``arch`` names an entry of ARCHS
    or is a dict with the same keys."""
    a = ARCHS[arch] if isinstance(arch, str) else arch
    h, i, q = a["hidden"], a["intermediate"], a["heads"] * a["head_dim"]
    kv = a["kv_heads"] * a["head_dim"]
    out = [("model.embed_tokens.weight", (a["vocab"], h), -1)]
    for l in range(a["layers"]):
        p = f"model.layers.{l}."
        out += [(p + "self_attn.q_proj.weight", (q, h), l),
                (p + "self_attn.k_proj.weight", (kv, h), l),
                (p + "self_attn.v_proj.weight", (kv, h), l),
                (p + "self_attn.o_proj.weight", (h, q), l),
                (p + "mlp.gate_proj.weight", (i, h), l),
                (p + "mlp.up_proj.weight", (i, h), l),
                (p + "mlp.down_proj.weight", (h, i), l),
                (p + "input_layernorm.weight", (h,), l),
                (p + "post_attention_layernorm.weight", (h,), l)]
    out += [("model.norm.weight", (h,), -1), ("lm_head.weight", (a["vocab"], h), -1)]
    return out


def rank_units(arch, world: int, rank: int) -> list[tuple[str, tuple, int]]:
    """This rank's tensors: its contiguous layer range (layer_ranges) plus the
    non-layer tensors placed by element count (assign_units), in model order."""
    units = model_units(arch)
    a = ARCHS[arch] if isinstance(arch, str) else arch
    layers = set(layer_ranges(a["layers"], world)[rank])
    extra = {n: float(_numel(s)) for n, s, l in units if l < 0}
    # the layer ranges already load the ranks: count them in before placing the rest
    mine_extra = set(_assign_with_base(extra, units, world)[rank])
    return [u for u in units if (u[2] in layers) or (u[2] < 0 and u[0] in mine_extra)]


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def _assign_with_base(extra: dict, units, world: int) -> list[list]:
    """assign_units for the non-layer tensors, starting from each rank's layer load."""
    arch_layers = max(l for _, _, l in units) + 1
    load = [0.0] * world
    for r, rng in enumerate(layer_ranges(arch_layers, world)):
        load[r] = float(sum(_numel(s) for _, s, l in units if l in rng))
    out: list[list] = [[] for _ in range(world)]
    for name, cost in sorted(extra.items(), key=lambda kv: (-kv[1], str(kv[0]))):
        r = min(range(world), key=lambda i: (load[i], i))
        out[r].append(name)
        load[r] += cost
    return out
