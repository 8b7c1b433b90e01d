"""Multi-process sharding logic on CPU: world-size-2 gloo ranks on 127.0.0.1."""
import os
import socket

import pytest

from haagenti_b200 import shard


def _ref_partition(total, stages):
    """partition.rs:114-125, written out as the reference computes it."""
    per = -(-total // stages)
    return [(i * per, min((i + 1) * per, total)) for i in range(stages)]


@pytest.mark.parametrize("total,world", [(80, 8), (80, 3), (32, 1), (32, 5), (10, 8), (0, 2),
                                         (7, 7), (1, 4)])
def test_layer_ranges_follow_reference_partition(total, world):
    got = shard.layer_ranges(total, world)
    ref = _ref_partition(total, world)
    assert len(got) == world
    for r, (s, e) in zip(got, ref):
        assert list(r) == list(range(s, e))  # start > end in the reference = empty
    covered = [i for r in got for i in r]
    assert covered == list(range(total))


def test_assign_units_balances_and_is_deterministic():
    costs = {"embed": 1050.0, "lm_head": 1050.0, "norm0": 1.0, "norm1": 1.0, "final_norm": 1.0}
    a = shard.assign_units(costs, 2)
    assert a == shard.assign_units(dict(reversed(list(costs.items()))), 2)
    assert sorted(n for r in a for n in r) == sorted(costs)
    assert {"embed", "lm_head"} - set(a[0]) and {"embed", "lm_head"} - set(a[1])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        mine = list(shard.layer_ranges(80, world)[rank])
        every = [None] * world
        dist.all_gather_object(every, mine)
        tmax = shard.max_over_ranks(10.0 + rank)
        units = shard.assign_units({"embed": 3.0, "lm_head": 3.0, "norm": 1.0}, world)
        all_units = [None] * world
        dist.all_gather_object(all_units, units)
        q.put((rank, every, tmax, all_units))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_without_overlap():
    import torch.multiprocessing as mp

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
    for rank, every, tmax, all_units in res:
        # every rank sees the same disjoint cover of the 80 layers
        flat = [i for r in every for i in r]
        assert sorted(flat) == list(range(80)) and len(flat) == 80
        assert every[rank] == list(shard.layer_ranges(80, world)[rank])
        # the timing reduction is the max over ranks
        assert tmax == 11.0
        # every rank computed the same unit placement on its own
        assert all_units[0] == all_units[1]


def _replicate_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # equal-shaped units one per rank (all-gather rounds) and odd ones
        # (broadcasts)
        names = ["embed", "layer0.q", "layer0.k", "layer1.q", "layer1.k", "lm_head", "norm"]
        shapes = {"embed": (7, 5), "layer0.q": (4, 6), "layer1.q": (4, 6), "layer0.k": (2, 6),
                  "layer1.k": (2, 6), "lm_head": (7, 5), "norm": (9,)}
        owner = {"embed": 0, "lm_head": 0, "layer0.q": 0, "layer1.q": 1, "layer0.k": 0,
                 "layer1.k": 1, "norm": 1}
        specs = {n: (shapes[n], torch.bfloat16, torch.device("cpu")) for n in names}

        def value(n):  # what the owner decoded
            g = torch.Generator().manual_seed(names.index(n))
            return torch.randn(shapes[n], generator=g).to(torch.bfloat16)

        mine = {n: value(n) for n in names if owner[n] == rank}
        got = shard.replicate_units(mine, owner, specs)
        ok = sorted(got) == sorted(names) and all(torch.equal(got[n], value(n)) for n in names)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_replicate_decoded_units():
    """The replicated-weights mode: every rank ends with every unit, bit for
    bit, whether it travelled in an all-gather round or a broadcast."""
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_replicate_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [ok for _, ok in res] == [True, True]



@pytest.mark.parametrize("arch", sorted(shard.ARCHS))
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_rank_units_cover_the_model_once(arch, world):
    units = shard.model_units(arch)
    names = [n for n, _, _ in units]
    assert len(names) == len(set(names))
    got = [shard.rank_units(arch, world, r) for r in range(world)]
    flat = sorted(n for g in got for n, _, _ in g)
    assert flat == sorted(names)
    ranges = shard.layer_ranges(shard.ARCHS[arch]["layers"], world)
    for r, g in enumerate(got):
        assert {l for _, _, l in g if l >= 0} <= set(ranges[r])


def test_model_sizes_match_the_architectures():
    tot = {a: sum(shard._numel(s) for _, s, _ in shard.model_units(a)) for a in shard.ARCHS}
    assert tot["llama2-70b"] == 68_976_648_192
    assert tot["llama3-8b"] == 8_030_261_248
