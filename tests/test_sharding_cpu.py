"""Multi-rank logic on CPU with the gloo backend (world size 2): head sharding
covers every unit exactly once, and the all-reduced per-rank losses (computed
by the oracle on each rank's shard) equal the single-process total."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from linearard_b200.sharding import allreduce_loss, partition_units, rel_head_units
from linearard_b200.synth import RelationConfig


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


CFG = RelationConfig("tiny_gqa", 1, 4, 2, 16, 40, 1e4)


def _unit_losses(units):
    from oracle import attn_kl_oracle as O
    from linearard_b200.synth import make_relations
    rels = make_relations(CFG, seed=3)
    out = 0.0
    for _, rel, h in units:
        s, t = rels[rel]
        a = s[:, h:h + 1].double().numpy()
        b = t[:, h:h + 1].double().numpy()
        out += O.oracle_attn_kl_align(a, a, b, b)[0]
    return out


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        units = partition_units(rel_head_units(CFG, layers=2), world, rank)
        local = torch.tensor(_unit_losses(units), dtype=torch.float64)
        total = allreduce_loss(local)
        q.put((rank, len(units), float(total)))
    finally:
        dist.destroy_process_group()


def test_partition_covers_every_unit_once():
    units = rel_head_units(CFG, layers=3)
    assert len(units) == 3 * (4 + 2 + 2)
    for world in (1, 2, 3, 4, 8):
        shards = [partition_units(units, world, r) for r in range(world)]
        flat = [u for s in shards for u in s]
        assert flat == units
        sizes = [len(s) for s in shards]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        partition_units(units, 2, 2)


def test_allreduce_loss_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = _unit_losses(rel_head_units(CFG, layers=2))
    for rank, n, total in res:
        assert n == 8
        assert abs(total - expect) <= 1e-9 * abs(expect)


def test_allreduce_is_noop_without_process_group():
    x = torch.tensor(3.5)
    assert allreduce_loss(x) is x
