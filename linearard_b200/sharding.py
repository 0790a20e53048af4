"""Work partitioning across GPUs for the relation-KL loss.

Every (relation, layer, batch, head) unit of the loss is independent: its
value is a sum over its own rows and its gradient touches only its own
[T, D] slices.  Multi-GPU runs therefore shard whole units (or whole
sequences) across ranks and exchange only the scalar loss -- plus, in
training, DDP's all-reduce of the LoRA gradients (``train.py:297``).  There is
no collective inside the data path.

All units of one workload cost the same (causal n^2 d each), so a contiguous
near-equal split is balanced.
"""
from __future__ import annotations

from typing import Sequence

import torch

__all__ = ["rel_head_units", "partition_units", "allreduce_loss", "sequence_seed"]


def rel_head_units(cfg, layers: int = 1) -> list[tuple[int, str, int]]:
    """(layer, relation, head) units of one sequence, relation-major order."""
    return [(layer, rel, h) for layer in range(layers) for rel in cfg.relations
            for h in range(cfg.heads(rel))]


def partition_units(units: Sequence, world: int, rank: int) -> list:
    """Contiguous near-equal share of ``units`` for ``rank`` (sizes differ by at
    most one; every unit lands on exactly one rank)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    n = len(units)
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return list(units[start:stop])


def allreduce_loss(loss: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of the per-rank scalar losses (the only exchange of the data path).
    A no-op when torch.distributed is not initialised."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return loss
    out = loss.detach().clone().reshape(1)
    dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out.reshape(())


def sequence_seed(base: int, rank: int) -> int:
    """Seed of the sequence a rank owns in weak-scaling runs (no scatter: each
    rank generates its own inputs)."""
    return base + 1000 * rank
