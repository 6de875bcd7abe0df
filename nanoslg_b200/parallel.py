"""Parallel topology and the TP collectives used on the per-layer path.

Same surface and rank layout as nanoslg/parallel.py:15-184, 229-255: rank =
pp_rank * tp_size + tp_rank, TP groups are contiguous ranks, PP groups stride by
tp_size, layers split by ``get_layers_for_pp_rank``.  The RowParallel all-reduce and the
LM-head all-gather stay NCCL collectives (over NVLink on a B200 node).
"""
from dataclasses import dataclass
from enum import Enum
from typing import Dict, List, Optional

import torch
import torch.distributed as dist


class ParallelMode(Enum):
    PIPELINE = "pipeline"
    TENSOR = "tensor"
    HYBRID = "hybrid"
    DATA = "data"


@dataclass
class ParallelConfig:
    mode: ParallelMode
    world_size: int
    tp_size: int = 1
    pp_size: int = 1
    pp_layer_splits: Dict[int, List[int]] = None

    def __post_init__(self):
        if self.mode == ParallelMode.PIPELINE:
            self.tp_size, self.pp_size = 1, self.world_size
        elif self.mode == ParallelMode.TENSOR:
            self.tp_size, self.pp_size = self.world_size, 1
        elif self.mode == ParallelMode.HYBRID:
            if self.tp_size * self.pp_size != self.world_size:
                raise ValueError(f"TP({self.tp_size}) * PP({self.pp_size}) != "
                                 f"world_size({self.world_size})")

    def get_tp_rank(self, rank):
        return rank % self.tp_size

    def get_pp_rank(self, rank):
        return rank // self.tp_size

    def get_tp_group_ranks(self, rank):
        pp = self.get_pp_rank(rank)
        return [pp * self.tp_size + i for i in range(self.tp_size)]

    def get_pp_group_ranks(self, rank):
        tp = self.get_tp_rank(rank)
        return [i * self.tp_size + tp for i in range(self.pp_size)]


class ParallelContext:
    """Process-wide singleton holding this rank's TP/PP coordinates and groups."""
    _instance: Optional["ParallelContext"] = None

    def __init__(self, config: ParallelConfig, rank: int, device=None):
        self.config = config
        self.rank = rank
        self.device = torch.device(device) if device is not None else torch.device(f"cuda:{rank}")
        self.tp_rank = config.get_tp_rank(rank)
        self.pp_rank = config.get_pp_rank(rank)
        self.tp_group = None
        self.pp_group = None
        self._initialized = False

    @classmethod
    def initialize(cls, config, rank, device=None):
        cls._instance = cls(config, rank, device)
        return cls._instance

    @classmethod
    def get(cls):
        return cls._instance

    def setup_groups(self):
        """Creates the TP and PP groups; every rank takes part in every new_group call."""
        if self._initialized:
            return
        tp, pp = self.config.tp_size, self.config.pp_size
        if tp > 1:
            for p in range(pp):
                ranks = [p * tp + i for i in range(tp)]
                g = dist.new_group(ranks)
                if self.rank in ranks:
                    self.tp_group = g
        if pp > 1:
            for t in range(tp):
                ranks = [i * tp + t for i in range(pp)]
                g = dist.new_group(ranks)
                if self.rank in ranks:
                    self.pp_group = g
        self._initialized = True

    @property
    def is_first_pp_stage(self):
        return self.pp_rank == 0

    @property
    def is_last_pp_stage(self):
        return self.pp_rank == self.config.pp_size - 1

    @property
    def is_tp_master(self):
        return self.tp_rank == 0

    def get_pp_prev_rank(self):
        return None if self.pp_rank == 0 else (self.pp_rank - 1) * self.config.tp_size + self.tp_rank

    def get_pp_next_rank(self):
        if self.pp_rank == self.config.pp_size - 1:
            return None
        return (self.pp_rank + 1) * self.config.tp_size + self.tp_rank


def get_parallel_context() -> ParallelContext:
    ctx = ParallelContext.get()
    if ctx is None:
        raise RuntimeError("ParallelContext not initialized")
    return ctx


def all_reduce_tp(tensor, op=dist.ReduceOp.SUM):
    """In-place SUM all-reduce over the TP group (parallel.py:167-172)."""
    ctx = ParallelContext.get()
    if ctx and ctx.config.tp_size > 1 and ctx.tp_group is not None:
        dist.all_reduce(tensor, op=op, group=ctx.tp_group)
    return tensor


def all_gather_tp(tensor, dim=-1):
    """All-gather over the TP group, concatenated along ``dim`` (parallel.py:175-184)."""
    ctx = ParallelContext.get()
    if ctx is None or ctx.config.tp_size == 1:
        return tensor
    parts = [torch.empty_like(tensor) for _ in range(ctx.config.tp_size)]
    dist.all_gather(parts, tensor.contiguous(), group=ctx.tp_group)
    return torch.cat(parts, dim=dim)


def get_layers_for_pp_rank(total_layers: int, pp_size: int, pp_rank: int) -> List[int]:
    """Contiguous, near-equal layer split (parallel.py:247-255)."""
    per, rem = divmod(total_layers, pp_size)
    start = pp_rank * per + min(pp_rank, rem)
    return list(range(start, start + per + (1 if pp_rank < rem else 0)))
