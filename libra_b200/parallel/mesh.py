"""Rank mesh for TP x CP x EP x DP x PP (reference ``engine/train_parallel.py``).

Rank layout (fastest first): TP, CP, DP, PP - TP groups are consecutive ranks
so they stay inside one NVSwitch box; expert parallelism subdivides the DP
dimension (EP must divide DP).  Every rank calls ``dist.new_group`` for every
group in the same order, as torch.distributed requires.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

try:
    import torch.distributed as dist
except ModuleNotFoundError:  # pragma: no cover
    dist = None


@dataclass
class MeshCoords:
    tp: int
    cp: int
    dp: int
    pp: int
    ep: int


class ParallelMesh:
    def __init__(self, world_size: int, tp: int = 1, pp: int = 1, cp: int = 1, ep: int = 1,
                 dp: Optional[int] = None, create_groups: bool = True, backend: Optional[str] = None):
        if tp < 1 or pp < 1 or cp < 1 or ep < 1:
            raise ValueError("parallel sizes must be positive")
        base = tp * pp * cp
        if world_size % base:
            raise ValueError(f"world_size {world_size} is not divisible by tp*pp*cp={base}")
        self.world_size, self.tp, self.pp, self.cp = world_size, tp, pp, cp
        self.dp = dp if dp is not None else world_size // base
        if self.dp * base != world_size:
            raise ValueError(f"tp*cp*dp*pp = {self.dp * base} != world_size {world_size}")
        if self.dp % ep:
            raise ValueError(f"ep={ep} must divide dp={self.dp}")
        self.ep = ep
        self.groups: Dict[str, Dict[Tuple[int, ...], object]] = {}
        self._members: Dict[str, List[List[int]]] = {k: self._enumerate(k) for k in ("tp", "cp", "dp", "pp", "ep",
                                                                                    "edp", "mp")}
        if create_groups and dist is not None and dist.is_available() and dist.is_initialized():
            for kind, lists in self._members.items():
                self.groups[kind] = {}
                for ranks in lists:
                    self.groups[kind][tuple(ranks)] = dist.new_group(ranks, backend=backend)

    # ------------------------------------------------------------------ coordinates
    def coords(self, rank: int) -> MeshCoords:
        tp = rank % self.tp
        cp = (rank // self.tp) % self.cp
        dp = (rank // (self.tp * self.cp)) % self.dp
        pp = rank // (self.tp * self.cp * self.dp)
        return MeshCoords(tp, cp, dp, pp, dp % self.ep)

    def rank_of(self, tp: int = 0, cp: int = 0, dp: int = 0, pp: int = 0) -> int:
        return ((pp * self.dp + dp) * self.cp + cp) * self.tp + tp

    def _enumerate(self, kind: str) -> List[List[int]]:
        out = []
        if kind == "tp":
            for pp in range(self.pp):
                for dp in range(self.dp):
                    for cp in range(self.cp):
                        out.append([self.rank_of(t, cp, dp, pp) for t in range(self.tp)])
        elif kind == "cp":
            for pp in range(self.pp):
                for dp in range(self.dp):
                    for tp in range(self.tp):
                        out.append([self.rank_of(tp, c, dp, pp) for c in range(self.cp)])
        elif kind == "dp":
            for pp in range(self.pp):
                for cp in range(self.cp):
                    for tp in range(self.tp):
                        out.append([self.rank_of(tp, cp, d, pp) for d in range(self.dp)])
        elif kind == "pp":
            for dp in range(self.dp):
                for cp in range(self.cp):
                    for tp in range(self.tp):
                        out.append([self.rank_of(tp, cp, dp, p) for p in range(self.pp)])
        elif kind == "ep":  # consecutive DP ranks share experts
            for pp in range(self.pp):
                for cp in range(self.cp):
                    for tp in range(self.tp):
                        for blk in range(self.dp // self.ep):
                            out.append([self.rank_of(tp, cp, blk * self.ep + e, pp) for e in range(self.ep)])
        elif kind == "edp":  # expert-data-parallel: same expert shard across EP blocks
            for pp in range(self.pp):
                for cp in range(self.cp):
                    for tp in range(self.tp):
                        for e in range(self.ep):
                            out.append([self.rank_of(tp, cp, blk * self.ep + e, pp) for blk in range(self.dp // self.ep)])
        elif kind == "mp":  # model parallel = one DP replica (TP x CP x PP)
            for dp in range(self.dp):
                out.append(sorted(self.rank_of(t, c, dp, p) for p in range(self.pp) for c in range(self.cp)
                                  for t in range(self.tp)))
        return out

    def members(self, kind: str, rank: int) -> List[int]:
        for ranks in self._members[kind]:
            if rank in ranks:
                return ranks
        raise KeyError(rank)

    def group(self, kind: str, rank: int):
        return self.groups.get(kind, {}).get(tuple(self.members(kind, rank)))

    def is_pipeline_first(self, rank: int) -> bool:
        return self.coords(rank).pp == 0

    def is_pipeline_last(self, rank: int) -> bool:
        return self.coords(rank).pp == self.pp - 1

    def is_batch_source(self, rank: int) -> bool:
        """TP rank 0 of the first pipeline stage feeds data to its replica."""
        c = self.coords(rank)
        return c.tp == 0 and c.cp == 0 and c.pp == 0
