"""Who talks to whom in a core-attention-disaggregated deployment.

The union world is the AFD one: attention ranks ``0 .. A-1`` (one per data-parallel lane, attention TP 1),
then the model ranks ``A .. A+M-1`` (the expert ranks of the AFD topology). ``A`` is a multiple of ``M``;
model rank ``j`` serves the ``r = A / M`` consecutive lanes ``j*r .. j*r + r - 1``, its *peers*, and a lane's
position among the peers of its model rank is its *peer index*.

Prefill steps stay AFD steps (the attention ranks run the dense layers, the model ranks serve the experts);
in a decode step the roles turn: a model rank runs everything but the attention core for the rows of its
peers, and each peer keeps the KV cache and runs the attention core of its own rows.

Reference: python/minisgl/cad/groups.py:13-52 (CadRanks), python/minisgl/cad/layout.py (peers_of, model_of).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

from ..protocol import AfdTopology


class CadTopologyError(ValueError):
    pass


def check_topology(num_attn: int, num_model: int) -> None:
    if num_attn < 1 or num_model < 1:
        raise CadTopologyError("a CAD deployment needs at least one attention rank and one model rank")
    if num_attn % num_model:
        raise CadTopologyError(f"{num_attn} attention ranks cannot be shared evenly among {num_model} model ranks")


@dataclass(frozen=True)
class CadRanks:
    num_attn: int
    num_model: int

    def __post_init__(self):
        check_topology(self.num_attn, self.num_model)

    @staticmethod
    def of(topo: AfdTopology) -> "CadRanks":
        if topo.colocated:
            raise CadTopologyError("a colocated deployment has no attention core to move away")
        if topo.attn_tp != 1:
            raise CadTopologyError("CAD runs attention TP 1: a lane is one attention rank")
        return CadRanks(topo.attn_world, topo.mlp_world)

    @property
    def r(self) -> int:
        """Attention ranks per model rank."""
        return self.num_attn // self.num_model

    @property
    def world(self) -> int:
        return self.num_attn + self.num_model

    def role(self, rank: int) -> str:
        if not 0 <= rank < self.world:
            raise CadTopologyError(f"rank {rank} outside the world of {self.world}")
        return "attn" if rank < self.num_attn else "model"

    def model_index(self, rank: int) -> int:
        """Index of a model rank among the model ranks."""
        if self.role(rank) != "model":
            raise CadTopologyError(f"rank {rank} is an attention rank")
        return rank - self.num_attn

    def model_ranks(self) -> List[int]:
        return list(range(self.num_attn, self.world))

    def peers_of(self, model_index: int) -> List[int]:
        """Attention ranks (= lanes) served by a model rank, in peer order."""
        if not 0 <= model_index < self.num_model:
            raise CadTopologyError(f"model index {model_index} outside 0..{self.num_model - 1}")
        return list(range(model_index * self.r, (model_index + 1) * self.r))

    def model_of(self, attn_rank: int) -> int:
        """Union rank of the model rank that serves an attention rank."""
        if self.role(attn_rank) != "attn":
            raise CadTopologyError(f"rank {attn_rank} is a model rank")
        return self.num_attn + attn_rank // self.r

    def peer_index(self, attn_rank: int) -> int:
        self.model_of(attn_rank)
        return attn_rank % self.r
