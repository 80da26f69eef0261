"""Wire protocol between the coordinator and the AFD workers.

* :class:`AfdTopology` - rank arithmetic of the union world (attention ranks first, then
  expert ranks) with DP / TP / EP sizes.
* Step plans - what one worker has to execute in one step: :class:`AgStepPlan` for an
  attention rank (micro-batches with request rows, lengths, page grants, optional prompt
  tokens) and :class:`EgStepPlan` for an expert rank (token counts per lane only).
* Commands / replies and a pickle-free codec (msgpack with raw numpy buffers).

Reference: python/minisgl/afd_protocol.py (AfdTopology :19-166, AfdAGStepPlan :330-481,
AfdEGStepPlan :485-509, commands/replies :260-296,927-1000, codec :1023-1101).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import msgpack
import numpy as np


@dataclass(frozen=True)
class AfdTopology:
    """Union world = attention ranks [0, attn_world) then expert ranks [attn_world, world).

    Attention rank r belongs to DP lane r // attn_tp and is TP rank r % attn_tp. Expert
    ranks form mlp_dp replicas of mlp_tp * (mlp_ep / mlp_tp ...) - with pure EP (the
    benchmarked layout) every expert rank of a replica owns a contiguous expert range."""
    attn_dp: int = 1
    attn_tp: int = 1
    mlp_dp: int = 1
    mlp_tp: int = 1
    mlp_ep: int = 1
    colocated: bool = False      # one process / GPU holds both roles (world 1)

    def __post_init__(self):
        for name in ("attn_dp", "attn_tp", "mlp_dp", "mlp_tp", "mlp_ep"):
            if getattr(self, name) < 1:
                raise ValueError(f"{name} must be >= 1")
        mlp_world = self.mlp_world
        if self.attn_dp % self.mlp_dp != 0:
            raise ValueError("attn_dp must be a multiple of mlp_dp (every expert replica serves the same number of lanes)")
        if self.mlp_ep not in (1, self.mlp_tp, mlp_world // self.mlp_dp):
            raise ValueError("mlp_ep must be 1, mlp_tp or the size of one MLP replica")

    @property
    def attn_world(self) -> int:
        return self.attn_dp * self.attn_tp

    @property
    def mlp_replica(self) -> int:
        """Ranks in one MLP replica."""
        return max(self.mlp_tp, self.mlp_ep)

    @property
    def mlp_world(self) -> int:
        return self.mlp_dp * max(self.mlp_tp, self.mlp_ep)

    @property
    def world(self) -> int:
        return 1 if self.colocated else self.attn_world + self.mlp_world

    def is_attention(self, rank: int) -> bool:
        return 0 <= rank < self.attn_world

    def is_expert(self, rank: int) -> bool:
        return rank == 0 if self.colocated else self.attn_world <= rank < self.world

    def attn_lane(self, rank: int) -> int:
        return rank // self.attn_tp

    def attn_tp_rank(self, rank: int) -> int:
        return rank % self.attn_tp

    def attn_tp_group(self, lane: int) -> List[int]:
        return list(range(lane * self.attn_tp, (lane + 1) * self.attn_tp))

    def expert_index(self, rank: int) -> int:
        return rank - self.attn_world

    def expert_ranks(self) -> List[int]:
        return list(range(self.attn_world, self.world))

    def attention_ranks(self) -> List[int]:
        return list(range(self.attn_world))

    # ---- MLP data parallelism: mlp_dp replicas of the expert set; lane l uses replica l % mlp_dp
    def replica_of_lane(self, lane: int) -> int:
        return lane % self.mlp_dp

    def replica_of_expert_rank(self, rank: int) -> int:
        return self.expert_index(rank) // self.mlp_replica

    def expert_ranks_for(self, attn_rank: int) -> List[int]:
        """Expert ranks that serve the lane of `attn_rank` (one replica of the expert set)."""
        rep = self.replica_of_lane(self.attn_lane(attn_rank))
        first = self.attn_world + rep * self.mlp_replica
        return list(range(first, first + self.mlp_replica))

    def attention_ranks_for(self, expert_rank: int) -> List[int]:
        """Attention ranks (dispatch sources) whose lanes are served by the replica of `expert_rank`."""
        rep = self.replica_of_expert_rank(expert_rank)
        return [r for r in range(self.attn_world) if self.replica_of_lane(self.attn_lane(r)) == rep]

    def dispatch_sources(self) -> List[int]:
        """Attention ranks that push tokens into the experts. After the TP all-reduce every
        TP rank of a lane holds the same hidden states, so only TP rank 0 of each lane
        dispatches (the reference makes every attention worker a source,
        python/minisgl/afd_worker_base.py:571; de-duplicating cuts N2M/M2N traffic by attn_tp)."""
        return [lane * self.attn_tp for lane in range(self.attn_dp)]

    def ep_rank(self, rank: int) -> int:
        return self.expert_index(rank) % self.mlp_replica

    @staticmethod
    def for_world(world: int, attn_tp: int = 1, attn_gpus: int = 0) -> "AfdTopology":
        """Split `world` GPUs into attention and expert GPUs: `attn_gpus` attention GPUs (0 = half
        of them) in DP lanes of `attn_tp`, the rest expert-parallel. World 1 = colocated."""
        if world == 1:
            return AfdTopology(colocated=True)
        n_attn = attn_gpus if attn_gpus > 0 else world // 2
        if not 0 < n_attn < world or n_attn % attn_tp != 0:
            raise ValueError(f"cannot place {n_attn} attention GPUs (TP {attn_tp}) in a world of {world}")
        return AfdTopology(attn_dp=n_attn // attn_tp, attn_tp=attn_tp, mlp_dp=1, mlp_tp=1, mlp_ep=world - n_attn)


def validate_parallel_args(topo: AfdTopology, num_experts: int, num_q_heads: int, num_kv_heads: int,
                           linear_k_heads: int = 0, linear_v_heads: int = 0) -> None:
    """Mutual divisibility rules (python/minisgl/server/args.py:135-180). `linear_*_heads`: head counts of the
    linear-attention layers of a hybrid model (0: none); they are sharded by heads like the attention heads."""
    for name, n in (("linear-attention key", linear_k_heads), ("linear-attention value", linear_v_heads)):
        if n and n % topo.attn_tp:
            raise ValueError(f"attn_tp={topo.attn_tp} does not divide {n} {name} heads")
    if num_q_heads % topo.attn_tp:
        raise ValueError(f"attn_tp={topo.attn_tp} does not divide {num_q_heads} query heads")
    if num_kv_heads % topo.attn_tp and topo.attn_tp % num_kv_heads:
        raise ValueError(f"attn_tp={topo.attn_tp} incompatible with {num_kv_heads} kv heads")
    if topo.mlp_ep > num_experts:
        raise ValueError("more expert ranks than experts")


# ------------------------------------------------------------------------- plans
@dataclass
class MicroBatchPlan:
    """One micro-batch of one attention lane.

    decode : `rows` are token-pool / page-table rows (padding rows = the lane's dummy row),
             `seq_lens` the KV length after this step's token; the input token is read on the
             device from the token pool at position seq_len - 1.
    prefill: additionally `input_ids` (concatenated new tokens) and `extend_lens` (new tokens
             per request; seq_len - extend_len tokens are already cached)."""
    rows: np.ndarray                      # int32 [B]
    seq_lens: np.ndarray                  # int32 [B]
    num_real: int = 0
    input_ids: Optional[np.ndarray] = None        # int32 [sum(extend_lens)]
    extend_lens: Optional[np.ndarray] = None      # int32 [B]
    sample_rows: Optional[np.ndarray] = None      # bool [B]: request finishes its prompt this step

    @property
    def is_prefill(self) -> bool:
        return self.extend_lens is not None

    @property
    def num_tokens(self) -> int:
        return int(self.extend_lens.sum()) if self.is_prefill else len(self.rows)


@dataclass
class AgStepPlan:
    step_id: int
    phase: str                            # "prefill" | "decode" | "verify"
    bucket: int                           # padded tokens per micro-batch (decode graph size)
    mbs: List[MicroBatchPlan] = field(default_factory=list)
    # page grants: (row, first_page_slot, page_ids...) flattened
    grant_rows: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))
    grant_slots: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))
    grant_pages: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))
    free_rows: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))
    # sampling (per micro-batch row, concatenated over mbs); empty = all greedy
    temperatures: Optional[np.ndarray] = None
    top_ks: Optional[np.ndarray] = None
    top_ps: Optional[np.ndarray] = None
    spec_block: int = 0


@dataclass
class EgStepPlan:
    step_id: int
    phase: str
    tokens_per_mb: List[int] = field(default_factory=list)   # tokens each source pushes, per lane
    num_layers_moe: int = 0


@dataclass
class RunStepCmd:
    plan: Any
    mb_tokens: Optional[List[int]] = None    # tokens every source sends per micro-batch (prefill padding)


@dataclass
class StopCmd:
    reason: str = ""


@dataclass
class AgStepReply:
    step_id: int
    rank: int
    next_tokens: np.ndarray               # int32, concatenated over mbs (bucket-padded for decode)
    status: int = 0
    step_ms: float = 0.0
    accepted: Optional[np.ndarray] = None   # spec decode: emitted counts per request


@dataclass
class EgStepReply:
    step_id: int
    rank: int
    status: int = 0
    step_ms: float = 0.0


@dataclass
class WorkerReady:
    rank: int
    role: str
    num_pages: int = 0
    info: Dict[str, Any] = field(default_factory=dict)


@dataclass
class WorkerFailure:
    rank: int
    error: str


# ---- core-attention disaggregation: decode steps with the roles turned (cad/coordinator.py)
@dataclass
class CadInitCmd:
    """Sent once to every rank before the first CAD step: the decode buckets, the largest bucket, the rows
    of a lane's request table (with its padding row) and the micro-batches per step."""
    buckets: List[int]
    t_max: int
    table_rows: int
    num_mb: int
    use_graph: bool = True


@dataclass
class CadStepCmd:
    """One decode step. An attention rank gets its lane's `plan` (rows, lengths, page grants: the KV side of
    the step); a model rank gets `rows`, int32 [n, 6] as cad.tokens.pack_rows lays them out."""
    step_id: int
    bucket: int
    plan: Optional[AgStepPlan] = None
    rows: Optional[np.ndarray] = None


@dataclass
class CadStepReply:
    """`tokens`: peer index -> sampled tokens of that peer's lane in the lane scheduler's order (model ranks
    only). `err` != 0: a wait ran out, the step's result is void and the rank keeps serving."""
    step_id: int
    rank: int
    tokens: Dict[int, np.ndarray] = field(default_factory=dict)
    err: int = 0
    step_ms: float = 0.0


_TYPES = {c.__name__: c for c in (MicroBatchPlan, AgStepPlan, EgStepPlan, RunStepCmd, StopCmd, AgStepReply,
                                  EgStepReply, WorkerReady, WorkerFailure, CadInitCmd, CadStepCmd, CadStepReply)}


def _enc(o: Any) -> Any:
    if isinstance(o, np.ndarray):
        return {"__nd__": True, "d": o.dtype.str, "s": list(o.shape), "b": o.tobytes()}
    if isinstance(o, (np.integer,)):
        return int(o)
    if isinstance(o, (np.floating,)):
        return float(o)
    if type(o).__name__ in _TYPES:
        return {"__t__": type(o).__name__, "f": {k: _enc(v) for k, v in o.__dict__.items()}}
    if isinstance(o, (list, tuple)):
        return [_enc(v) for v in o]
    if isinstance(o, dict):
        return {k: _enc(v) for k, v in o.items()}
    return o


def _dec(o: Any) -> Any:
    if isinstance(o, dict):
        if o.get("__nd__"):
            return np.frombuffer(o["b"], dtype=np.dtype(o["d"])).reshape(o["s"]).copy()
        if "__t__" in o:
            return _TYPES[o["__t__"]](**{k: _dec(v) for k, v in o["f"].items()})
        return {k: _dec(v) for k, v in o.items()}
    if isinstance(o, list):
        return [_dec(v) for v in o]
    return o


def encode(msg: Any) -> bytes:
    """Serialise a command / reply: msgpack with tensors as raw buffers (no pickle)."""
    return msgpack.packb(_enc(msg), use_bin_type=True)


def decode(data: bytes) -> Any:
    return _dec(msgpack.unpackb(data, raw=False, strict_map_key=False))
