"""The CAD half of a worker process.

A worker process of an AFD deployment (`fastafd_b200.worker.main`) keeps serving AFD steps (prefill); when the
coordinator runs in CAD mode it also gets :class:`CadInitCmd` once and a :class:`CadStepCmd` per decode step.
`CadWorkerState` holds what those need on this rank: on an attention rank the window to its model rank and the
attention side bound to the worker's KV cache and page table; on a model rank (an expert rank of the AFD
topology) the dense weights, one window per peer, the token path, and the expert exchange among the model
ranks.

Between CPU processes a window's rows travel as gloo messages: "put rows, release flag" is one send, the
acquire-wait is the matching receive (bounded by the process group's timeout), so the step programs of
`cad/deploy.py` run unchanged with windows of this kind. Sends are asynchronous and are completed at the end of
the step, which keeps the two sides from blocking in a send towards each other. Between GPU processes the same
places are taken by the hop kernels over the peer-mapped fabric (`cad/gpu.py`); that wiring is not part of this
module.

Experts: model rank j holds the expert slice of expert rank j. In a decode step the model ranks gather each
other's routed rows, every rank applies its own experts to all of them, and a sum over the ranks gives each
rank the expert outputs of its own rows: every model rank is a dispatch source and an expert rank at once.

Reference: python/minisgl/cad/model_worker.py:52-188, python/minisgl/afd_attention_worker.py:1067-1171,
python/minisgl/cad/m2n_dual.py:107-153 (the dual-role round among the model ranks).
"""
from __future__ import annotations

import time
from typing import List, Optional

import torch
import torch.distributed as dist

from ..models.transformer import AttentionStage
from ..protocol import CadInitCmd, CadStepCmd, CadStepReply
from .deploy import CadAttentionSide, CadModelRank
from .program import check_balanced
from .ranks import CadRanks
from .runtime import CadLayout, CadWindow
from .tokens import CadTokenPath


class GlooWindow(CadWindow):
    """One side's end of the window between a model rank process and one of its attention rank processes."""

    def __init__(self, layout: CadLayout, dtype, peer_rank: int, peer_index: int, group=None):
        z = CadWindow.local(layout, dtype, "cpu")
        super().__init__(layout, z.qkv, z.o, z.flags, z.err)
        self.peer_rank, self.peer_index, self.group = peer_rank, peer_index, group
        self.bucket = 0
        self._sends: List[tuple] = []

    def _rows(self, kind: int, mb: int) -> torch.Tensor:
        lo = self.peer_index * self.bucket
        return (self.qkv if kind == 0 else self.o)[mb][lo:lo + self.bucket]

    def release(self, kind: int, layer: int, mb: int) -> None:
        rows = self._rows(kind, mb).clone()              # the buffer is reused by the next layer before the send ends
        self._sends.append((dist.isend(rows, dst=self.peer_rank, group=self.group), rows))

    def ready(self, kind: int, layer: int, mb: int) -> bool:
        dist.recv(self._rows(kind, mb), src=self.peer_rank, group=self.group)
        return True

    def end_step(self) -> None:
        for work, _rows in self._sends:
            work.wait()
        self._sends = []


class CadWorkerState:
    def __init__(self, engine, rank: int, group=None):
        self.engine, self.rank, self.group = engine, rank, group
        self.ranks = CadRanks.of(engine.topo)
        self.role = self.ranks.role(rank)
        self.side = None
        # every rank of the world creates the model ranks' group, in the same place of its start-up
        self.model_group = dist.new_group(self.ranks.model_ranks()) if self.ranks.num_model > 1 else None

    # ------------------------------------------------------------------ init
    def init(self, cmd: CadInitCmd) -> None:
        e, rk, cfg = self.engine, self.ranks, self.engine.cfg
        if e.device.type != "cpu":
            raise NotImplementedError("CAD worker processes run on CPU ranks; the GPU hop wiring is separate")
        if any(cfg.layer_type(i) != "full" for i in range(cfg.num_layers)):
            raise ValueError("CAD serves models whose layers all have full attention")
        check_balanced(cfg.num_layers, cmd.num_mb, rk.r)
        lay = CadLayout(cfg.num_layers, cmd.num_mb, rk.r * cmd.t_max, cfg.q_size, cfg.kv_size)
        if self.role == "attn":
            win = GlooWindow(lay, e.dtype, rk.model_of(self.rank), rk.peer_index(self.rank), self.group)
            self.side = CadAttentionSide(e.attn, win, rk.peer_index(self.rank))
            return
        j = rk.model_index(self.rank)
        stage = AttentionStage(cfg, e.device, e.dtype, 0, 1, None)        # the dense weights, as the attention ranks hold them
        e._attention_weight_init(e.checkpoint, e.seed, False)(stage)
        wins = [GlooWindow(lay, e.dtype, a, p, self.group) for p, a in enumerate(rk.peers_of(j))]
        self.side = _ModelRankOverGroup(cfg, stage, e.expert_stage, wins,
                                        CadTokenPath(rk.r, cmd.num_mb, cmd.t_max, cmd.table_rows, e.device),
                                        self.model_group, j, rk.num_model)

    # ------------------------------------------------------------------ one step
    def run(self, cmd: CadStepCmd) -> CadStepReply:
        if self.side is None:
            raise RuntimeError("CAD step before the CAD init command")
        t0 = time.perf_counter()
        gen = self.side.step(cmd)
        tokens: Optional[dict] = None
        try:
            while True:
                next(gen)                    # a window of this kind never reports "not ready": the receive blocks
        except StopIteration as fin:
            tokens = fin.value
        return CadStepReply(step_id=cmd.step_id, rank=self.rank, tokens=tokens or {}, err=0,
                            step_ms=(time.perf_counter() - t0) * 1e3)


class _ModelRankOverGroup(CadModelRank):
    """A model rank that holds one slice of the experts: the routed rows of all model ranks visit every slice."""

    def __init__(self, cfg, stage, experts, windows, tokens, group, index: int, size: int):
        super().__init__(cfg, stage, experts, windows, tokens)
        self.group, self.index, self.size = group, index, size

    def expert_rows(self, layer: int, x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return super().expert_rows(layer, x, idx)
        T = x.shape[0]
        xs = [torch.empty_like(x) for _ in range(self.size)]
        ids = [torch.empty_like(idx) for _ in range(self.size)]
        dist.all_gather(xs, x.contiguous(), group=self.group)
        dist.all_gather(ids, idx.contiguous(), group=self.group)
        rows = self.experts.run_experts_dense(layer, torch.cat(xs), torch.cat(ids))      # [K, size*T, H], own experts only
        dist.all_reduce(rows, group=self.group)
        return rows[:, self.index * T:(self.index + 1) * T].contiguous()
