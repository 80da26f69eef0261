"""A core-attention-disaggregated deployment inside one process: every rank is an object, the windows are plain
tensors that the two sides share, and a cooperative scheduler advances whichever rank's next task finds its
flags set. It is the transport behind :class:`fastafd_b200.cad.coordinator.CadCoordinator` for CPU runs and
tests, and it pins the protocol that separate processes follow: what each role does with a prefill step (an
AFD step) and with a decode step (its half of the CAD programs), what it answers, and what happens when a
flag never arrives.

Per decode step
  attention rank (`CadAttentionSide`): apply the plan's page grants, derive positions / KV slots / page-table
  rows of its micro-batches from its own request table, then for every full-attention layer and micro-batch
  wait for its q|k|v rows, store K and V, run the attention core and write the output rows into the model
  rank's window, release the o flag.
  model rank (`CadModelRank`): stage the step's rows (token or -1, request slot, position), embed, and run the
  model program: put q|k|v rows for each peer, wait for all peers' o rows, o_proj, norm, route, experts, next
  norm; final norm, LM head, greedy sample, keep every request's token in its slot.

Reference: python/minisgl/cad/attn_side.py:178-191, python/minisgl/cad/model_side.py:117-130,
python/minisgl/cad/model_worker.py:148-188, python/minisgl/afd_attention_worker.py:1143-1171.
"""
from __future__ import annotations

import time
from typing import Dict, Generator, List, Optional, Tuple

import torch

from .. import ops
from ..config import ModelConfig, RuntimeConfig
from ..models.transformer import AttentionStage, ExpertStage
from ..protocol import (AfdTopology, AgStepPlan, CadInitCmd, CadStepCmd, CadStepReply, EgStepPlan, EgStepReply,
                        WorkerFailure, WorkerReady)
from ..reference import ops_ref as ref
from ..worker.attention_worker import AttentionWorker
from ..worker.moe_client import LocalMoeClient
from .coordinator import CadTransport
from .program import attention_program, check_balanced, model_program
from .ranks import CadRanks
from .runtime import CadLayout, CadModelMath, CadWindow
from .tokens import CadTokenPath, tokens_by_peer, unpack_rows

Blocked = Tuple[str, int, int]      # what a side waits for: (flag kind, layer, micro-batch)


class DroppableWindow(CadWindow):
    """A window whose next release of one named flag can be withheld: the host-side way to make a peer's
    wait run out."""

    drop: Optional[Blocked] = None

    def release(self, kind: int, layer: int, mb: int) -> None:
        if self.drop == (("qkv", "o")[kind], layer, mb):
            self.drop = None
            return
        super().release(kind, layer, mb)


class CadAttentionSide:
    """The CAD half of an attention rank: KV cache, page table and attention core of one lane."""

    def __init__(self, worker: AttentionWorker, window: CadWindow, peer: int):
        self.w, self.win, self.peer = worker, window, peer
        self.cfg = worker.cfg

    def step(self, cmd: CadStepCmd) -> Generator[Blocked, None, None]:
        w, c, plan, B = self.w, self.cfg, cmd.plan, cmd.bucket
        if plan.phase != "decode" or plan.bucket != B:
            raise ValueError(f"CAD attention step {cmd.step_id}: phase {plan.phase}, bucket {plan.bucket} != {B}")
        self.win.begin_step(B)
        w.apply_grants(plan)
        w._stage_decode(plan)
        for mb in range(w.num_mb):
            w._prepare_decode_inputs(mb, B)
        D, Hq, Hkv = c.head_dim, c.num_q_heads, c.num_kv_heads
        lo = self.peer * B
        for t in attention_program(c.num_layers, w.num_mb):
            if t.kind == "pre":
                while not self.win.ready(0, t.layer, t.mb):
                    yield ("qkv", t.layer, t.mb)
                continue
            b, li = w.bufs[t.mb], w.model.full_index[t.layer]
            rows = self.win.qkv[t.mb][lo:lo + B]
            q = rows[:, :Hq * D].reshape(B, Hq, D)
            k = rows[:, Hq * D:(Hq + Hkv) * D].reshape(B, Hkv, D)
            v = rows[:, (Hq + Hkv) * D:].reshape(B, Hkv, D)
            loc = b.out_loc[:B].long()
            w.kv.k[li][loc] = k.to(w.kv.k.dtype)
            w.kv.v[li][loc] = v.to(w.kv.v.dtype)
            o = ops.decode_attention(q.contiguous(), w.kv.k[li], w.kv.v[li], b.page_table[:B], b.seq_lens[:B], Hq, Hkv, D,
                                     1, w.page_size, ref.softmax_scale(D))
            self.win.o[t.mb][lo:lo + B] = o.reshape(B, Hq * D).to(self.win.o.dtype)
            self.win.release(1, t.layer, t.mb)
        self.win.end_step()


class CadModelRank(CadModelMath):
    """The CAD half of a model rank: everything but the attention core, for the rows of its peers."""

    def __init__(self, cfg: ModelConfig, stage: AttentionStage, experts: ExpertStage, windows: List[CadWindow],
                 tokens: CadTokenPath):
        self.cfg, self.stage, self.experts, self.windows, self.tokens = cfg, stage, experts, windows, tokens
        self.r = len(windows)

    def step(self, cmd: CadStepCmd) -> Generator[Blocked, None, Dict[int, "torch.Tensor"]]:
        c, tok, B = self.cfg, self.tokens, cmd.bucket
        tok.bind(B)
        tok.stage(unpack_rows(cmd.rows))
        for w in self.windows:
            w.begin_step(B)
        ids, pos = tok.input_ids(), tok.positions()
        owner = torch.arange(self.r, device=ids.device).repeat_interleave(B)
        states = [self.embed_mb(ids[tok.mb_rows(m)], pos[tok.mb_rows(m)], owner) for m in range(tok.num_mb)]
        for t in model_program(c.num_layers, tok.num_mb):
            if t.kind == "hqkv":
                self._hqkv(t.layer, t.mb, states[t.mb], None, None, None)
            elif t.kind == "hpost":
                while not all(w.ready(1, t.layer, t.mb) for w in self.windows):
                    yield ("o", t.layer, t.mb)
                self._hpost_ffn(t.layer, t.mb, states[t.mb])
        tok.record(torch.cat([self.sample_mb(st) for st in states]))
        for w in self.windows:
            w.end_step()
        return tokens_by_peer(tok.out[:tok.rows].tolist(), self.r, tok.num_mb, B)


class CadLocalWorkers(CadTransport):
    """All ranks of a CAD deployment as objects of this process (CPU)."""

    def __init__(self, cfg: ModelConfig, rt: RuntimeConfig, topo: AfdTopology, *, seed: int = 0, device="cpu",
                 dtype=torch.float32):
        if any(cfg.layer_type(i) != "full" for i in range(cfg.num_layers)):
            raise ValueError("CAD serves models whose layers all have full attention")
        self.cfg, self.rt, self.topo, self.ranks = cfg, rt, topo, CadRanks.of(topo)
        self.device, self.dtype, self.seed = torch.device(device), dtype, seed
        from ..engine import resolve_checkpoint

        self.checkpoint = resolve_checkpoint(rt)       # a checkpoint directory, or None: random weights from the seed
        self.experts = ExpertStage(cfg, self.device, dtype, 0, 1)
        if self.checkpoint is None:
            self.experts.init_random(seed)
        else:
            from ..models.loader import load_expert_stage

            load_expert_stage(self.experts, self.checkpoint)
        self.workers = {a: AttentionWorker(cfg, rt, self.device, LocalMoeClient([self.experts]), dtype=dtype, rank=a,
                                           dp_lane=a, weight_init=self._init_dense)
                        for a in range(self.ranks.num_attn)}
        self.num_pages = min(w.num_pages for w in self.workers.values())
        self.attn_sides: Dict[int, CadAttentionSide] = {}
        self.model_sides: Dict[int, CadModelRank] = {}
        self._out: List[object] = []
        self.steps_run = 0

    def _init_dense(self, stage: AttentionStage) -> None:
        if self.checkpoint is None:
            stage.init_random(self.seed)
        else:
            from ..models.loader import load_attention_stage

            load_attention_stage(stage, self.checkpoint)

    # ------------------------------------------------------------------ CAD init
    def send_cad_init(self, cmd: CadInitCmd) -> None:
        cfg, rk = self.cfg, self.ranks
        check_balanced(cfg.num_layers, cmd.num_mb, rk.r)
        stage = AttentionStage(cfg, self.device, self.dtype, 0, 1, None)      # the model ranks' dense weights
        self._init_dense(stage)
        lay = CadLayout(cfg.num_layers, cmd.num_mb, rk.r * cmd.t_max, cfg.q_size, cfg.kv_size)
        for j, rank in enumerate(rk.model_ranks()):
            wins = []
            for p, a in enumerate(rk.peers_of(j)):
                z = CadWindow.local(lay, self.dtype, self.device)
                win = DroppableWindow(lay, z.qkv, z.o, z.flags, z.err)
                wins.append(win)
                self.attn_sides[a] = CadAttentionSide(self.workers[a], win, p)
            self.model_sides[rank] = CadModelRank(cfg, stage, self.experts, wins,
                                                  CadTokenPath(rk.r, cmd.num_mb, cmd.t_max, cmd.table_rows, self.device))
        self._out += [WorkerReady(rank=r, role="cad-" + rk.role(r)) for r in range(rk.world)]

    # ------------------------------------------------------------------ AFD steps (prefill)
    def send_step(self, step_id: int, ag_plans: Dict[int, Tuple[AgStepPlan, List[int]]], eg_plans: Dict[int, EgStepPlan]) -> None:
        for r, (plan, mb_tokens) in ag_plans.items():
            try:
                self._out.append(self.workers[r].run_step(plan, mb_tokens))
            except Exception as e:                                  # a worker that raises is a worker failure
                self._out.append(WorkerFailure(rank=r, error=repr(e)))
        for r in eg_plans:
            self._out.append(EgStepReply(step_id=step_id, rank=r))

    # ------------------------------------------------------------------ CAD steps (decode)
    def drop_next(self, attn_rank: int, flag: Blocked) -> None:
        """Withhold the next release of `flag` ("qkv" | "o", layer, micro-batch) on the window of `attn_rank`."""
        self.attn_sides[attn_rank].win.drop = flag

    def send_cad_step(self, step_id: int, attn_cmds: Dict[int, CadStepCmd], model_cmds: Dict[int, CadStepCmd]) -> None:
        t0 = time.perf_counter()
        gens = {r: self.attn_sides[r].step(c) for r, c in attn_cmds.items()}
        gens.update({r: self.model_sides[r].step(c) for r, c in model_cmds.items()})
        tokens: Dict[int, dict] = {}
        blocked: Dict[int, Blocked] = {}
        wins = [s.win for s in self.attn_sides.values()]
        while gens:
            before = sum(int(w.flags.sum()) for w in wins) - len(gens)
            for r in list(gens):
                try:
                    blocked[r] = next(gens[r])
                except StopIteration as fin:
                    tokens[r] = fin.value or {}
                    blocked.pop(r, None)
                    del gens[r]
            if gens and sum(int(w.flags.sum()) for w in wins) - len(gens) == before:
                break                   # a whole round, no flag moved and no rank finished: nobody can progress any more
        err = 0
        if gens:                        # the bounded wait of a GPU rank, decided at once here: set err, end the step
            err = 1
            for g in gens.values():
                g.close()
            for w in wins:
                w.set_err(1)
        ms = (time.perf_counter() - t0) * 1e3
        for r in attn_cmds:
            self._out.append(CadStepReply(step_id=step_id, rank=r, err=err, step_ms=ms))
        for r in model_cmds:
            self._out.append(CadStepReply(step_id=step_id, rank=r, tokens={} if err else tokens[r], err=err, step_ms=ms))
        self.last_blocked = dict(blocked) if err else {}
        for w in wins:                  # the epoch bump closes the step; after an abort it also voids stale flags
            w.err.zero_()
            w.bump_epoch()
        self.steps_run += 1

    def poll(self, timeout_s: float) -> List[object]:
        out, self._out = self._out, []
        return out
