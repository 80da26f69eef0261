"""Coordinator of a core-attention-disaggregated deployment.

Admission, lanes, page ledgers, prefill planning and the step window are those of the AFD coordinator; prefill
steps are AFD steps (the attention ranks run the dense layers, the model ranks serve the experts). A decode
step is planned by the same lane schedulers and then split by role:

* attention rank ``a`` gets its lane's plan (rows, KV lengths, page grants): it owns the KV cache and runs only
  the attention core of its rows;
* model rank ``j`` gets one row list for the lanes it serves (peer, micro-batch, index, request-table row,
  position, input token): it runs everything else and samples.

Planning ahead: a decode step may be launched while earlier decode steps are still out, because a model rank
keeps each request's last sampled token on the device (the row then carries -1 instead of a token). What
cannot be planned ahead is the first decode step of a request whose prefill reply is still out: its first
token was sampled on an attention rank and reaches the model rank through the host. Such a step waits.

A step whose workers report that a wait ran out is void: its requests are ended (reported as finished without
new tokens), everything else keeps running and the workers keep serving.

Reference: python/minisgl/afd_coordinator.py (the CAD init / step commands and the watchdog around them),
python/minisgl/cad/tokens.py:42-46 (host token or -1), python/minisgl/cad/model_worker.py:148-188.
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from ..coordinator import AfdCoordinator, CoordinatorError, WorkerTransport, _Inflight
from ..core import SamplingParams
from ..protocol import AgStepReply, CadInitCmd, CadStepCmd, CadStepReply, WorkerReady
from ..scheduler.buckets import per_mb_real, select_bucket
from .ranks import CadRanks
from .tokens import CadRow, host_token, pack_rows


class CadTransport(WorkerTransport):
    """A worker transport that also carries CAD commands."""

    def send_cad_init(self, cmd: CadInitCmd) -> None:
        raise NotImplementedError

    def send_cad_step(self, step_id: int, attn_cmds: Dict[int, CadStepCmd], model_cmds: Dict[int, CadStepCmd]) -> None:
        """attn_cmds: attention rank -> command with its plan; model_cmds: model rank -> command with its rows."""
        raise NotImplementedError


class CadCoordinator(AfdCoordinator):
    def __init__(self, cfg, rt, topo, transport: CadTransport, *, cad_init_timeout_s: Optional[float] = None, **kw):
        if rt.spec_block > 1:
            raise ValueError("CAD decode steps are plain decode steps: speculative decoding is off in this mode")
        super().__init__(cfg, rt, topo, transport, **kw)
        self.ranks = CadRanks.of(topo)
        self._dev_len: Dict[int, int] = {}      # uid -> KV length whose next input token sits in the model rank's slot
        self._cad_steps: Dict[int, dict] = {}   # step id -> {"err": int, "uids": [...]} of CAD steps in flight
        self.aborted_steps: List[int] = []
        # Every rank acknowledges the init command once its CAD state is built. Nothing waits for that up front
        # (commands reach a rank in order), but a decode step that gets no answer while ranks still owe the
        # acknowledgement is reported as what it is: an init that did not finish, with the ranks named.
        from .config import CadConfig

        self.cad_init_timeout_s = CadConfig.from_env().init_timeout_s if cad_init_timeout_s is None else cad_init_timeout_s
        self.cad_ready: set = set()
        self._cad_init_at = time.monotonic()
        table_rows = self.lanes[0].max_running + 1
        transport.send_cad_init(CadInitCmd(buckets=list(self.buckets), t_max=self.buckets[-1], table_rows=table_rows,
                                           num_mb=rt.num_mb, use_graph=rt.use_cuda_graph))

    # ------------------------------------------------------------------ admission
    def add_request(self, uid: int, input_ids: Sequence[int], sampling: SamplingParams) -> None:
        if not sampling.is_greedy:
            raise CoordinatorError("CAD samples greedily on the model ranks: temperature 0 / top_k 1 only")
        super().add_request(uid, input_ids, sampling)

    # ------------------------------------------------------------------ planning
    def _input_known(self, st) -> bool:
        """Can the next decode step of this request be launched now? Its input token (position = planned
        length) must be on the host or in the request's slot on the model rank."""
        pos = st.planned_len
        return pos < st.req.total_len or self._dev_len.get(st.req.uid) == pos

    def plan_and_launch(self) -> bool:
        if self._next_phase() != "decode":
            return super().plan_and_launch()          # prefill (an AFD step) or nothing to do
        if not all(self._input_known(st) for lane in self.lanes for st in lane.decodable()):
            if not self.inflight:
                raise CoordinatorError("a request waits for a token that no step in flight will deliver")
            return False
        sid = self.step_id
        self.step_id += 1
        nmb, rk = self.rt.num_mb, self.ranks
        real = max(l.decode_real() for l in self.lanes)
        bucket = select_bucket(per_mb_real(real, nmb), self.buckets)
        plans = [l.schedule_decode(sid, bucket, 1) if l.decode_real() else l.dummy_step(sid, "decode", bucket)
                 for l in self.lanes]
        rec = _Inflight(sid, "decode", bucket, time.perf_counter())
        rec.real = [sum(mb.num_real for mb in p.mbs) for p in plans]
        rows: Dict[int, List[CadRow]] = {m: [] for m in rk.model_ranks()}
        uids: List[Tuple[int, int]] = []
        for lane, (sched, plan) in enumerate(zip(self.lanes, plans)):
            rec.sizes[lane] = sum(len(mb.rows) for mb in plan.mbs)
            model, peer = rk.model_of(lane), rk.peer_index(lane)
            for m, slots in enumerate(sched.records[sid].slots):
                for i, (uid, _emits) in enumerate(slots):
                    if uid < 0:
                        continue
                    st = sched.states[uid]
                    pos = int(plan.mbs[m].seq_lens[i]) - 1
                    known = st.req.input_ids + st.req.output_ids
                    rows[model].append(CadRow(peer, m, i, int(plan.mbs[m].rows[i]), pos, host_token(known, pos)))
                    self._dev_len[uid] = pos + 1
                    uids.append((lane, uid))
        attn_cmds = {lane: CadStepCmd(step_id=sid, bucket=bucket, plan=plan) for lane, plan in enumerate(plans)}
        model_cmds = {m: CadStepCmd(step_id=sid, bucket=bucket, rows=pack_rows(q)) for m, q in rows.items()}
        rec.waiting_ag, rec.waiting_eg = set(attn_cmds), set(model_cmds)
        self._cad_steps[sid] = {"err": 0, "uids": uids}
        self.transport.send_cad_step(sid, attn_cmds, model_cmds)
        self.inflight.append(rec)
        if self.log_steps:
            self._step_log(f"[cad-step] launch step={sid} bucket={bucket} real={rec.real} inflight={len(self.inflight)}")
        return True

    # ------------------------------------------------------------------ completion
    def _on_reply(self, msg) -> None:
        if isinstance(msg, WorkerReady):
            if msg.role.startswith("cad-"):
                self.cad_ready.add(msg.rank)
            return
        if not isinstance(msg, CadStepReply):
            return super()._on_reply(msg)
        rec = next((r for r in self.inflight if r.step_id == msg.step_id), None)
        info = self._cad_steps.get(msg.step_id)
        if rec is None or info is None:
            return
        info["err"] = info["err"] or int(msg.err)
        self._note_latency(msg.rank, rec)
        if self.ranks.role(msg.rank) == "attn":
            rec.waiting_ag.discard(msg.rank)
            return
        rec.waiting_eg.discard(msg.rank)
        peers = self.ranks.peers_of(self.ranks.model_index(msg.rank))
        for p, toks in msg.tokens.items():
            lane = peers[int(p)]
            rec.replies[lane] = AgStepReply(step_id=msg.step_id, rank=lane, next_tokens=np.asarray(toks, np.int32))

    def collect(self, block: bool) -> bool:
        owing = sorted(set(range(self.ranks.world)) - self.cad_ready)
        if owing and self.inflight and self.inflight[0].step_id in self._cad_steps \
                and time.monotonic() - self._cad_init_at > self.cad_init_timeout_s:
            for m in self.transport.poll(0.0):
                self._on_reply(m)
            owing = sorted(set(range(self.ranks.world)) - self.cad_ready)
            if owing:
                self.failure = f"CAD init: ranks {owing} did not finish within {self.cad_init_timeout_s}s"
                raise CoordinatorError(self.failure)
        return super().collect(block)

    def _complete_oldest(self) -> None:
        info = self._cad_steps.pop(self.inflight[0].step_id, None)
        if info is None or not info["err"]:
            if info is not None:
                done = self.inflight[0]
                for lane in range(self.num_lanes):       # a void reply (no tokens for a lane) is a protocol error
                    if lane not in done.replies:
                        raise CoordinatorError(f"CAD step {done.step_id}: no tokens for lane {lane}")
            super()._complete_oldest()
            self._forget_finished()
            return
        # a wait ran out somewhere: the step is void and so is the state of the requests that were in it
        rec = self.inflight.popleft()
        self.aborted_steps.append(rec.step_id)
        items = []
        for lane, uid in info["uids"]:
            if uid in self.lanes[lane].states and not self.lanes[lane].states[uid].dead:
                self.lanes[lane].abort(uid)
                self.uid_lane.pop(uid, None)
                items.append((uid, [], True))
            self._dev_len.pop(uid, None)
        for lane, sched in enumerate(self.lanes):
            sched.complete(rec.step_id, np.zeros(rec.sizes[lane], np.int32), None)
        self._step_log(f"[cad-step] step={rec.step_id} aborted (err {info['err']}): {len(items)} requests ended")
        if items:
            self.on_tokens(items)

    def _forget_finished(self) -> None:
        if len(self._dev_len) > 4 * sum(len(l.states) for l in self.lanes) + 64:
            live = {uid for l in self.lanes for uid in l.states}
            self._dev_len = {u: n for u, n in self._dev_len.items() if u in live}
